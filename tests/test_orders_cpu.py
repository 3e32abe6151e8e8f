"""Cell orderings (rt_column_order, rt_rcm_order) and the synthetic batch
generator against the oracle's restatement of headwater/src/sampler.rs:
655-784 -- bit-exact, on generator batches and on adversarial FK graphs
(dense, cyclic, self loops, isolated rows, row ids past max_rows). Host code
only: runs without a GPU."""
import ctypes

import numpy as np
import pytest

from oracle import rt_oracle as orc
from tributary_b200 import _lib, batch as rb

CONFIGS = [
    # (seed, B, S, tables, lo, hi, p_fk, pad, max_parents)
    (1, 3, 256, 3, 4, 8, 0.6, 0.05, 1),
    (2, 2, 1024, 6, 4, 16, 0.7, 0.10, 1),
    (3, 2, 777, 24, 4, 16, 0.9, 0.05, 2),
    (4, 1, 64, 1, 1, 1, 1.0, 0.0, 3),
]


@pytest.mark.parametrize("cfg", CONFIGS)
def test_generator_matches_oracle(cfg):
    seed, B, S, t, lo, hi, p, pad, mp = cfg
    want = orc.make_batch(seed, B, S, t, lo, hi, p, pad, max_parents=mp)
    got = rb.make_batch(seed, B, S, t, lo, hi, p, pad, max_parents=mp)
    assert set(want) == set(got)
    for k in want:
        assert got[k].dtype == want[k].dtype, k
        np.testing.assert_array_equal(got[k], want[k], err_msg=k)


def _adversarial(seed, S, R):
    rng = np.random.default_rng(seed)
    fk = (rng.random((R, R)) < rng.uniform(0.02, 0.3)).astype(np.uint8)
    np.fill_diagonal(fk, rng.integers(0, 2, R).astype(np.uint8))  # self loops are dropped
    fk[rng.integers(0, R, 3)] = 0  # isolated rows
    rows = rng.integers(0, R + 3, S).astype(np.uint16)  # some ids past max_rows
    pad = (rng.random(S) < 0.1).astype(np.uint8)
    col = rng.integers(0, 9, S).astype(np.int32)
    return fk, rows, pad, col


@pytest.mark.parametrize("seed", range(8))
def test_orders_match_oracle_on_adversarial_graphs(seed):
    S, R = 300, 40
    fks, rows, pads, cols = zip(*(_adversarial(100 * seed + b, S, R) for b in range(3)))
    fk, rows, pad, col = (np.stack(x) for x in (fks, rows, pads, cols))
    got_col = rb.column_order(col, pad)
    got_out = rb.rcm_order(fk, rows, pad, True)
    got_in = rb.rcm_order(fk, rows, pad, False)
    for b in range(3):
        np.testing.assert_array_equal(got_col[b], orc.compute_col_perm(col[b], pad[b]))
        np.testing.assert_array_equal(got_out[b], orc.compute_rcm_perm(fk[b], rows[b], pad[b], True))
        np.testing.assert_array_equal(got_in[b], orc.compute_rcm_perm(fk[b], rows[b], pad[b], False))
        for p in (got_col[b], got_out[b], got_in[b]):  # every order is a permutation
            np.testing.assert_array_equal(np.sort(p), np.arange(S, dtype=np.uint16))


def test_orders_reject_bad_arguments():
    lib = _lib.load()
    out = np.zeros(4, dtype=np.uint16)
    ok = np.zeros(4, dtype=np.int32)
    p = ctypes.c_void_p(out.ctypes.data)
    assert lib.rt_column_order(None, None, 1, 4, p) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_column_order(ctypes.c_void_p(ok.ctypes.data), p, 1, 70000, p) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_rcm_order(None, p, p, 1, 4, 2, 1, p) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_rcm_order(None, None, None, 0, 0, 0, 1, None) == _lib.RT_OK  # empty batch: no-op
