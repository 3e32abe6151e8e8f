"""Parity at the shapes and with the generators the benchmark runs.

The forward kernel is persistent (one CTA per SM, each CTA streaming its
work items (b, h, q-tile) as one sequence of live tiles), so a problem with
far more items than SMs exercises what a small case never reaches: the
second Q slot, the alternating O buffers, the epilogue two items ahead, and
the list prefetch across item boundaries. These cases run many items per
CTA, items with more than 32 live tiles (S = 8192), the benchmark's
multi-parent FK generator (up to 2 parents per row), and the full
B=32, S=1024, H=8, Dh=32 shape, and compare o, lse, dq, dk and dv with the
float64 oracle head by head (confluence/confluence/layers.py:82-97 and its
autodiff), and the tile plans bit for bit (model.py:201-264).
"""
import numpy as np
import pytest

from oracle import rt_oracle as orc
from rt_cases import TOL_GRAD_ROW, TOL_LSE, TOL_OUT, Case, from_bf16_tensor, per_head_errors

pytestmark = pytest.mark.gpu


def long_context_gen(seed, b, s):
    """The benchmark's long-context generator: 24 tables of 4-16 cells, up to
    two FK parents per row (each with p = 0.9), 5% trailing padding."""
    return (seed, b, s, 24, 4, 16, 0.9, 0.05, None, None, 2)


def short_context_gen(seed, b):
    """The B=32, S=1024 workload's generator: 6 tables of 4-16 cells, one FK
    parent with p = 0.7, 10% padding."""
    return (seed, b, 1024, 6, 4, 16, 0.7, 0.10)


def run_and_check(c, bwd=True):
    from tributary_b200.attention import attention_bwd, attention_fwd, device_status
    o, lse = attention_fwd(c.qd, c.kd, c.vd, c.plan, c.scale)
    got = [o]
    if bwd:
        got += list(attention_bwd(c.qd, c.kd, c.vd, o, lse, c.dod, c.plan, c.scale))
    assert device_status() == 0
    lse_got = lse.cpu().numpy()
    ref = c.oracle_by_head(bwd=bwd)
    errs = {}
    for name, g, r in zip(("o", "dq", "dk", "dv"), got, (ref[0],) + ref[2:]):
        gv = from_bf16_tensor(g)
        assert np.isfinite(gv).all(), name
        errs[name] = per_head_errors(gv, r)
    errs["lse"] = float(np.abs(lse_got - ref[1]).max())
    print({k: v for k, v in errs.items()})
    for name, v in errs.items():
        if name == "lse":
            assert v < TOL_LSE, (name, v)
        else:
            assert v[0] < TOL_OUT and v[1] < (TOL_OUT if name == "o" else TOL_GRAD_ROW), (name, v)
    return errs


@pytest.mark.parametrize("kind", [0, 1, 2, 3], ids=["column", "feature", "neighbor", "full"])
def test_many_items_per_cta_long_context(cuda_lib, kind):
    """B=2, H=16, S=4096, Dh=64: 1024 work items, about 7 per forward CTA."""
    c = Case(long_context_gen(81, 2, 4096), kind, h=16, dh=64, seed=810 + kind)
    assert c.b * c.h * c.plan.tiles >= 6 * 148
    run_and_check(c)


@pytest.mark.parametrize("kind", [1, 3], ids=["feature", "full"])
def test_long_items_s8192(cuda_lib, kind):
    """S = 8192: a dense item has 64 live key tiles, past the 32 list entries
    the forward's producer prefetches per item (the feature kind's items reach
    about 28)."""
    c = Case(long_context_gen(82, 1, 8192), kind, h=2, dh=64, seed=820 + kind)
    n_ptr, _ = c.plan.q2k()
    assert int(np.diff(n_ptr.cpu().numpy()).max()) > (32 if kind == 3 else 16)
    run_and_check(c)


@pytest.mark.parametrize("kind", [0, 1, 2, 3], ids=["column", "feature", "neighbor", "full"])
def test_short_context_full_shape(cuda_lib, kind):
    """B=32, S=1024, H=8, Dh=32 (2048 work items)."""
    c = Case(short_context_gen(83, 32), kind, h=8, dh=32, seed=830 + kind)
    run_and_check(c)


@pytest.mark.parametrize("kind", [0, 1, 2, 3], ids=["column", "feature", "neighbor", "full"])
def test_tile_plan_benchmark_batch(cuda_lib, kind):
    """The prepass on the benchmark's own batch shape and generator: B=8,
    S=4096, multi-parent fk_adj, 256 (sample, q-tile) rows in the list scan."""
    from test_tile_plan_gpu import check_plan, to_dev
    bt = orc.make_batch(*long_context_gen(84, 8, 4096))
    assert bt["fk_adj"].sum(axis=2).max() >= 2  # some row has two parents
    check_plan(bt, kind, to_dev(bt))


@pytest.mark.parametrize("kind", [1, 2], ids=["feature", "neighbor"])
def test_tile_plan_rows_past_shared_memory(cuda_lib, kind):
    """S = 8192 with 1-3 cells per row: more than 2048 rows, so a query row's
    packed fk row exceeds the 64 words the prepass stages in shared memory and
    is read from global memory instead."""
    from test_tile_plan_gpu import check_plan, to_dev
    bt = orc.make_batch(85, 1, 8192, 5, 1, 3, 0.9, 0.02, None, None, 2)
    assert bt["fk_adj"].shape[1] > 64 * 32
    check_plan(bt, kind, to_dev(bt))


def test_attention_rows_past_shared_memory(cuda_lib):
    """Attention on the > 2048-row batch above (feature kind), forward and
    backward against the oracle."""
    c = Case((85, 1, 8192, 5, 1, 3, 0.9, 0.02, None, None, 2), 1, h=2, dh=64, seed=851)
    run_and_check(c)
