"""Prepass kernel parity: tile bitmaps, tile lists and per-tile element bits
must equal the oracle bit for bit (the oracle's masks are pinned to the
reference's build_attention_masks by tests/test_oracle.py)."""
import numpy as np
import pytest

from conftest import golden_files, load_golden
from oracle import rt_oracle as orc

pytestmark = pytest.mark.gpu

CASES = {
    "cfgA": (31, 4, 256, 3, 4, 8, 0.6, 0.05),
    "ragged_s200": (32, 2, 200, 4, 2, 9, 0.8, 0.2),
    "ragged_s1000": (33, 2, 1000, 6, 4, 16, 0.7, 0.1),
    "single_token": (34, 1, 1, 1, 1, 1, 0.0, 0.0),
    "all_padding_tail": (35, 1, 384, 2, 3, 5, 0.9, 0.7),
    "cfgB_slice": (36, 2, 1024, 6, 4, 16, 0.7, 0.1),
    "many_rows_s2048": (37, 1, 2048, 3, 1, 3, 0.9, 0.0),
}


def to_dev(bt):
    import torch
    dev = torch.device("cuda:0")
    out = {}
    for k, v in bt.items():
        v = np.ascontiguousarray(v)
        if v.dtype == np.uint16:
            out[k] = torch.from_numpy(v.view(np.int16)).to(dev)
        else:
            out[k] = torch.from_numpy(v).to(dev)
    return out


def check_plan(bt, kind, dev_bt, perm=None):
    from tributary_b200.attention import build_tile_plan
    if perm is None:
        perm = orc.perm_for_kind(bt, kind)
    import torch
    perm_d = torch.from_numpy(np.ascontiguousarray(perm).view(np.int16)).cuda()
    plan = build_tile_plan(perm_d, dev_bt["seq_row_ids"], dev_bt["column_ids"],
                           dev_bt["is_padding"], dev_bt["fk_adj"], kind)
    torch.cuda.synchronize()
    mp = orc.permute_mask(orc.mask_for_kind(kind, bt["seq_row_ids"], bt["fk_adj"],
                                            bt["column_ids"], bt["is_padding"]), perm)
    live_ref, full_ref = orc.tile_bitmaps(mp)
    np.testing.assert_array_equal(plan.live_bits().cpu().numpy().view(np.uint32), live_ref)
    np.testing.assert_array_equal(plan.full_bits().cpu().numpy().view(np.uint32), full_ref)
    q2k_ptr, q2k_idx, k2q_ptr, k2q_idx = orc.tile_lists(mp)
    gp, gi = plan.q2k()
    gp = gp.cpu().numpy()
    np.testing.assert_array_equal(gp, q2k_ptr)
    np.testing.assert_array_equal(gi.cpu().numpy()[:gp[-1]], q2k_idx)
    gp, gi = plan.k2q()
    gp = gp.cpu().numpy()
    np.testing.assert_array_equal(gp, k2q_ptr)
    np.testing.assert_array_equal(gi.cpu().numpy()[:gp[-1]], k2q_idx)
    assert plan.nnz() == int(q2k_ptr[-1])
    # element bits, only where the kernels read them: live and not fully live
    live, full = orc.tile_occupancy(mp)
    partial = live & ~full
    words = orc.tile_mask_words(mp)
    words_t = orc.tile_mask_words_t(mp)
    g = plan.tile_masks().cpu().numpy().view(np.uint32)
    gt = plan.tile_masks(transposed=True).cpu().numpy().view(np.uint32)
    np.testing.assert_array_equal(g[partial], words[partial])
    np.testing.assert_array_equal(gt[np.swapaxes(partial, 1, 2)],
                                  words_t[np.swapaxes(partial, 1, 2)])
    return plan


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("kind", [0, 1, 2, 3], ids=["column", "feature", "neighbor", "full"])
def test_tile_plan_bit_exact(cuda_lib, name, kind):
    bt = orc.make_batch(*CASES[name])
    check_plan(bt, kind, to_dev(bt))


@pytest.mark.parametrize("path", golden_files("masks"), ids=lambda p: p.split("/")[-1])
def test_tile_plan_on_reference_fixtures(cuda_lib, path):
    g = load_golden(path)
    bt = {k: g[k] for k in ("seq_row_ids", "column_ids", "is_padding", "fk_adj",
                            "col_perm", "out_perm", "in_perm")}
    dev_bt = to_dev(bt)
    for kind in range(4):
        check_plan(bt, kind, dev_bt)


def test_row_ids_beyond_R_are_clamped(cuda_lib):
    """jax gathers clamp out-of-range indices; the prepass does the same."""
    bt = orc.make_batch(38, 1, 256, 3, 2, 6, 0.8, 0.0)
    bt = {k: v.copy() for k, v in bt.items()}
    r = bt["fk_adj"].shape[1]
    bt["seq_row_ids"][0, 10:14] = r + 5
    clamped = {k: v.copy() for k, v in bt.items()}
    clamped["seq_row_ids"][0, 10:14] = r - 1
    import torch
    for kind in (1, 2):
        perm = orc.perm_for_kind(clamped, kind)
        plan = check_plan(clamped, kind, to_dev(clamped))
        dev_bt = to_dev(bt)
        perm_d = torch.from_numpy(np.ascontiguousarray(perm).view(np.int16)).cuda()
        from tributary_b200.attention import build_tile_plan
        p2 = build_tile_plan(perm_d, dev_bt["seq_row_ids"], dev_bt["column_ids"],
                             dev_bt["is_padding"], dev_bt["fk_adj"], kind)
        assert torch.equal(p2.live_bits(), plan.live_bits())
        n = plan.nnz()
        assert p2.nnz() == n
        assert torch.equal(p2.q2k()[1][:n], plan.q2k()[1][:n])


def test_orders_that_are_not_permutations(cuda_lib):
    """An order with repeated and out-of-range entries (clamped to S-1) is not a
    permutation: p_i == p_j then holds off the diagonal, and the prepass must
    still match the oracle's gather of the mask (the per-key diagonal path)."""
    bt = orc.make_batch(39, 2, 384, 3, 2, 6, 0.8, 0.1)
    dev_bt = to_dev(bt)
    for kind in range(4):
        perm = np.array(orc.perm_for_kind(bt, kind), dtype=np.uint16, copy=True)
        perm[0, 5:9] = perm[0, 200]          # repeats inside sample 0
        perm[0, 300:303] = 65535             # past the end: clamps to S-1
        perm[1, 17] = perm[1, 18]            # one repeat in sample 1
        check_plan(bt, kind, dev_bt, perm=perm)
