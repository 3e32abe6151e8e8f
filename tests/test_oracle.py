"""The oracle against golden vectors produced by running the reference source.

CPU only. Fixtures come from tests/golden/make_golden.py, which executed the
reference's build_attention_masks (confluence/confluence/model.py:201-264) and
GatedAttentionSublayer (confluence/confluence/layers.py:113-174).
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_files, load_golden, unpack_mask
from oracle import rt_oracle as orc


@pytest.mark.parametrize("path", golden_files("masks"), ids=lambda p: p.split("/")[-1])
def test_masks_match_reference(path):
    g = load_golden(path)
    s = int(g["S"])
    outbound, inbound, column, full = orc.build_attention_masks(
        g["seq_row_ids"], g["fk_adj"], g["column_ids"], g["is_padding"])
    np.testing.assert_array_equal(outbound, unpack_mask(g["ref_outbound_bits"], s))
    np.testing.assert_array_equal(inbound, unpack_mask(g["ref_inbound_bits"], s))
    np.testing.assert_array_equal(column, unpack_mask(g["ref_column_bits"], s))
    pad = g["is_padding"].astype(bool)
    exp_full = ((~pad[:, :, None]) & (~pad[:, None, :])) | np.eye(s, dtype=bool)[None]
    np.testing.assert_array_equal(full, exp_full)


def test_bookstore_example_visibility():
    """documentation/model_architecture/attention.md:42-75, restated as cells.

    Rows: 0 order1, 1 cust23, 2 book42, 3 order7, 4 order12, 5 order5; each
    row holds two cells (positions 2r, 2r+1).
    """
    g = load_golden(os.path.join(GOLDEN, "masks_bookstore.npz"))
    s = int(g["S"])
    outbound, inbound, _, _ = orc.build_attention_masks(
        g["seq_row_ids"], g["fk_adj"], g["column_ids"], g["is_padding"])

    def rows_seen(mask, row):
        i = 2 * row
        cols = np.nonzero(mask[0, i, :12])[0]
        return sorted({int(c) // 2 for c in cols})

    # outbound: order 1 sees {order 1, customer 23, book 42}; customer 23 sees itself
    assert rows_seen(outbound, 0) == [0, 1, 2]
    assert rows_seen(outbound, 1) == [1]
    # inbound: customer 23 sees {order1, order7, order12}; book 42 sees {order1, order5}
    in_no_diag = inbound & ~np.eye(s, dtype=bool)[None]
    assert rows_seen(in_no_diag, 1) == [0, 3, 4]
    assert rows_seen(in_no_diag, 2) == [0, 5]
    # order 7 sees nothing but its own diagonal cell
    assert rows_seen(in_no_diag, 3) == []
    np.testing.assert_array_equal(outbound, unpack_mask(g["ref_outbound_bits"], s))


@pytest.mark.parametrize("path", golden_files("sublayer"), ids=lambda p: p.split("/")[-1])
def test_sublayer_forward_matches_reference(path):
    """Permutation, QK-norm, masked softmax attention and the sublayer
    epilogue of the oracle against the captured reference run."""
    g = load_golden(path)
    kind, h, dh = int(g["kind"]), int(g["H"]), int(g["Dh"])
    x = g["x"]
    b, s, d = x.shape
    perm = orc.perm_for_kind(g, kind)
    mask = orc.mask_for_kind(kind, g["seq_row_ids"], g["fk_adj"], g["column_ids"], g["is_padding"])
    mask_perm = orc.permute_mask(mask, perm)
    np.testing.assert_array_equal(mask_perm, unpack_mask(g["ref_mask_perm_bits"], s))

    # pre-norm (layers.py:16-29) and token gather
    gamma = g["w_norm_gamma"]
    rms = np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + np.float32(1e-6))
    x_norm = ((1.0 + gamma) * x / rms).astype(np.float32)
    x_perm = orc.gather_tokens(x_norm, perm)
    np.testing.assert_allclose(x_perm, g["ref_x_perm"], rtol=1e-6, atol=1e-6)

    qkv = x_perm @ g["w_qkv"]
    q, k, v = np.split(qkv, 3, axis=-1)
    heads = lambda t: t.reshape(b, s, h, dh).transpose(0, 2, 1, 3)
    qh, kh = orc.qk_normalize(heads(q), heads(k), g["tau"])
    o, lse = orc.attention_fwd(qh, kh, heads(v), mask_perm, 1.0 / np.sqrt(dh))
    merged = o.transpose(0, 2, 1, 3).reshape(b, s, d)
    np.testing.assert_allclose(merged, g["ref_attn_merged"], rtol=2e-5, atol=2e-5)

    out = (merged @ g["w_o"]) * g["output_scale"]
    unperm = orc.scatter_tokens(out, perm)
    gate = 1.0 / (1.0 + np.exp(-(x_norm @ g["w_gate"])))
    y = x + unperm * gate
    np.testing.assert_allclose(y, g["ref_y"], rtol=2e-5, atol=2e-5)


def test_lse_is_logsumexp_over_live_keys():
    bt = orc.make_batch(3, 2, 128, 3, 2, 6, 0.7, 0.1)
    q, k, v, _ = orc.make_qkv(4, 2, 2, 128, 32, dtype=np.float64)
    for kind in range(4):
        mp = orc.permute_mask(orc.mask_for_kind(kind, bt["seq_row_ids"], bt["fk_adj"],
                                                bt["column_ids"], bt["is_padding"]),
                              orc.perm_for_kind(bt, kind))
        _, lse = orc.attention_fwd(q, k, v, mp, 1 / np.sqrt(32), dtype=np.float64)
        s = np.einsum("bhid,bhjd->bhij", q, k) / np.sqrt(32)
        ref = np.log(np.where(mp[:, None], np.exp(s), 0.0).sum(-1))
        np.testing.assert_allclose(lse, ref, rtol=1e-12, atol=1e-12)


def test_backward_matches_finite_differences():
    """The analytic backward is the derivative of the (reference-pinned)
    forward: central differences in float64 on a small case."""
    rng = np.random.default_rng(5)
    bt = orc.make_batch(6, 1, 48, 3, 2, 5, 0.7, 0.1)
    mp = orc.permute_mask(orc.mask_for_kind(orc.MASK_FEATURE, bt["seq_row_ids"], bt["fk_adj"],
                                            bt["column_ids"], bt["is_padding"]), bt["out_perm"])
    b, h, s, dh = 1, 2, 48, 8
    q = rng.standard_normal((b, h, s, dh))
    k = rng.standard_normal((b, h, s, dh))
    v = rng.standard_normal((b, h, s, dh))
    do = rng.standard_normal((b, h, s, dh))
    scale = 0.7
    o, _ = orc.attention_fwd(q, k, v, mp, scale, dtype=np.float64)
    dq, dk, dv = orc.attention_bwd(q, k, v, o, do, mp, scale, dtype=np.float64)

    def loss(qq, kk, vv):
        oo, _ = orc.attention_fwd(qq, kk, vv, mp, scale, dtype=np.float64)
        return float((oo * do).sum())

    eps = 1e-6
    for name, arr, grad in (("q", q, dq), ("k", k, dk), ("v", v, dv)):
        for idx in [(0, 0, 3, 1), (0, 1, 17, 5), (0, 1, 40, 0), (0, 0, 47, 7)]:
            plus = arr.copy(); plus[idx] += eps
            minus = arr.copy(); minus[idx] -= eps
            args_p = {"q": q, "k": k, "v": v}; args_p[name] = plus
            args_m = {"q": q, "k": k, "v": v}; args_m[name] = minus
            fd = (loss(args_p["q"], args_p["k"], args_p["v"]) -
                  loss(args_m["q"], args_m["k"], args_m["v"])) / (2 * eps)
            assert abs(fd - grad[idx]) < 1e-6 * max(1.0, abs(fd)), (name, idx, fd, grad[idx])


def test_padding_rows_copy_their_value():
    """A padding query sees only its own diagonal, so o_i = v_i."""
    bt = orc.make_batch(7, 1, 64, 2, 3, 4, 0.5, 0.25)
    q, k, v, _ = orc.make_qkv(8, 1, 2, 64, 16, dtype=np.float64)
    for kind in range(4):
        m = orc.mask_for_kind(kind, bt["seq_row_ids"], bt["fk_adj"], bt["column_ids"],
                              bt["is_padding"])
        o, _ = orc.attention_fwd(q, k, v, m, 0.25, dtype=np.float64)
        pad = bt["is_padding"][0].astype(bool)
        np.testing.assert_allclose(o[0][:, pad], v[0][:, pad], rtol=1e-12, atol=1e-12)


def test_tile_lists_and_bitmaps_consistent():
    bt = orc.make_batch(9, 2, 640, 4, 3, 9, 0.6, 0.1)
    for kind in range(4):
        mp = orc.permute_mask(orc.mask_for_kind(kind, bt["seq_row_ids"], bt["fk_adj"],
                                                bt["column_ids"], bt["is_padding"]),
                              orc.perm_for_kind(bt, kind))
        live, full = orc.tile_occupancy(mp)
        lb, fb = orc.tile_bitmaps(mp)
        q2k_ptr, q2k_idx, k2q_ptr, k2q_idx = orc.tile_lists(mp)
        t = live.shape[1]
        assert q2k_ptr[-1] == live.sum() == k2q_ptr[-1]
        # diagonal tiles are always live; full implies live
        assert all(live[b, i, i] for b in range(2) for i in range(t))
        assert not (full & ~live).any()
        for bb in range(2):
            for qt in range(t):
                ent = q2k_idx[q2k_ptr[bb * t + qt]:q2k_ptr[bb * t + qt + 1]]
                kts = ent & 0x7FFFFFFF
                assert list(kts) == list(np.nonzero(live[bb, qt])[0])
                assert list((ent < 0)) == list(full[bb, qt, kts])
                for kt in range(t):
                    assert bool((lb[bb, qt, kt // 32] >> (kt % 32)) & 1) == live[bb, qt, kt]
                    assert bool((fb[bb, qt, kt // 32] >> (kt % 32)) & 1) == full[bb, qt, kt]
        words = orc.tile_mask_words(mp)
        unpacked = ((words[..., None] >> np.arange(32, dtype=np.uint32)) & 1).astype(bool)
        unpacked = unpacked.reshape(words.shape[:-1] + (128,))
        dense = orc.padded_tile_mask(mp).reshape(2, t, 128, t, 128).transpose(0, 1, 3, 2, 4)
        np.testing.assert_array_equal(unpacked, dense)


def test_rcm_perm_is_a_permutation_with_padding_last():
    bt = orc.make_batch(10, 3, 300, 5, 2, 11, 0.8, 0.15)
    for key in ("col_perm", "out_perm", "in_perm"):
        for bb in range(3):
            p = bt[key][bb].astype(np.int64)
            assert sorted(p) == list(range(300))
            pads = bt["is_padding"][bb][p]
            assert (np.diff(pads.astype(int)) >= 0).all()


def test_col_perm_groups_columns():
    bt = orc.make_batch(11, 1, 200, 3, 2, 6, 0.5, 0.0)
    p = bt["col_perm"][0].astype(np.int64)
    cols = bt["column_ids"][0][p]
    assert (np.diff(cols) >= 0).all()
