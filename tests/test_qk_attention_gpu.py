"""The sublayer step with one fused backward (tokens.qk_attention:
rt_qk_prepare + rt_attention_fwd forward, rt_attention_bwd_qkv backward)
against torch autograd of the reference's gather + L2 normalisation * tau +
dense masked attention in fp32 (confluence/confluence/layers.py:63-97,
139-142), and against the unfused kernels (rt_attention_bwd then
rt_qk_prepare_bwd). Token-order gradients of the projection and d tau; all
four kinds, both head widths, a ragged S and zero q / k rows (the clamped
norm)."""
import numpy as np
import pytest
import torch

from encoder_ref import RefOps, dense_attention
from oracle import rt_oracle as orc
from rt_cases import TOL_GRAD_ROW, TOL_OUT, max_rel, row_rel, to_dev_batch

pytestmark = pytest.mark.gpu


def _setup(kind, dh, heads, seed):
    from tributary_b200.attention import build_tile_plan
    bt = orc.make_batch(seed, 2, 300, 4, 2, 9, 0.8, 0.1)
    b, s = bt["seq_row_ids"].shape
    perm = orc.perm_for_kind(bt, kind)
    mask = orc.permute_mask(orc.mask_for_kind(kind, bt["seq_row_ids"], bt["fk_adj"], bt["column_ids"],
                                              bt["is_padding"]), perm)
    dev = to_dev_batch(bt)
    order16 = torch.from_numpy(np.ascontiguousarray(perm).view(np.int16)).cuda()
    plan = build_tile_plan(order16, dev["seq_row_ids"], dev["column_ids"], dev["is_padding"], dev["fk_adj"], kind)
    g = torch.Generator(device="cpu").manual_seed(seed)
    d = heads * dh
    qkv = torch.randn(b, s, 3 * d, generator=g).to(torch.bfloat16).cuda()
    qkv[1, 5, :dh] = 0          # a zero q row of head 0: the clamped norm
    qkv[0, 9, d + dh:d + 2 * dh] = 0  # a zero k row of head 1
    tau = ((torch.rand(heads, generator=g) + 0.5) * dh ** 0.5).cuda()
    d_o = torch.randn(b, heads, s, dh, generator=g).to(torch.bfloat16).cuda()
    order = torch.from_numpy(perm.astype(np.int64)).cuda()
    return plan, order16, order, torch.from_numpy(mask).cuda(), qkv, tau, d_o


@pytest.mark.parametrize("dh,heads", [(64, 2), (32, 2)])
@pytest.mark.parametrize("kind", [0, 1, 2, 3], ids=["column", "feature", "neighbor", "full"])
def test_fused_sublayer_backward(cuda_lib, kind, dh, heads):
    from tributary_b200.attention import device_status, rt_attention
    from tributary_b200.tokens import qk_attention, qk_prepare
    plan, order16, order, mask, qkv, tau, d_o = _setup(kind, dh, heads, 700 + 10 * kind + dh)
    scale = 1.0 / dh ** 0.5

    x1, t1 = qkv.clone().requires_grad_(True), tau.clone().requires_grad_(True)
    o1 = qk_attention(x1, order16, t1, heads, dh, plan, scale)
    o1.backward(d_o)
    assert device_status() == 0

    x2, t2 = qkv.clone().requires_grad_(True), tau.clone().requires_grad_(True)
    q, k, v = qk_prepare(x2, order16, t2, heads, dh)
    o2 = rt_attention(q, k, v, plan, scale)
    o2.backward(d_o)
    assert torch.equal(o1, o2)  # the same forward kernels

    x3, t3 = qkv.float().clone().requires_grad_(True), tau.clone().requires_grad_(True)
    q, k, v = RefOps.qk_prepare(x3, order, t3, heads, dh)
    o3 = dense_attention(q, k, v, mask, scale)
    o3.backward(d_o.float())

    ref = x3.grad.cpu().numpy()
    for name, got in (("fused", x1.grad), ("unfused", x2.grad)):
        g = got.float().cpu().numpy()
        assert np.isfinite(g).all(), name
        assert max_rel(g, ref) < TOL_OUT, (name, max_rel(g, ref))
        # rows: one head's q, k or v slice of one token
        shape = g.shape[:2] + (3 * heads, dh)
        assert row_rel(g.reshape(shape), ref.reshape(shape)) < TOL_GRAD_ROW, name
    torch.testing.assert_close(t1.grad, t3.grad, rtol=2e-2, atol=2e-2 * t3.grad.abs().max().item())
    torch.testing.assert_close(t1.grad, t2.grad, rtol=2e-2, atol=2e-2 * t2.grad.abs().max().item())


def test_encoder_routes_through_the_fused_backward(cuda_lib):
    """KernelOps exposes qk_attention, so every attention sublayer of the
    encoder takes one rt_attention_bwd_qkv call in its backward."""
    from tributary_b200.encoder import KernelOps
    assert hasattr(KernelOps, "qk_attention")
