"""Token preparation kernels (rt_qk_prepare, rt_qk_prepare_bwd,
rt_heads_unpermute / rt_heads_permute) against torch autograd of the
reference's gather + L2 normalisation * tau (layers.py:63-80, 139-167),
including a zero row (the clamped norm) and both head widths."""
import pytest
import torch

from encoder_ref import RefOps

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dh,heads", [(64, 8), (32, 4)])
def test_qk_prepare_and_unpermute_match_torch(cuda_lib, dh, heads):
    from tributary_b200.tokens import heads_unpermute, qk_prepare
    torch.manual_seed(dh + heads)
    b, s = 3, 300
    d = heads * dh
    qkv = torch.randn(b, s, 3 * d, device="cuda").to(torch.bfloat16)
    qkv[1, 5, :dh] = 0  # a zero q row: the clamped norm
    qkv[2, 7, d:d + dh] = 0  # a zero k row
    order = torch.stack([torch.randperm(s) for _ in range(b)]).cuda()
    tau = (torch.rand(heads, device="cuda") + 0.5) * dh ** 0.5
    x1 = qkv.clone().float().requires_grad_(True)
    t1 = tau.clone().requires_grad_(True)
    x2 = qkv.clone().float().requires_grad_(True)
    t2 = tau.clone().requires_grad_(True)
    got = qk_prepare(x1.to(torch.bfloat16), order.to(torch.int32).to(torch.int16), t1, heads, dh)
    want = RefOps.qk_prepare(x2.to(torch.bfloat16), order, t2, heads, dh)
    for g, w in zip(got, want):
        torch.testing.assert_close(g.float(), w.float(), rtol=1e-2, atol=1e-2)
    gs = [torch.randn_like(g.float()).to(torch.bfloat16) for g in got]
    torch.autograd.backward(got, gs)
    torch.autograd.backward(want, gs)
    torch.testing.assert_close(x1.grad, x2.grad, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(t1.grad, t2.grad, rtol=1e-2, atol=1e-2)
    # unpermute and its backward
    o = torch.randn(b, heads, s, dh, device="cuda").to(torch.bfloat16)
    o1, o2 = o.clone().requires_grad_(True), o.clone().requires_grad_(True)
    u1 = heads_unpermute(o1, order.to(torch.int32).to(torch.int16))
    u2 = RefOps.heads_unpermute(o2, order)
    assert torch.equal(u1, u2)  # pure data movement: exact
    gu = torch.randn_like(u1.float()).to(torch.bfloat16)
    u1.backward(gu)
    u2.backward(gu)
    assert torch.equal(o1.grad, o2.grad)
