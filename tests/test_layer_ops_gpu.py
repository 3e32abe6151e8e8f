"""Fused encoder-layer kernels against a plain PyTorch fp32 reference of the
same op (ZeroCenteredRMSNorm, layers.py:16-30; the gated residual,
layers.py:170-174; SwiGLU, layers.py:177-200): forward and backward, with
bf16 outputs compared to the fp32 result within bf16 rounding."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

BF16_REL = 2.0 ** -8  # one bf16 rounding (round to nearest: 2^-9) plus fp32 evaluation-order slack


def _close(got, want, rel, name):
    got, want = got.double(), want.double()
    err = (got - want).abs().max().item()
    scale = want.abs().max().item()
    assert err <= rel * scale + 1e-30, (name, err, scale)


@pytest.mark.parametrize("rows,d", [(4096, 512), (777, 64), (333, 1024)])
def test_rms_norm_forward_and_backward(cuda_lib, rows, d):
    from tributary_b200.layer_ops import rms_norm
    g = torch.Generator(device="cuda").manual_seed(rows + d)
    x = torch.randn(rows, d, device="cuda", generator=g) * 3
    gamma = torch.randn(d, device="cuda", generator=g) * 0.1
    dy = torch.randn(rows, d, device="cuda", generator=g).to(torch.bfloat16)
    xk, gk = x.clone().requires_grad_(True), gamma.clone().requires_grad_(True)
    y = rms_norm(xk, gk, 1e-6)
    assert y.dtype == torch.bfloat16
    y.backward(dy)
    xr, gr = x.clone().requires_grad_(True), gamma.clone().requires_grad_(True)
    yr = F.rms_norm(xr, (d,), 1.0 + gr, 1e-6)
    yr.backward(dy.float())
    # the kernel's y is the fp32 value rounded once to bf16
    _close(y.float(), yr, BF16_REL, "y")
    _close(xk.grad, xr.grad, 1e-5, "dx")
    _close(gk.grad, gr.grad, 1e-5, "dgamma")
    # dgamma is summed in a fixed order: identical on a second call
    gk2 = gamma.clone().requires_grad_(True)
    rms_norm(x, gk2, 1e-6).backward(dy)
    assert torch.equal(gk2.grad, gk.grad)


def test_gate_residual_forward_and_backward(cuda_lib):
    from tributary_b200.layer_ops import gate_residual
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(2, 300, 512, device="cuda", generator=g)
    out = torch.randn(2, 300, 512, device="cuda", generator=g).to(torch.bfloat16)
    gate = (torch.randn(2, 300, 512, device="cuda", generator=g) * 2).to(torch.bfloat16)
    dy = torch.randn(2, 300, 512, device="cuda", generator=g)
    scale = 0.1443
    args = [t.clone().requires_grad_(True) for t in (x, out, gate)]
    y = gate_residual(*args, scale)
    y.backward(dy)
    ref = [t.clone().float().requires_grad_(True) for t in (x, out, gate)]
    yr = ref[0] + scale * ref[1] * torch.sigmoid(ref[2])
    yr.backward(dy)
    _close(y, yr, 1e-6, "y")
    assert torch.equal(args[0].grad, dy)
    _close(args[1].grad.float(), ref[1].grad, BF16_REL, "d_out")
    _close(args[2].grad.float(), ref[2].grad, BF16_REL, "d_gate")


def test_residual_add_forward_and_backward(cuda_lib):
    from tributary_b200.layer_ops import residual_add
    g = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn(3, 200, 512, device="cuda", generator=g)
    h = torch.randn(3, 200, 512, device="cuda", generator=g).to(torch.bfloat16)
    dy = torch.randn(3, 200, 512, device="cuda", generator=g)
    xk, hk = x.clone().requires_grad_(True), h.clone().requires_grad_(True)
    y = residual_add(xk, hk, 0.1443)
    y.backward(dy)
    _close(y, x + 0.1443 * h.float(), 1e-6, "y")
    assert torch.equal(xk.grad, dy)
    _close(hk.grad.float(), dy * 0.1443, BF16_REL, "dh")


@pytest.mark.parametrize("rows,f", [(4096, 1536), (129, 64)])
def test_swiglu_forward_and_backward(cuda_lib, rows, f):
    from tributary_b200.layer_ops import swiglu
    g = torch.Generator(device="cuda").manual_seed(rows)
    u = (torch.randn(rows, 2 * f, device="cuda", generator=g) * 2).to(torch.bfloat16)
    dh = torch.randn(rows, f, device="cuda", generator=g).to(torch.bfloat16)
    uk = u.clone().requires_grad_(True)
    h = swiglu(uk)
    h.backward(dh)
    ur = u.float().requires_grad_(True)
    hr = F.silu(ur[:, :f]) * ur[:, f:]
    hr.backward(dh.float())
    _close(h.float(), hr, BF16_REL, "h")
    _close(uk.grad.float(), ur.grad, BF16_REL, "du")


def test_layer_ops_reject_bad_widths(cuda_lib):
    from tributary_b200 import _lib
    lib = _lib.load()
    x = torch.zeros(4, 12, device="cuda")
    y = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")
    r = torch.zeros(4, device="cuda")
    gamma = torch.zeros(12, device="cuda")
    assert lib.rt_rms_norm(x.data_ptr(), gamma.data_ptr(), 4, 12, 1e-6, y.data_ptr(), r.data_ptr(), None) == \
        _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_swiglu(y.data_ptr(), 4, 6, y.data_ptr(), None) == _lib.RT_ERR_INVALID_ARGUMENT
