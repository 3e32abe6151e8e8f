"""Autograd wrappers of the library's fused encoder-layer kernels (the
training step's non-attention work): ZeroCenteredRMSNorm
(confluence/confluence/layers.py:16-30), the gated residual of the attention
sublayer (layers.py:170-174), the SwiGLU activation (layers.py:177-200) and
the FFN's residual.
CUDA tensors only; each forward and backward is one kernel of
libtributary_b200.so."""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .attention import _stream_ptr


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


class RMSNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, eps):
        x = x.float().contiguous()
        d = x.shape[-1]
        rows = x.numel() // d
        y = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        g = gamma.float().contiguous()
        _lib.check(_lib.load().rt_rms_norm(_p(x), _p(g), rows, d, float(eps), _p(y), _p(rstd),
                                           _stream_ptr(x.device)), "rt_rms_norm")
        ctx.save_for_backward(x, g, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, g, rstd = ctx.saved_tensors
        lib = _lib.load()
        d = x.shape[-1]
        rows = x.numel() // d
        dy = dy.to(torch.bfloat16).contiguous()
        dx = torch.empty_like(x)
        dgamma = torch.empty_like(g)
        ws = torch.empty(lib.rt_rms_norm_bwd_workspace_bytes(rows, d), dtype=torch.uint8, device=x.device)
        _lib.check(lib.rt_rms_norm_bwd(_p(dy), _p(x), _p(g), _p(rstd), rows, d, _p(dx), _p(dgamma), _p(ws),
                                       ws.numel(), _stream_ptr(x.device)), "rt_rms_norm_bwd")
        return dx, dgamma, None


class GateResidualFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, out, gate, scale):
        x = x.float().contiguous()
        out = out.to(torch.bfloat16).contiguous()
        gate = gate.to(torch.bfloat16).contiguous()
        y = torch.empty_like(x)
        _lib.check(_lib.load().rt_gate_residual(_p(x), _p(out), _p(gate), x.numel(), float(scale), _p(y),
                                                _stream_ptr(x.device)), "rt_gate_residual")
        ctx.save_for_backward(out, gate)
        ctx.scale = scale
        return y

    @staticmethod
    def backward(ctx, dy):
        out, gate = ctx.saved_tensors
        dy = dy.float().contiguous()
        d_out = torch.empty_like(out)
        d_gate = torch.empty_like(gate)
        _lib.check(_lib.load().rt_gate_residual_bwd(_p(dy), _p(out), _p(gate), dy.numel(), float(ctx.scale),
                                                    _p(d_out), _p(d_gate), _stream_ptr(dy.device)),
                   "rt_gate_residual_bwd")
        return dy, d_out, d_gate, None


class ResidualAddFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, h, scale):
        x = x.float().contiguous()
        h = h.to(torch.bfloat16).contiguous()
        y = torch.empty_like(x)
        _lib.check(_lib.load().rt_residual_add(_p(x), _p(h), x.numel(), float(scale), _p(y), _stream_ptr(x.device)),
                   "rt_residual_add")
        ctx.scale = scale
        return y

    @staticmethod
    def backward(ctx, dy):
        dy = dy.float().contiguous()
        dh = torch.empty(dy.shape, dtype=torch.bfloat16, device=dy.device)
        _lib.check(_lib.load().rt_residual_add_bwd(_p(dy), dy.numel(), float(ctx.scale), _p(dh),
                                                   _stream_ptr(dy.device)), "rt_residual_add_bwd")
        return dy, dh, None


class SwiGLUFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u):
        u = u.to(torch.bfloat16).contiguous()
        f = u.shape[-1] // 2
        rows = u.numel() // u.shape[-1]
        h = torch.empty(u.shape[:-1] + (f,), dtype=torch.bfloat16, device=u.device)
        _lib.check(_lib.load().rt_swiglu(_p(u), rows, f, _p(h), _stream_ptr(u.device)), "rt_swiglu")
        ctx.save_for_backward(u)
        return h

    @staticmethod
    def backward(ctx, dh):
        (u,) = ctx.saved_tensors
        f = u.shape[-1] // 2
        rows = u.numel() // u.shape[-1]
        dh = dh.to(torch.bfloat16).contiguous()
        du = torch.empty_like(u)
        _lib.check(_lib.load().rt_swiglu_bwd(_p(dh), _p(u), rows, f, _p(du), _stream_ptr(u.device)), "rt_swiglu_bwd")
        return du


def rms_norm(x, gamma, eps: float):
    """bf16 (1 + gamma) * x / sqrt(mean(x^2) + eps) of an fp32 [..., d] tensor."""
    return RMSNormFunction.apply(x, gamma, eps)


def gate_residual(x, out, gate, scale: float):
    """fp32 x + scale * out * sigmoid(gate) (out, gate: the bf16 W_O and W_gate outputs)."""
    return GateResidualFunction.apply(x, out, gate, scale)


def residual_add(x, h, scale: float):
    """fp32 x + scale * h (h: the bf16 W_down output)."""
    return ResidualAddFunction.apply(x, h, scale)


def swiglu(u):
    """bf16 silu(u[..., :f]) * u[..., f:] of the fused [..., 2f] gate / up projection."""
    return SwiGLUFunction.apply(u)
