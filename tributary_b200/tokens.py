"""Token preparation of an attention sublayer on the library's kernels, with
autograd: the fused gather + head split + QK L2 normalisation * tau
(rt_qk_prepare, confluence/confluence/layers.py:63-80 and 139-142) and the
scatter of the attention output back to token order (rt_heads_unpermute,
layers.py:99 and 159-167).

Orders are [B, S] int16 tensors holding the uint16 cell order of the
sublayer's mask kind.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .attention import _stream_ptr


def _order16(order: torch.Tensor) -> torch.Tensor:
    if order.dtype == torch.int16:
        return order.contiguous()
    return order.to(torch.int32).to(torch.int16).contiguous()


def _prepare(qkv, order16, tau, heads: int, head_dim: int):
    """rt_qk_prepare: (q_hat * tau, k_hat, v) in cell order, the bf16
    contiguous qkv and fp32 tau it read, and the inverse norms."""
    b, s, three_d = qkv.shape
    if three_d != 3 * heads * head_dim:
        raise ValueError("qkv must be [B, S, 3 * heads * head_dim]")
    qkv = qkv.to(torch.bfloat16).contiguous()
    tau32 = tau.detach().float().contiguous()
    q, k, v = (torch.empty(b, heads, s, head_dim, dtype=torch.bfloat16, device=qkv.device) for _ in range(3))
    rnorm = torch.empty(2, b, heads, s, dtype=torch.float32, device=qkv.device)
    _lib.check(_lib.load().rt_qk_prepare(qkv.data_ptr(), order16.data_ptr(), tau32.data_ptr(), b, heads, s,
                                         head_dim, q.data_ptr(), k.data_ptr(), v.data_ptr(), rnorm.data_ptr(),
                                         _stream_ptr(qkv.device)), "rt_qk_prepare")
    return q, k, v, qkv, tau32, rnorm


class QKPrepare(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, order16, tau, heads: int, head_dim: int):
        q, k, v, qkv, tau32, rnorm = _prepare(qkv, order16, tau, heads, head_dim)
        ctx.save_for_backward(qkv, order16, tau32, rnorm)
        ctx.dims = (qkv.shape[0], heads, qkv.shape[1], head_dim)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, order16, tau32, rnorm = ctx.saved_tensors
        b, heads, s, head_dim = ctx.dims
        z = None
        shape = (b, heads, s, head_dim)
        dq, dk, dv = ((g if g is not None else qkv.new_zeros(shape)).to(torch.bfloat16).contiguous()
                      for g in (dq, dk, dv))
        dqkv = torch.empty_like(qkv)
        dtau_rows = torch.empty(b, heads, s, dtype=torch.float32, device=qkv.device)
        _lib.check(_lib.load().rt_qk_prepare_bwd(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), qkv.data_ptr(),
                                                 order16.data_ptr(), tau32.data_ptr(), rnorm.data_ptr(), b, heads,
                                                 s, head_dim, dqkv.data_ptr(), dtau_rows.data_ptr(),
                                                 _stream_ptr(qkv.device)), "rt_qk_prepare_bwd")
        return dqkv, z, dtau_rows.sum(dim=(0, 2)), z, z


class QKAttention(torch.autograd.Function):
    """Gather + QK normalisation (rt_qk_prepare) and the attention forward in
    one autograd node, so that the backward is a single rt_attention_bwd_qkv
    call: the normalisation's Jacobian and the scatter to token order run in
    the attention backward's epilogues (layers.py:63-97, 139-142)."""

    @staticmethod
    def forward(ctx, qkv, order16, tau, heads: int, head_dim: int, plan, scale: float):
        from .attention import attention_fwd
        q, k, v, qkv_c, tau32, rnorm = _prepare(qkv, order16, tau, heads, head_dim)
        o, lse = attention_fwd(q, k, v, plan, scale)
        ctx.save_for_backward(qkv_c, order16, tau32, rnorm, q, k, v, o, lse)
        ctx.plan, ctx.scale = plan, scale
        return o

    @staticmethod
    def backward(ctx, d_o):
        qkv, order16, tau32, rnorm, q, k, v, o, lse = ctx.saved_tensors
        b, heads, s, head_dim = q.shape
        lib = _lib.load()
        d_o = d_o.to(torch.bfloat16).contiguous()
        dqkv = torch.empty_like(qkv)
        dtau_rows = torch.empty(b, heads, s, dtype=torch.float32, device=qkv.device)
        ws = torch.empty(max(lib.rt_attention_bwd_workspace_bytes(b, heads, s), 256), dtype=torch.uint8,
                         device=qkv.device)
        _lib.check(lib.rt_attention_bwd_qkv(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), d_o.data_ptr(), lse.data_ptr(), b, heads, s,
            head_dim, float(ctx.scale), ctypes.byref(ctx.plan.c), order16.data_ptr(), qkv.data_ptr(),
            tau32.data_ptr(), rnorm.data_ptr(), dqkv.data_ptr(), dtau_rows.data_ptr(), ws.data_ptr(), ws.numel(),
            _stream_ptr(qkv.device)), "rt_attention_bwd_qkv")
        z = None
        return dqkv, z, dtau_rows.sum(dim=(0, 2)), z, z, z, z


class HeadsUnpermute(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, order16):
        b, h, s, dh = o.shape
        o = o.contiguous()
        out = torch.empty(b, s, h * dh, dtype=o.dtype, device=o.device)
        _lib.check(_lib.load().rt_heads_unpermute(o.data_ptr(), order16.data_ptr(), b, h, s, dh, out.data_ptr(),
                                                  _stream_ptr(o.device)), "rt_heads_unpermute")
        ctx.save_for_backward(order16)
        ctx.dims = (b, h, s, dh)
        return out

    @staticmethod
    def backward(ctx, g):
        (order16,) = ctx.saved_tensors
        b, h, s, dh = ctx.dims
        g = g.to(torch.bfloat16).contiguous()
        out = torch.empty(b, h, s, dh, dtype=torch.bfloat16, device=g.device)
        _lib.check(_lib.load().rt_heads_permute(g.data_ptr(), order16.data_ptr(), b, h, s, dh, out.data_ptr(),
                                                _stream_ptr(g.device)), "rt_heads_permute")
        return out, None


def qk_prepare(qkv, order16, tau, heads: int, head_dim: int):
    """[B,S,3D] QKV projection in token order -> (q_hat * tau, k_hat, v), each
    bf16 [B,H,S,Dh] in the cell order ``order16``."""
    return QKPrepare.apply(qkv, order16, tau, heads, head_dim)


def qk_attention(qkv, order16, tau, heads: int, head_dim: int, plan, scale: float | None = None):
    """[B,S,3D] QKV projection in token order -> attention output [B,H,S,Dh]
    in the cell order ``order16`` of ``plan``'s kind: rt_qk_prepare and
    rt_attention_fwd forward, one rt_attention_bwd_qkv backward."""
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    return QKAttention.apply(qkv, order16, tau, heads, head_dim, plan, scale)


def heads_unpermute(o, order16):
    """Attention output [B,H,S,Dh] in cell order -> [B,S,H*Dh] in token order."""
    return HeadsUnpermute.apply(o, order16)
