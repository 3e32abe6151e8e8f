"""JAX binding of the library through XLA FFI: what the reference model calls
in place of confluence/confluence/layers.py:82-97 (masked softmax attention
and, through jax.custom_vjp, its autodiff backward) and of
confluence/confluence/model.py:201-264 (one tile plan per mask kind instead of
three dense [B,S,S] masks).

Needs jax and the handlers built by build_ffi.py; importing this module
without jax raises ImportError. The plan buffer and the backward's workspace
are XLA outputs whose sizes come from the library (rt_tile_plan_bytes,
rt_attention_bwd_workspace_bytes) at trace time.
"""
from __future__ import annotations

import ctypes
import functools

import jax
import jax.numpy as jnp
import numpy as np

from .. import _lib
from .build_ffi import FFI_LIB

_REGISTERED = False


def register():
    global _REGISTERED
    if _REGISTERED:
        return
    handlers = ctypes.CDLL(FFI_LIB)
    for name in ("rt_tile_plan_ffi", "rt_attention_fwd_ffi", "rt_attention_bwd_ffi"):
        jax.ffi.register_ffi_target(name, jax.ffi.pycapsule(getattr(handlers, name)), platform="CUDA")
    _REGISTERED = True


def tile_plan(perm, seq_row_ids, column_ids, is_padding, fk_adj, kind: int):
    """u8 plan buffer of one mask kind (model.py:201-264 plus the permutation
    of layers.py:144-152): perm, seq_row_ids uint16 [B,S], column_ids int32,
    is_padding uint8 [B,S], fk_adj uint8 [B,R,R]."""
    register()
    b, s = perm.shape
    r = fk_adj.shape[1]
    nbytes = int(_lib.load().rt_tile_plan_bytes(b, s, r))
    out = jax.ShapeDtypeStruct((nbytes,), jnp.uint8)
    return jax.ffi.ffi_call("rt_tile_plan_ffi", out)(perm, seq_row_ids, column_ids, is_padding, fk_adj,
                                                     kind=np.int32(kind))


def _fwd_call(q, k, v, plan, max_rows, scale):
    b, h, s, dh = q.shape
    outs = (jax.ShapeDtypeStruct(q.shape, jnp.bfloat16), jax.ShapeDtypeStruct((b, h, s), jnp.float32))
    return jax.ffi.ffi_call("rt_attention_fwd_ffi", outs)(q, k, v, plan, max_rows=np.int32(max_rows),
                                                          scale=np.float32(scale))


@functools.partial(jax.custom_vjp, nondiff_argnums=(4, 5))
def rt_attention(q, k, v, plan, max_rows: int, scale: float):
    """o = softmax(q k^T * scale masked by the plan) v for bf16 [B,H,S,Dh]
    q_hat, k_hat, v in the plan's cell order."""
    register()
    return _fwd_call(q, k, v, plan, max_rows, scale)[0]


def _rt_attention_fwd(q, k, v, plan, max_rows, scale):
    register()
    o, lse = _fwd_call(q, k, v, plan, max_rows, scale)
    return o, (q, k, v, plan, o, lse)


def _rt_attention_bwd(max_rows, scale, res, d_o):
    q, k, v, plan, o, lse = res
    b, h, s, dh = q.shape
    ws = int(_lib.load().rt_attention_bwd_workspace_bytes(b, h, s))
    outs = tuple(jax.ShapeDtypeStruct(q.shape, jnp.bfloat16) for _ in range(3)) + (
        jax.ShapeDtypeStruct((ws,), jnp.uint8),)
    dq, dk, dv, _ = jax.ffi.ffi_call("rt_attention_bwd_ffi", outs)(
        q, k, v, o, d_o.astype(jnp.bfloat16), lse, plan, max_rows=np.int32(max_rows), scale=np.float32(scale))
    return dq, dk, dv, None


rt_attention.defvjp(_rt_attention_fwd, _rt_attention_bwd)
