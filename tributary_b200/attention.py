"""PyTorch host layer over the CUDA library, mirroring the reference interface.

Reference interface (confluence/confluence):

* ``build_attention_masks(batch, max_rows) -> (outbound, inbound, column)``
  model.py:201-264 -- here it returns one ``TilePlan`` per kind instead of
  dense [B,S,S] masks (the plan is built on the GPU by the prepass kernel and
  already accounts for the sublayer's permutation, layers.py:144-152).
* ``QKNormedMultiHeadAttention`` / ``GatedAttentionSublayer`` -- the core
  lines layers.py:82-97 become ``rt_attention(q_hat, k_hat, v, plan, scale)``,
  a ``torch.autograd.Function`` whose forward and backward are the library's
  sm_100a kernels.

PyTorch only supplies device memory, streams and autograd plumbing. Every
call goes through the C ABI (``tributary_b200._lib``); there is no CPU or
eager fallback, and a missing library raises.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib

MASK_COLUMN = _lib.RT_MASK_COLUMN
MASK_FEATURE = _lib.RT_MASK_FEATURE
MASK_NEIGHBOR = _lib.RT_MASK_NEIGHBOR
MASK_FULL = _lib.RT_MASK_FULL
MASK_KINDS = {"column": MASK_COLUMN, "feature": MASK_FEATURE, "outbound": MASK_FEATURE,
              "neighbor": MASK_NEIGHBOR, "inbound": MASK_NEIGHBOR, "full": MASK_FULL}
TILE = _lib.TILE


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(t: torch.Tensor, name: str, dtype: torch.dtype, shape=None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")


@dataclass
class TilePlan:
    """Device-resident output of the prepass for one (batch, mask kind, perm).

    ``buffer`` owns the memory; ``c`` is the C struct whose pointers index it.
    """
    kind: int
    batch: int
    seq_len: int
    max_rows: int
    buffer: torch.Tensor
    c: _lib.RtTilePlan

    @property
    def tiles(self) -> int:
        return self.c.tiles

    def _view(self, ptr_field: str, count: int, dtype: torch.dtype) -> torch.Tensor:
        base = self.buffer.data_ptr()
        off = getattr(self.c, ptr_field) - base
        nbytes = count * torch.tensor([], dtype=dtype).element_size()
        return self.buffer[off:off + nbytes].view(dtype)

    def live_bits(self):
        b, t, w = self.batch, self.c.tiles, self.c.words
        return self._view("live_bits", b * t * w, torch.int32).view(b, t, w)

    def full_bits(self):
        b, t, w = self.batch, self.c.tiles, self.c.words
        return self._view("full_bits", b * t * w, torch.int32).view(b, t, w)

    def q2k(self):
        n = self.batch * self.c.tiles
        ptr = self._view("q2k_ptr", n + 1, torch.int32)
        return ptr, self._view("q2k_idx", n * self.c.tiles, torch.int32)

    def k2q(self):
        n = self.batch * self.c.tiles
        ptr = self._view("k2q_ptr", n + 1, torch.int32)
        return ptr, self._view("k2q_idx", n * self.c.tiles, torch.int32)

    def tile_masks(self, transposed: bool = False):
        b, t = self.batch, self.c.tiles
        field = "tile_masks_t" if transposed else "tile_masks"
        return self._view(field, b * t * t * TILE * 4, torch.int32).view(b, t, t, TILE, 4)

    def nnz(self) -> int:
        return int(self._view("nnz", 1, torch.int32).item())


def build_tile_plan(perm, seq_row_ids, column_ids, is_padding, fk_adj, kind: int,
                    max_rows: int | None = None) -> TilePlan:
    """Run the prepass kernel for one mask kind (replaces model.py:201-264 +
    layers.py:144-152). Tensors are the headwater batch tensors on the GPU:
    perm/seq_row_ids uint16 (int16 storage accepted), column_ids int32,
    is_padding uint8 (or bool), fk_adj uint8 (or bool) [B,R,R]."""
    lib = _lib.load()
    if isinstance(kind, str):
        kind = MASK_KINDS[kind]
    dev = perm.device
    b, s = perm.shape
    r = fk_adj.shape[1] if max_rows is None else max_rows

    def u16(t):
        if t.dtype == torch.uint16 or t.dtype == torch.int16:
            return t.contiguous()
        return t.to(torch.int32).to(torch.int16).contiguous()

    perm_c = u16(perm)
    rows_c = u16(seq_row_ids)
    cols_c = column_ids.to(torch.int32).contiguous()
    pad_c = is_padding.to(torch.uint8).contiguous()
    fk_c = fk_adj.to(torch.uint8).contiguous()
    for name, t in (("perm", perm_c), ("seq_row_ids", rows_c), ("column_ids", cols_c),
                    ("is_padding", pad_c), ("fk_adj", fk_c)):
        if not t.is_cuda or t.device != dev:
            raise ValueError(f"{name} must be on {dev}")
    nbytes = lib.rt_tile_plan_bytes(b, s, r)
    buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    plan = _lib.RtTilePlan()
    _lib.check(lib.rt_tile_plan_bind(buf.data_ptr(), nbytes, b, s, r, ctypes.byref(plan)),
               "rt_tile_plan_bind")
    _lib.check(lib.rt_build_tile_plan(perm_c.data_ptr(), rows_c.data_ptr(), cols_c.data_ptr(),
                                      pad_c.data_ptr(), fk_c.data_ptr(), b, s, r, kind,
                                      ctypes.byref(plan), _stream_ptr(dev)),
               "rt_build_tile_plan")
    return TilePlan(kind=kind, batch=b, seq_len=s, max_rows=r, buffer=buf, c=plan)


def column_order(column_ids: torch.Tensor, is_padding: torch.Tensor) -> torch.Tensor:
    """The column kind's cell order (sampler.rs:655-668: padding flag, column
    id, position) computed on the GPU from [B,S] device tensors; int16 storage
    of the uint16 order, bit-identical to the host rt_column_order."""
    lib = _lib.load()
    cols = column_ids.to(torch.int32).contiguous()
    pad = is_padding.to(torch.uint8).contiguous()
    b, s = cols.shape
    out = torch.empty((b, s), dtype=torch.int16, device=cols.device)
    _lib.check(lib.rt_column_order_device(cols.data_ptr(), pad.data_ptr(), b, s, out.data_ptr(),
                                          _stream_ptr(cols.device)), "rt_column_order_device")
    return out


def build_attention_masks(batch: dict, max_rows: int | None = None, kinds=("feature", "neighbor",
                                                                              "column")):
    """Drop-in for model.py:201 ``build_attention_masks(batch, max_rows)``.

    Returns tile plans in the reference's order (outbound, inbound, column),
    each built under the permutation its sublayer uses (out_perm, in_perm,
    col_perm; layers.py:219-232). Pass ``kinds`` to add "full" (identity
    permutation)."""
    out = []
    b, s = batch["seq_row_ids"].shape
    for name in kinds:
        kind = MASK_KINDS[name]
        if kind == MASK_FEATURE:
            perm = batch["out_perm"]
        elif kind == MASK_NEIGHBOR:
            perm = batch["in_perm"]
        elif kind == MASK_COLUMN:
            perm = batch["col_perm"]
        else:
            perm = torch.arange(s, device=batch["seq_row_ids"].device,
                                dtype=torch.int32).to(torch.int16).expand(b, s)
        out.append(build_tile_plan(perm, batch["seq_row_ids"], batch["column_ids"],
                                   batch["is_padding"], batch["fk_adj"], kind, max_rows))
    return tuple(out)


def device_status(reset: bool = True) -> int:
    return _lib.load().rt_device_status(1 if reset else 0)


# ----------------------------------------------------------------------------
# attention core (layers.py:83-94) and its backward
# ----------------------------------------------------------------------------

def _check_qkv(q, k, v, plan: TilePlan):
    b, h, s, dh = q.shape
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(t, name, torch.bfloat16, (b, h, s, dh))
    if plan.batch != b or plan.seq_len != s:
        raise ValueError(f"plan built for batch={plan.batch}, seq_len={plan.seq_len}; "
                         f"got q of shape {tuple(q.shape)}")
    return b, h, s, dh


def attention_fwd(q, k, v, plan: TilePlan, scale: float | None = None, out=None, lse=None):
    """o, lse = masked softmax attention of already-normalised q_hat (tau folded
    in), k_hat, v: [B,H,S,Dh] bf16 in the plan's permuted token order."""
    b, h, s, dh = _check_qkv(q, k, v, plan)
    if scale is None:
        scale = 1.0 / math.sqrt(dh)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((b, h, s), dtype=torch.float32, device=q.device)
    _lib.check(_lib.load().rt_attention_fwd(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), b, h, s, dh, float(scale), ctypes.byref(plan.c),
        out.data_ptr(), lse.data_ptr(), _stream_ptr(q.device)), "rt_attention_fwd")
    return out, lse


def attention_bwd(q, k, v, o, lse, d_o, plan: TilePlan, scale: float | None = None,
                  dq=None, dk=None, dv=None, workspace=None):
    """dq, dk, dv of attention_fwd for upstream gradient d_o (bf16 outputs,
    fp32 accumulation)."""
    b, h, s, dh = _check_qkv(q, k, v, plan)
    _require_cuda(o, "o", torch.bfloat16, q.shape)
    _require_cuda(d_o, "d_o", torch.bfloat16, q.shape)
    _require_cuda(lse, "lse", torch.float32, (b, h, s))
    if scale is None:
        scale = 1.0 / math.sqrt(dh)
    lib = _lib.load()
    dq = torch.empty_like(q) if dq is None else dq
    dk = torch.empty_like(k) if dk is None else dk
    dv = torch.empty_like(v) if dv is None else dv
    ws_bytes = lib.rt_attention_bwd_workspace_bytes(b, h, s)
    if workspace is None:
        workspace = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=q.device)
    _lib.check(lib.rt_attention_bwd(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), d_o.data_ptr(), lse.data_ptr(),
        b, h, s, dh, float(scale), ctypes.byref(plan.c), dq.data_ptr(), dk.data_ptr(),
        dv.data_ptr(), workspace.data_ptr(), workspace.numel(), _stream_ptr(q.device)),
        "rt_attention_bwd")
    return dq, dk, dv


class RTAttentionFunction(torch.autograd.Function):
    """autograd wrapper: forward and backward are the library's kernels."""

    @staticmethod
    def forward(ctx, q, k, v, plan, scale):
        o, lse = attention_fwd(q, k, v, plan, scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.plan = plan
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, d_o):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = attention_bwd(q, k, v, o, lse, d_o.contiguous(), ctx.plan, ctx.scale)
        return dq, dk, dv, None, None


def rt_attention(q, k, v, plan: TilePlan, scale: float | None = None):
    """Masked attention core (layers.py:83-94) with autograd; q, k, v bf16
    [B,H,S,Dh] in the plan's permuted order, q already L2-normalised and
    multiplied by tau, k normalised."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    return RTAttentionFunction.apply(q, k, v, plan, scale)
