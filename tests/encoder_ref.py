"""Test helpers for the RT encoder: a dense fp32 masked attention with the
reference's semantics (confluence/confluence/layers.py:83-97), dense permuted
masks from the oracle, and batch conversion. Used as the encoder's attention
in CPU tests (gloo ranks) and as the comparison in the GPU tests."""
import numpy as np
import torch
import torch.nn.functional as F

from oracle import rt_oracle as orc
from tributary_b200 import batch as rb
from tributary_b200.encoder import EncoderConfig

ARRAY_KEYS = ("seq_row_ids", "column_ids", "is_padding", "fk_adj", "col_perm", "out_perm", "in_perm", "stypes",
              "numeric_values", "timestamp_values", "bool_values", "categorical_ids", "text_ids", "text_vectors",
              "is_null", "is_target")


def dense_attention(q, k, v, mask, scale):
    s = torch.einsum("bhid,bhjd->bhij", q.float(), k.float()) * scale
    s = torch.where(mask[:, None], s, torch.full_like(s, -1e9))
    return torch.einsum("bhij,bhjd->bhid", torch.softmax(s, -1), v.float()).to(q.dtype)


def inverse_order(order):
    inv = torch.empty_like(order)
    return inv.scatter_(1, order, torch.arange(order.shape[1], device=order.device).expand_as(order))


class RefOps:
    """The sublayer's token preparation and attention in plain torch with the
    reference's semantics (layers.py:63-97, 139-167); ``order`` is the int64
    cell order, ``ctx`` the dense permuted mask."""

    @staticmethod
    def qk_prepare(qkv, order, tau, heads, head_dim):
        b, s, w = qkv.shape
        x = torch.gather(qkv, 1, order[:, :, None].expand(b, s, w))
        x = x.view(b, s, 3, heads, head_dim).permute(2, 0, 3, 1, 4)
        q, k = x[0].float(), x[1].float()
        q = q / q.norm(dim=-1, keepdim=True).clamp_min(1e-6) * tau.view(1, heads, 1, 1)
        k = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-6)
        return q.to(qkv.dtype), k.to(qkv.dtype), x[2].contiguous()

    attention = staticmethod(dense_attention)

    @staticmethod
    def heads_unpermute(o, order):
        b, h, s, dh = o.shape
        o = o.permute(0, 2, 1, 3).reshape(b, s, h * dh)
        inv = inverse_order(order)
        return torch.gather(o, 1, inv[:, :, None].expand(b, s, h * dh))

    # the layer norm, gated residual and SwiGLU activation in plain torch
    # (layers.py:16-30, 170-174, 177-200)
    @staticmethod
    def rms_norm(x, gamma, eps):
        y = F.rms_norm(x.float(), (x.shape[-1],), 1.0 + gamma, eps)
        if torch.is_autocast_enabled(x.device.type):  # the output only feeds matmuls
            y = y.to(torch.get_autocast_dtype(x.device.type))
        return y

    @staticmethod
    def gate_residual(x, out, gate, scale):
        return x + (out * scale * torch.sigmoid(gate)).float()

    @staticmethod
    def swiglu(u):
        f = u.shape[-1] // 2
        return F.silu(u[..., :f]) * u[..., f:]

    @staticmethod
    def residual_add(x, h, scale):
        return x + (h * scale).float()


def tiny_config(**kw):
    base = dict(d_model=64, n_heads=1, d_head=64, d_ff=128, n_layers=1, d_text=16, d_time=8, max_categories=16)
    base.update(kw)
    return EncoderConfig(**base)


def make_cells(seed, B=2, S=128, **kw):
    kw.setdefault("d_text", 16)
    return rb.make_cells(seed, B, S, 3, 4, 8, 0.6, 0.05, n_categories=64, max_categories=16, **kw)


def to_torch(cells, device):
    out = {}
    for k in ARRAY_KEYS:
        a = cells[k]
        if a.dtype == np.uint16:
            a = a.astype(np.int32)
        out[k] = torch.from_numpy(np.ascontiguousarray(a)).to(device)
    for k in ("target_stype", "cat_start"):
        out[k] = cells[k]
    col = torch.from_numpy(cells["col_table"]).to(device)
    cat = torch.from_numpy(cells["cat_table"]).to(device)
    return out, col, cat


def dense_masks(cells, kinds, device):
    """(int64 cell order, dense permuted mask) per kind, from the oracle."""
    out = []
    for kind in kinds:
        perm = rb.order_for_kind(cells, kind)
        m = orc.mask_for_kind(kind, cells["seq_row_ids"], cells["fk_adj"], cells["column_ids"], cells["is_padding"])
        mp = torch.from_numpy(orc.permute_mask(m, perm)).to(device)
        o = torch.from_numpy(perm.astype(np.int64)).to(device)
        out.append((o, mp))
    return out
