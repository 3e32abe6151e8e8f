"""Relational Transformer encoder: the training-step caller of the masked
attention kernels.

PyTorch restatement of confluence/confluence/model.py and layers.py:
  value encoder (model.py:46-177)  ->  n_layers x [gated attention sublayer
  per mask kind (layers.py:114-174) + SwiGLU FFN (layers.py:177-200)]  ->
  final RMSNorm  ->  decoder heads (model.py:180-210); loss per
  confluence/confluence/loss.py:33-170.

Each layer runs one attention sublayer per mask kind in ``kinds`` (the
reference uses feature/outbound, neighbor/inbound, column; the benchmark's
full-step configuration cycles column -> feature -> neighbor -> full). Inside a
sublayer, attention runs in the kind's cell order (layers.py:139-167): the QKV
projection is applied in token order (a per-token linear map commutes with the
gather), then one kernel gathers, splits heads and L2-normalises q and k with
tau (rt_qk_prepare), the attention kernels run under the kind's tile plan, and
one kernel returns the output to token order (rt_heads_unpermute). In the
backward, one call (rt_attention_bwd_qkv) runs the attention backward with the
normalisation's Jacobian and the scatter back to token order in its epilogues.

Matmuls run under bf16 autocast with fp32 parameters and an fp32 residual
stream; norms, QK normalisation and softmax statistics are computed in fp32
(layers.py:63-80), the attention kernels take bf16 q_hat * tau, k_hat, v and
accumulate in fp32.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import rt_attention

STYPE_IDENTIFIER, STYPE_NUMERICAL, STYPE_TIMESTAMP, STYPE_BOOLEAN = 0, 1, 2, 3
STYPE_CATEGORICAL, STYPE_TEXT, STYPE_IGNORED = 4, 5, 6
NUM_STYPES = 7


@dataclass
class EncoderConfig:
    d_model: int = 512
    n_heads: int = 8
    d_head: int = 64
    d_ff: int = 1536
    n_layers: int = 12
    d_text: int = 384          # frozen column-name / categorical / text embedding width
    d_time: int = 8            # timestamp feature width
    rms_eps: float = 1e-6
    max_categories: int = 256  # categorical loss: size of the target column's category set
    z_loss_weight: float = 1e-4
    huber_delta: float = 1.0
    ts_scalar_weight: float = 2.0
    kinds: tuple = field(default_factory=lambda: (0, 1, 2, 3))  # column, feature, neighbor, full


class ZeroCenteredRMSNorm(nn.Module):
    """(1 + gamma) * x / sqrt(mean(x^2) + eps), gamma initialised to 0
    (layers.py:16-30), computed by ``ops.rms_norm`` (the output only feeds
    matmuls: bf16 under autocast)."""

    def __init__(self, d: int, eps: float):
        super().__init__()
        self.gamma = nn.Parameter(torch.zeros(d))
        self.eps = eps

    def forward(self, x, ops):
        return ops.rms_norm(x, self.gamma, self.eps)


class KernelOps:
    """The encoder's token preparation, attention and fused layer kernels on
    the library: ``order`` is the [B,S] int16 cell order, ``ctx`` the
    TilePlan; rms_norm, gate_residual and swiglu are one kernel each way, and
    qk_attention is token preparation + attention with one fused backward."""

    @staticmethod
    def rms_norm(x, gamma, eps):
        from .layer_ops import rms_norm
        return rms_norm(x, gamma, eps)

    @staticmethod
    def gate_residual(x, out, gate, scale):
        from .layer_ops import gate_residual
        return gate_residual(x, out, gate, scale)

    @staticmethod
    def swiglu(u):
        from .layer_ops import swiglu
        return swiglu(u)

    @staticmethod
    def residual_add(x, h, scale):
        from .layer_ops import residual_add
        return residual_add(x, h, scale)

    @staticmethod
    def qk_prepare(qkv, order, tau, heads, head_dim):
        from .tokens import qk_prepare
        return qk_prepare(qkv, order, tau, heads, head_dim)

    @staticmethod
    def attention(q, k, v, ctx, scale):
        return rt_attention(q, k, v, ctx, scale)

    @staticmethod
    def qk_attention(qkv, order, tau, heads, head_dim, ctx, scale):
        from .tokens import qk_attention
        return qk_attention(qkv, order, tau, heads, head_dim, ctx, scale)

    @staticmethod
    def heads_unpermute(o, order):
        from .tokens import heads_unpermute
        return heads_unpermute(o, order)


def _xavier(lin: nn.Linear):
    nn.init.xavier_uniform_(lin.weight)
    return lin


class GatedAttention(nn.Module):
    """RMSNorm -> gather into the kind's cell order -> QK-normalised MHA ->
    scatter back -> sigmoid gate -> residual (layers.py:33-174)."""

    def __init__(self, cfg: EncoderConfig, output_scale: float):
        super().__init__()
        d = cfg.d_model
        self.cfg = cfg
        self.norm = ZeroCenteredRMSNorm(d, cfg.rms_eps)
        self.qkv = nn.Linear(d, 3 * d, bias=False)
        self.tau = nn.Parameter(torch.full((cfg.n_heads,), math.sqrt(cfg.d_head)))
        self.wo = _xavier(nn.Linear(d, d, bias=False))
        self.w_gate = nn.Linear(d, d, bias=False)
        self.output_scale = output_scale

    def forward(self, x, order, mask_ctx, ops):
        cfg = self.cfg
        h, dh = cfg.n_heads, cfg.d_head
        x_norm = self.norm(x, ops)
        scale = 1.0 / math.sqrt(dh)
        if hasattr(ops, "qk_attention"):  # one backward for gather, QK norm and attention
            o = ops.qk_attention(self.qkv(x_norm), order, self.tau, h, dh, mask_ctx, scale)
        else:
            q, k, v = ops.qk_prepare(self.qkv(x_norm), order, self.tau, h, dh)
            o = ops.attention(q, k, v, mask_ctx, scale)
        o = ops.heads_unpermute(o, order)
        if not torch.is_autocast_enabled(o.device.type):  # autocast feeds W_O bf16 as it is
            o = o.to(x.dtype)
        return ops.gate_residual(x, self.wo(o), self.w_gate(x_norm), self.output_scale)


class SwiGLU(nn.Module):
    """W_down (silu(W_gate x) * W_up x), no biases (layers.py:177-200); the
    gate and up projections run as one matmul whose [.., 2 d_ff] output
    ``ops.swiglu`` turns into the activation."""

    def __init__(self, cfg: EncoderConfig, output_scale: float):
        super().__init__()
        d, f = cfg.d_model, cfg.d_ff
        self.w_gate = nn.Linear(d, f, bias=False)
        self.w_up = nn.Linear(d, f, bias=False)
        self.w_down = nn.Linear(f, d, bias=False)
        self.output_scale = output_scale

    def forward(self, x, ops):
        """The FFN's output before its residual scale (EncoderLayer adds it)."""
        u = F.linear(x, torch.cat([self.w_gate.weight, self.w_up.weight], 0))
        return self.w_down(ops.swiglu(u))


class EncoderLayer(nn.Module):
    def __init__(self, cfg: EncoderConfig):
        super().__init__()
        scale = 1.0 / math.sqrt(4.0 * cfg.n_layers)  # residual-variance control (layers.py:220)
        self.attn = nn.ModuleList(GatedAttention(cfg, scale) for _ in cfg.kinds)
        self.ffn_norm = ZeroCenteredRMSNorm(cfg.d_model, cfg.rms_eps)
        self.ffn = SwiGLU(cfg, scale)

    def forward(self, x, masks, ops):
        for sub, (order, ctx) in zip(self.attn, masks):
            x = sub(x, order, ctx, ops)
        return ops.residual_add(x, self.ffn(self.ffn_norm(x, ops), ops), self.ffn.output_scale)


class ValueEncoder(nn.Module):
    """h0 = RMSNorm(column-name encoding + type-specific value encoding),
    with null and target replacement (model.py:46-177)."""

    def __init__(self, cfg: EncoderConfig):
        super().__init__()
        d, dt = cfg.d_model, cfg.d_text
        self.column_name = nn.Linear(dt, d)
        self.identifier = nn.Parameter(torch.randn(d) * 0.02)
        self.numerical = nn.Linear(1, d)
        self.timestamp = nn.Linear(cfg.d_time, d)
        self.boolean = nn.Parameter(torch.randn(2, d) * 0.02)
        self.categorical = nn.Linear(dt, d)
        self.text = nn.Linear(dt, d)
        self.null_emb = nn.Parameter(torch.randn(d) * 0.02)
        self.mask_emb = nn.Parameter(torch.randn(d) * 0.02)
        self.norm = ZeroCenteredRMSNorm(d, cfg.rms_eps)

    def forward(self, cells, col_table, cat_table, ops):
        col = self.column_name(col_table[cells["column_ids"]])
        vals = torch.stack([
            self.identifier.expand_as(col).to(col.dtype),
            self.numerical(cells["numeric_values"][..., None]),
            self.timestamp(cells["timestamp_values"]),
            (self.boolean[0] + cells["bool_values"][..., None].to(col.dtype) * (self.boolean[1] - self.boolean[0]))
            .to(col.dtype),
            self.categorical(cat_table[cells["categorical_ids"]]),
            self.text(cells["text_vectors"][cells["text_ids"]]),
            torch.zeros_like(col),
        ], dim=2)  # [B, S, 7, D]
        # each cell's own semantic-type slice (the one-hot contraction of the
        # reference picks exactly this row)
        sel = cells["stypes"].long().clamp(0, NUM_STYPES - 1)[..., None, None].expand(-1, -1, 1, vals.shape[-1])
        raw = torch.gather(vals, 2, sel).squeeze(2)
        is_null = cells["is_null"][..., None].to(raw.dtype)
        is_target = cells["is_target"][..., None].to(raw.dtype)
        v = is_null * self.null_emb.to(raw.dtype) + (1 - is_null) * raw
        v = is_target * self.mask_emb.to(raw.dtype) + (1 - is_target) * v
        return self.norm(col + v, ops).float()  # the residual stream stays fp32


class RTEncoder(nn.Module):
    """Value encoder -> layers -> final norm -> decoder heads (model.py:267-321).

    ``ops`` (qk_prepare, attention, heads_unpermute, rms_norm, gate_residual,
    swiglu, residual_add) defaults to the library kernels (KernelOps); each entry of ``masks`` passed to forward is
    (cell order, mask context) for one sublayer kind -- for KernelOps the
    int16 order and the kind's TilePlan (train.build_masks).
    """

    def __init__(self, cfg: EncoderConfig, ops=None):
        super().__init__()
        self.cfg = cfg
        self.ops = ops or KernelOps()
        self.value_encoder = ValueEncoder(cfg)
        self.layers = nn.ModuleList(EncoderLayer(cfg) for _ in range(cfg.n_layers))
        self.final_norm = ZeroCenteredRMSNorm(cfg.d_model, cfg.rms_eps)
        d = cfg.d_model
        self.null_head = nn.Linear(d, 1)
        self.numerical_head = nn.Linear(d, 1)
        self.boolean_head = nn.Linear(d, 1)
        self.timestamp_head = nn.Linear(d, cfg.d_time)
        self.categorical_head = nn.Linear(d, d)

    def forward(self, cells, masks, col_table, cat_table):
        x = self.value_encoder(cells, col_table, cat_table, self.ops)
        for layer in self.layers:
            x = layer(x, masks, self.ops)
        x = self.final_norm(x, self.ops)
        return {
            "null": self.null_head(x).squeeze(-1),
            "num": self.numerical_head(x).squeeze(-1),
            "bool": self.boolean_head(x).squeeze(-1),
            "ts": self.timestamp_head(x),
            "cat": self.categorical_head(x),
        }

    def loss(self, out, cells, cat_table):
        """Mean over target cells of null BCE + (1 - is_null) * the loss of the
        batch's target type (loss.py:33-170): Huber for numerical, BCE for
        boolean, Huber (cyclic dims averaged + weighted scalar) for
        timestamps, cross-entropy + z-loss over the target column's category
        set for categorical."""
        cfg = self.cfg
        f = {k: v.float() for k, v in out.items()}
        is_target = cells["is_target"].float()
        is_null = cells["is_null"].float()
        null_loss = F.binary_cross_entropy_with_logits(f["null"], is_null, reduction="none")
        num_loss = F.huber_loss(f["num"], cells["numeric_values"].float(), reduction="none", delta=cfg.huber_delta)
        bool_loss = F.binary_cross_entropy_with_logits(f["bool"], cells["bool_values"].float(), reduction="none")
        ts_err = F.huber_loss(f["ts"], cells["timestamp_values"].float(), reduction="none", delta=cfg.huber_delta)
        ts_loss = ts_err[..., :-1].mean(-1) + cfg.ts_scalar_weight * ts_err[..., -1]
        k = cfg.max_categories
        start = cells["cat_start"]
        cand = self.value_encoder.categorical(cat_table[start:start + k]).float()  # [K, D]
        logits = torch.einsum("bsd,kd->bsk", f["cat"], cand)
        tgt = (cells["categorical_ids"].long() - start).clamp(0, k - 1)
        lse = torch.logsumexp(logits, -1)
        cat_loss = lse - logits.gather(-1, tgt[..., None]).squeeze(-1) + cfg.z_loss_weight * lse.pow(2)
        type_loss = {STYPE_NUMERICAL: num_loss, STYPE_BOOLEAN: bool_loss, STYPE_TIMESTAMP: ts_loss,
                     STYPE_CATEGORICAL: cat_loss}[int(cells["target_stype"])]
        cell = null_loss + (1 - is_null) * type_loss
        return (cell * is_target).sum() / is_target.sum().clamp_min(1.0)
