"""Shared case construction for the GPU parity tests: seeded metadata and
q/k/v/dO from the oracle's generator, uploaded as the library expects."""
from __future__ import annotations

import numpy as np

from oracle import rt_oracle as orc

# max-relative tolerance for outputs and gradients, absolute for lse
# (bf16 inputs/outputs, fp32 accumulation)
TOL_OUT = 2e-2
TOL_LSE = 1e-3


def max_rel(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / denom)


def to_dev_batch(bt):
    import torch
    out = {}
    for k, v in bt.items():
        v = np.ascontiguousarray(v)
        if v.dtype == np.uint16:
            out[k] = torch.from_numpy(v.view(np.int16)).cuda()
        else:
            out[k] = torch.from_numpy(v).cuda()
    return out


def bf16_tensor(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(orc.to_bf16_bits(x)).view(np.int16)).cuda().view(
        torch.bfloat16)


def from_bf16_tensor(t):
    import torch
    return orc.from_bf16_bits(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


class Case:
    """One attention problem: metadata batch, mask kind, bf16-rounded inputs,
    the oracle's permuted dense mask, and the device plan."""

    def __init__(self, gen, kind, h, dh, seed, scale=None):
        import torch
        from tributary_b200.attention import build_tile_plan
        self.bt = orc.make_batch(*gen)
        self.kind = kind
        b, s = self.bt["seq_row_ids"].shape
        self.b, self.h, self.s, self.dh = b, h, s, dh
        self.scale = 1.0 / np.sqrt(dh) if scale is None else scale
        q, k, v, do = orc.make_qkv(seed, b, h, s, dh)
        self.q, self.k, self.v, self.do = (orc.round_bf16(x) for x in (q, k, v, do))
        perm = orc.perm_for_kind(self.bt, kind)
        mask = orc.mask_for_kind(kind, self.bt["seq_row_ids"], self.bt["fk_adj"],
                                 self.bt["column_ids"], self.bt["is_padding"])
        self.mask_perm = orc.permute_mask(mask, perm)
        dev = to_dev_batch(self.bt)
        perm_d = torch.from_numpy(np.ascontiguousarray(perm).view(np.int16)).cuda()
        self.plan = build_tile_plan(perm_d, dev["seq_row_ids"], dev["column_ids"],
                                    dev["is_padding"], dev["fk_adj"], kind)
        self.qd, self.kd, self.vd, self.dod = (bf16_tensor(x) for x in
                                               (self.q, self.k, self.v, self.do))

    def oracle_fwd(self):
        return orc.attention_fwd(self.q, self.k, self.v, self.mask_perm, self.scale,
                                 dtype=np.float64)

    def oracle_bwd(self, o=None):
        if o is None:
            o, _ = self.oracle_fwd()
        return orc.attention_bwd(self.q, self.k, self.v, o, self.do, self.mask_perm,
                                 self.scale, dtype=np.float64)
