"""Shared case construction for the GPU parity tests: seeded metadata and
q/k/v/dO from the oracle's generator, uploaded as the library expects."""
from __future__ import annotations

import numpy as np

from oracle import rt_oracle as orc

# max-relative tolerance for outputs and gradients, absolute for lse
# (bf16 inputs/outputs, fp32 accumulation)
TOL_OUT = 2e-2
TOL_LSE = 1e-3
# row by row (row_rel), gradients: the backward forms delta = rowsum(dO * O)
# from the bf16 O the forward returned, as the reference's autodiff does from
# its fp32 o. A query with two live keys has dq = p1 p2 (dp1 - dp2)(k1 - k2)
# scale, which can be a few percent of the tensor's RMS while the bf16
# rounding of O moves delta by ~2^-9 |dO| |O|; a float32 emulation of these
# steps gives row errors of 2% at Dh = 32 against the float64 oracle, so
# gradient rows are held to 5e-2 (outputs o stay at 2e-2).
TOL_GRAD_ROW = 5e-2


def max_rel(got, ref):
    """Largest absolute error over the tensor, relative to its largest |ref|."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / denom)


def row_rel(got, ref):
    """Largest error of each row (last axis: one query's output or gradient
    vector), relative to that row's own largest |ref|, maximised over rows.
    Rows far below the tensor's typical magnitude (padding keys, whose dk is
    exactly 0, or gradients that cancel) are measured against the tensor's
    RMS instead, so that max_rel's whole-tensor normalisation cannot hide an
    error confined to small rows."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    floor = max(float(np.sqrt(np.mean(ref * ref))), 1e-30)
    denom = np.maximum(np.abs(ref).max(axis=-1), floor)
    return float((np.abs(got - ref).max(axis=-1) / denom).max())


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

    def oracle_by_head(self, bwd=True, rows=1024):
        """The float64 oracle one (b, h) at a time, over blocks of `rows`
        queries, so that host memory stays bounded at long sequence lengths:
        o and lse per block are the oracle's forward on those queries against
        all keys; dq per block, and dk / dv summed over the blocks (both are
        sums over queries), are the oracle's backward. The (b, h) problems run
        on a pool of host threads. Returns o, lse and, with bwd, dq, dk, dv as
        float64 arrays."""
        import os
        from concurrent.futures import ThreadPoolExecutor

        from threadpoolctl import threadpool_limits
        b_, h_, s, dh = self.q.shape
        o = np.empty((b_, h_, s, dh))
        lse = np.empty((b_, h_, s))
        grads = [np.zeros((b_, h_, s, dh)) for _ in range(3)] if bwd else None

        def one(bh):
            b, h = bh
            sel = (slice(b, b + 1), slice(h, h + 1))
            k, v = self.k[sel], self.v[sel]
            for r0 in range(0, s, rows):
                r = slice(r0, min(s, r0 + rows))
                q = self.q[sel + (r,)]
                m = self.mask_perm[b:b + 1, r]
                ob, lb = orc.attention_fwd(q, k, v, m, self.scale, dtype=np.float64)
                o[b, h, r], lse[b, h, r] = ob[0, 0], lb[0, 0]
                if bwd:
                    dq, dk, dv = orc.attention_bwd(q, k, v, ob, self.do[sel + (r,)], m,
                                                   self.scale, dtype=np.float64)
                    grads[0][b, h, r] = dq[0, 0]
                    grads[1][b, h] += dk[0, 0]
                    grads[2][b, h] += dv[0, 0]

        workers = max(1, min(8, len(os.sched_getaffinity(0))))
        with threadpool_limits(limits=1), ThreadPoolExecutor(max_workers=workers) as pool:
            list(pool.map(one, [(b, h) for b in range(b_) for h in range(h_)]))
        return (o, lse) + (tuple(grads) if bwd else ())


def per_head_errors(got, ref):
    """(max over heads of max_rel per (b, h), row_rel over the tensor)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    worst = 0.0
    for b in range(ref.shape[0]):
        for h in range(ref.shape[1]):
            worst = max(worst, max_rel(got[b, h], ref[b, h]))
    return worst, row_rel(got, ref)
