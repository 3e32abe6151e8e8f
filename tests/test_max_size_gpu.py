"""The largest supported problem: S = 65536 (T = 512 tiles per side, every
order value of the uint16 range, 512-entry tile lists), full kind without
padding (every tile fully live), B = H = 1, Dh = 64. The plan must list all
T^2 tiles as full; o and lse at sampled query rows, dq there, and dk / dv at
sampled key rows are checked against the exact attention (model.py:227-262
with every element live; layers.py:82-97), computed in float64 from the
bf16 inputs, the row log-sum-exps of all queries coming from chunked float32
products on the GPU."""
import math

import numpy as np
import pytest
import torch

from rt_cases import TOL_LSE, TOL_OUT, max_rel

pytestmark = pytest.mark.gpu

S, DH = 65536, 64


def test_full_kind_at_the_maximum_sequence_length(cuda_lib):
    from tributary_b200.attention import attention_bwd, attention_fwd, build_tile_plan, device_status
    dev = "cuda"
    order = torch.arange(S, dtype=torch.int32).to(torch.int16).view(1, S).to(dev)  # 0..65535 as uint16
    zeros16 = torch.zeros(1, S, dtype=torch.int16, device=dev)
    cols = torch.zeros(1, S, dtype=torch.int32, device=dev)
    pad = torch.zeros(1, S, dtype=torch.uint8, device=dev)
    fk = torch.zeros(1, 1, 1, dtype=torch.uint8, device=dev)
    plan = build_tile_plan(order, zeros16, cols, pad, fk, 3)
    T = S // 128
    assert plan.nnz() == T * T
    n_ptr, idx = plan.q2k()
    n_ptr = n_ptr.cpu().numpy()
    assert np.all(np.diff(n_ptr) == T)
    assert np.all(idx.cpu().numpy()[:T * T] < 0)  # bit 31: fully live

    g = torch.Generator(device="cpu").manual_seed(65536)
    q = torch.randn(1, 1, S, DH, generator=g)
    k = torch.randn(1, 1, S, DH, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True) * 4.0).to(torch.bfloat16).to(dev)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16).to(dev)
    v = torch.randn(1, 1, S, DH, generator=g).to(torch.bfloat16).to(dev)
    do = torch.randn(1, 1, S, DH, generator=g).to(torch.bfloat16).to(dev)
    scale = 1.0 / math.sqrt(DH)
    o, lse = attention_fwd(q, k, v, plan, scale)
    dq, dk, dv = attention_bwd(q, k, v, o, lse, do, plan, scale)
    torch.cuda.synchronize()
    assert device_status() == 0

    qf, kf, vf, dof = (t[0, 0].float() for t in (q, k, v, do))
    # log-sum-exp of every query row (needed for dk, dv), float32 on the GPU in chunks
    lse_all = torch.empty(S, device=dev)
    for r0 in range(0, S, 4096):
        lse_all[r0:r0 + 4096] = torch.logsumexp(qf[r0:r0 + 4096] @ kf.T * scale, dim=-1)
    rows = np.array([0, 1, 127, 128, 30000, 40961, 65534, 65535])
    K = kf.double().cpu().numpy()
    V = vf.double().cpu().numpy()
    Q = qf.double().cpu().numpy()
    dO = dof.double().cpu().numpy()
    o_cpu = o[0, 0].float().double().cpu().numpy()
    for i in rows:  # o, lse, dq of query row i against all keys, float64
        s = K @ Q[i] * scale
        m = s.max()
        p = np.exp(s - m)
        l_ref = m + math.log(p.sum())
        p /= p.sum()
        o_ref = p @ V
        delta = float(dO[i] @ o_cpu[i])  # the backward's delta uses the returned (bf16) o
        dq_ref = (p * (V @ dO[i] - delta)) @ K * scale
        assert abs(float(lse[0, 0, i]) - l_ref) < TOL_LSE, i
        assert max_rel(o[0, 0, i].float().cpu().numpy(), o_ref) < TOL_OUT, i
        assert max_rel(dq[0, 0, i].float().cpu().numpy(), dq_ref) < TOL_OUT, i
    # dk, dv of key row j: sums over all 65536 queries, float64 from the float32 lse
    L = lse_all.double().cpu().numpy()
    delta_all = (dof.double() * o[0, 0].double()).sum(-1).cpu().numpy()
    for j in rows:
        p = np.exp(Q @ K[j] * scale - L)  # column j of P
        dv_ref = p @ dO
        dk_ref = (p * (dO @ V[j] - delta_all)) @ Q * scale
        assert max_rel(dv[0, 0, j].float().cpu().numpy(), dv_ref) < TOL_OUT, j
        assert max_rel(dk[0, 0, j].float().cpu().numpy(), dk_ref) < TOL_OUT, j
