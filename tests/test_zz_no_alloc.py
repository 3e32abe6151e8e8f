"""rt_attention_bwd_noalloc: the backward for callers that cannot allocate.

Callers such as a plugin host or FFI handler with no scratch-allocation hook,
or a service that may not call cudaMalloc after start-up, cannot hand
rt_attention_bwd its workspace; this entry point keeps that workspace in a
fixed array inside the library. These tests call it through the C ABI and
compare it with rt_attention_bwd on the same inputs and with the float64
oracle's gradients, for consecutive calls on different problems (the array
keeps the previous call's contents).

The file name makes pytest collect it last.
"""
import ctypes

import pytest

from rt_cases import TOL_GRAD_ROW, TOL_OUT, Case, from_bf16_tensor, max_rel, row_rel

pytestmark = pytest.mark.gpu


def _noalloc_bwd(lib, c, o, lse):
    import torch
    dq, dk, dv = (torch.full_like(c.qd, float("nan")) for _ in range(3))
    st = lib.rt_attention_bwd_noalloc(
        c.qd.data_ptr(), c.kd.data_ptr(), c.vd.data_ptr(), o.data_ptr(), c.dod.data_ptr(),
        lse.data_ptr(), c.b, c.h, c.s, c.dh, float(c.scale), ctypes.byref(c.plan.c),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return st, (dq, dk, dv)


def test_noalloc_backward_matches_workspace_backward(cuda_lib):
    import torch
    from tributary_b200 import _lib
    from tributary_b200.attention import attention_bwd, attention_fwd, device_status
    lib = _lib.load()
    cases = [
        Case((61, 2, 1000, 6, 4, 16, 0.7, 0.1), 1, h=3, dh=64, seed=71),
        Case((62, 4, 256, 3, 4, 8, 0.6, 0.05), 3, h=2, dh=32, seed=72),
    ]
    cases.append(cases[0])  # a third call back on the first problem
    oracle = {}
    for c in cases:
        o, lse = attention_fwd(c.qd, c.kd, c.vd, c.plan, c.scale)
        want = attention_bwd(c.qd, c.kd, c.vd, o, lse, c.dod, c.plan, c.scale)
        st, got = _noalloc_bwd(lib, c, o, lse)
        _lib.check(st, "rt_attention_bwd_noalloc")
        torch.cuda.synchronize()
        assert device_status() == 0
        if id(c) not in oracle:
            oracle[id(c)] = c.oracle_bwd()
        for name, g, w, r in zip(("dq", "dk", "dv"), got, want, oracle[id(c)]):
            gv = from_bf16_tensor(g)
            assert max_rel(gv, from_bf16_tensor(w)) < TOL_OUT, name
            assert max_rel(gv, r) < TOL_OUT, name
            assert row_rel(gv, r) < TOL_GRAD_ROW, name


def test_noalloc_backward_rejects_problems_beyond_its_array(cuda_lib):
    from tributary_b200 import _lib
    lib = _lib.load()
    plan = _lib.RtTilePlan()
    fake = ctypes.c_void_p(1 << 21)
    # 8 * 16 * 16384 padded query rows = 2^21 > 2^20
    st = lib.rt_attention_bwd_noalloc(fake, fake, fake, fake, fake, fake, 8, 16, 16384, 64, 0.125,
                                      ctypes.byref(plan), fake, fake, fake, None)
    assert st == _lib.RT_ERR_WORKSPACE
