"""Device-side failure path, exercised without a fault: a bounded wait that
runs out (on an mbarrier nothing arrives at) must end its kernel through the
abort flag, free tensor memory, raise the sticky RT_ERR_TIMEOUT status that
rt_device_status() reads, and leave the context usable for the next call."""
import ctypes

import numpy as np
import pytest

from rt_cases import TOL_OUT, Case, from_bf16_tensor, max_rel

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_reports_timeout_and_context_survives(cuda_lib):
    import torch
    from tributary_b200 import _lib
    from tributary_b200.attention import attention_fwd, device_status
    lib = _lib.load()
    assert device_status(reset=True) == 0
    report = torch.zeros(4, dtype=torch.int32, device="cuda")
    limit = 200_000_000  # SM clocks, about 0.1 s
    try:
        st = lib.rt_selftest_bounded_wait(limit, ctypes.c_void_p(report.data_ptr()),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        _lib.check(st, "rt_selftest_bounded_wait")
        status = device_status(reset=False)
    finally:
        device_status(reset=True)  # the sticky status must not leak into later tests
    assert status == _lib.RT_ERR_TIMEOUT
    abort, gave_up, waited, others = report.cpu().tolist()
    assert abort == 1 and gave_up == 3
    # the running-out wait took its limit; the others left through the abort
    # flag long before their own (ten times longer) limit
    assert limit // 1_000_000 <= waited < 3 * limit // 1_000_000
    assert others < 3 * limit // 1_000_000
    assert device_status(reset=False) == 0
    # tensor memory was freed and the context works: a normal forward runs
    c = Case((91, 2, 384, 3, 4, 8, 0.6, 0.05), 3, h=2, dh=64, seed=91)
    o, lse = attention_fwd(c.qd, c.kd, c.vd, c.plan, c.scale)
    assert device_status() == 0
    o_ref, _ = c.oracle_fwd()
    assert max_rel(from_bf16_tensor(o), o_ref) < TOL_OUT


def test_selftest_rejects_bad_arguments(cuda_lib):
    import torch
    from tributary_b200 import _lib
    lib = _lib.load()
    report = torch.zeros(4, dtype=torch.int32, device="cuda")
    assert lib.rt_selftest_bounded_wait(0, ctypes.c_void_p(report.data_ptr()), None) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_selftest_bounded_wait(10**12, ctypes.c_void_p(report.data_ptr()), None) == \
        _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_selftest_bounded_wait(1000, None, None) == _lib.RT_ERR_INVALID_ARGUMENT
