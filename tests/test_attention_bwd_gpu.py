"""Backward kernels parity against the oracle's analytic gradients (which
tests/test_oracle.py pins to finite differences of the reference-pinned
forward): dq, dk, dv within 2e-2 max-relative."""
import numpy as np
import pytest

from rt_cases import TOL_GRAD_ROW, TOL_OUT, Case, from_bf16_tensor, max_rel, per_head_errors, row_rel

pytestmark = pytest.mark.gpu

GENS = {
    "cfgA": (51, 4, 256, 3, 4, 8, 0.6, 0.05),
    "ragged_s200": (52, 2, 200, 4, 2, 9, 0.8, 0.2),
    "s1000": (53, 2, 1000, 6, 4, 16, 0.7, 0.1),
    "s1024_dense_fk": (54, 1, 1024, 2, 3, 5, 1.0, 0.0),
}


def run_fwd_bwd(c):
    from tributary_b200.attention import attention_bwd, attention_fwd, device_status
    o, lse = attention_fwd(c.qd, c.kd, c.vd, c.plan, c.scale)
    dq, dk, dv = attention_bwd(c.qd, c.kd, c.vd, o, lse, c.dod, c.plan, c.scale)
    assert device_status() == 0
    return o, lse, dq, dk, dv


@pytest.mark.parametrize("dh", [32, 64])
@pytest.mark.parametrize("kind", [0, 1, 2, 3], ids=["column", "feature", "neighbor", "full"])
@pytest.mark.parametrize("gen", sorted(GENS))
def test_backward_matches_oracle(cuda_lib, gen, kind, dh):
    c = Case(GENS[gen], kind, h=2, dh=dh, seed=2000 + 10 * kind + dh + len(gen))
    _, _, dq, dk, dv = run_fwd_bwd(c)
    dq_ref, dk_ref, dv_ref = c.oracle_bwd()
    for name, got, ref in (("dq", dq, dq_ref), ("dk", dk, dk_ref), ("dv", dv, dv_ref)):
        g = from_bf16_tensor(got)
        assert np.isfinite(g).all(), name
        err = max_rel(g, ref)
        assert err < TOL_OUT, (name, err)
        err = row_rel(g, ref)
        assert err < TOL_GRAD_ROW, (name, "row", err)


def _same_up_to_dq_order(r1, r2):
    """o, lse, dk and dv are written once per element: bit-identical across
    runs. dQ sums one fp32 partial per live key tile through vector
    reductions whose order the memory system decides, so two runs may differ
    by fp32 rounding -- at most one bf16 unit in the last place after the
    final rounding."""
    import torch
    for i, (a, b) in enumerate(zip(r1, r2)):
        if a is None:
            continue
        if i == 2:  # dq
            af, bf = from_bf16_tensor(a), from_bf16_tensor(b)
            assert np.all(np.abs(af - bf) <= 2.0 ** -7 * np.maximum(np.abs(af), np.abs(bf)) + 1e-30)
        else:
            assert torch.equal(a, b)


def test_backward_deterministic(cuda_lib):
    c = Case(GENS["s1000"], 2, h=3, dh=64, seed=7)
    _same_up_to_dq_order(run_fwd_bwd(c), run_fwd_bwd(c))


def test_autograd_function_uses_kernels(cuda_lib):
    import torch
    from tributary_b200.attention import attention_bwd, attention_fwd, rt_attention
    c = Case(GENS["cfgA"], 1, h=2, dh=32, seed=8)
    q = c.qd.clone().requires_grad_(True)
    k = c.kd.clone().requires_grad_(True)
    v = c.vd.clone().requires_grad_(True)
    o = rt_attention(q, k, v, c.plan, c.scale)
    o.backward(c.dod)
    o2, lse = attention_fwd(c.qd, c.kd, c.vd, c.plan, c.scale)
    dq, dk, dv = attention_bwd(c.qd, c.kd, c.vd, o2, lse, c.dod, c.plan, c.scale)
    assert torch.equal(o.detach(), o2)
    assert torch.equal(k.grad, dk) and torch.equal(v.grad, dv)
    _same_up_to_dq_order((None, None, q.grad), (None, None, dq))


def test_gradient_of_padding_keys_only_from_diagonal(cuda_lib):
    """A padding key is seen only by its own (padding) query, whose p == 1:
    dv_j = do_j and dk_j = 0 (ds = p (dp - delta) = 0 when p == 1)."""
    from oracle import rt_oracle as orc
    c = Case((55, 1, 384, 2, 3, 5, 0.5, 0.3), 1, h=2, dh=64, seed=9)
    _, _, _, dk, dv = run_fwd_bwd(c)
    perm = orc.perm_for_kind(c.bt, 1)
    pad = c.bt["is_padding"][0][perm[0]].astype(bool)
    np.testing.assert_allclose(from_bf16_tensor(dv)[0][:, pad], c.do[0][:, pad], rtol=1e-2, atol=1e-2)
    assert np.abs(from_bf16_tensor(dk)[0][:, pad]).max() < 1e-2


def test_entry_points_work_from_a_worker_thread(cuda_lib):
    """Frameworks call kernels from their own threads (autograd workers, XLA
    FFI callbacks) that may have no current CUDA context yet."""
    import threading
    c = Case(GENS["cfgA"], 0, h=2, dh=64, seed=10)
    ref = run_fwd_bwd(c)
    out = {}

    def work():
        try:
            out["r"] = run_fwd_bwd(c)
        except Exception as e:  # pragma: no cover - reported below
            out["e"] = e

    t = threading.Thread(target=work)
    t.start()
    t.join()
    assert "e" not in out, out.get("e")
    _same_up_to_dq_order(ref, out["r"])


def test_backward_repeated_under_concurrent_copies(cuda_lib):
    """The fused backward's dQ reduce warps run behind the MMA issuer by up to a
    tile; every barrier phase must still be taken by each of its waiters before
    the next one completes. Repeat dense many-tile calls while a large copy runs
    on another stream (which shifts the timing) and require a clean device
    status, identical dK / dV every time, and dQ within tolerance of the
    float64 oracle head by head and row by row (a lost partial would move a
    whole row)."""
    import torch
    from tributary_b200.attention import attention_bwd, attention_fwd, device_status
    c = Case((56, 2, 2048, 3, 4, 8, 0.7, 0.0), 3, h=4, dh=64, seed=11)
    o, lse = attention_fwd(c.qd, c.kd, c.vd, c.plan, c.scale)
    ref = attention_bwd(c.qd, c.kd, c.vd, o, lse, c.dod, c.plan, c.scale)
    assert device_status() == 0
    dq_oracle = c.oracle_by_head()[2]
    side = torch.cuda.Stream()
    src = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    host = torch.empty(64 << 20, dtype=torch.uint8).pin_memory()
    for it in range(12):
        with torch.cuda.stream(side):
            if it % 2:
                host.copy_(src, non_blocking=True)
            else:
                src.copy_(host, non_blocking=True)
        dq, dk, dv = attention_bwd(c.qd, c.kd, c.vd, o, lse, c.dod, c.plan, c.scale)
        torch.cuda.synchronize()
        assert device_status() == 0, it
        assert torch.equal(dk, ref[1]) and torch.equal(dv, ref[2]), it
        head_err, row_err = per_head_errors(from_bf16_tensor(dq), dq_oracle)
        assert head_err < TOL_OUT and row_err < TOL_GRAD_ROW, (it, head_err, row_err)
        # and against the first call: reduction order moves an element by at
        # most about one bf16 unit of its own size
        err = max_rel(from_bf16_tensor(dq), from_bf16_tensor(ref[0]))
        assert err < 2.0 ** -7, (it, err)


@pytest.mark.parametrize("dh", [32, 64])
def test_backward_dq_complete_when_the_call_returns(cuda_lib, dh):
    """dQ is summed by asynchronous TMA reduce-adds into an fp32 buffer that
    the next kernel on the stream converts to bf16; every addition must have
    landed by then. A small case, where all blocks finish at about the same
    time, is where an addition still in flight at the end of the fused kernel
    would show, so it runs many times against the oracle."""
    from tributary_b200.attention import attention_bwd, attention_fwd, device_status
    c = Case(GENS["cfgA"], 0, h=2, dh=dh, seed=2004 + dh)
    dq_ref = c.oracle_bwd()[0]
    o, lse = attention_fwd(c.qd, c.kd, c.vd, c.plan, c.scale)
    for it in range(40):
        dq, _, _ = attention_bwd(c.qd, c.kd, c.vd, o, lse, c.dod, c.plan, c.scale)
        assert device_status() == 0, it
        err = max_rel(from_bf16_tensor(dq), dq_ref)
        assert err < TOL_OUT, (it, err)
