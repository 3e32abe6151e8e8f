"""The kernels' polynomial exp2 (rt_device.cuh, exp2_poly2): float32 emulation
of its exact steps -- clamp to [-125, 127], round-to-nearest by adding
1.5 * 2^23, f = x - n, degree-3 Horner in fp32, exponent add -- checked against
exp2 in float64. The coefficients below are the kernel's."""
import numpy as np

C1, C2, C3 = np.float32(0.6932829022407532), np.float32(0.24221095442771912), np.float32(0.05500892922282219)
ROUND = np.float32(12582912.0)


def exp2_poly(x):
    x = np.clip(np.asarray(x, dtype=np.float32), np.float32(-125.0), np.float32(127.0))
    t = (x + ROUND).astype(np.float32)
    n = (t - ROUND).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = (f * C3 + C2).astype(np.float32)
    p = (p * f + C1).astype(np.float32)
    p = (p * f + np.float32(1.0)).astype(np.float32)
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    return bits.astype(np.int32).view(np.float32)


def test_relative_error_over_the_softmax_range():
    x = np.linspace(-125.0, 127.0, 2_000_001, dtype=np.float32)
    got = exp2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1.0)
    assert rel.max() < 1.1e-4
    # far below the bf16 rounding (2^-9) that P goes through next
    assert rel.max() < 2.0 ** -9 / 16


def test_integer_and_half_integer_arguments():
    for k in range(-125, 128):
        for off in (0.0, 0.5, -0.5, 0.25):
            x = np.float32(k + off)
            if x < -125 or x > 127:
                continue
            assert abs(float(exp2_poly(x)) / 2.0 ** float(x) - 1.0) < 1.1e-4


def test_clamps_keep_results_finite_and_normal():
    out = exp2_poly(np.array([-np.inf, -1e30, -200.0, 200.0, 1e30, np.inf], dtype=np.float32))
    assert np.isfinite(out).all()
    assert (out > 0).all()
    tiny = np.finfo(np.float32).tiny
    assert out[:3].max() < 2.0 ** -124 and out[:3].min() >= tiny  # masked entries: about 2^-125, normal
    assert out[3:].min() > 2.0 ** 126  # past the forward's 2^100 row-sum guard
