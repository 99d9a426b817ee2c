"""The GPU kernels' GELU (erf by Abramowitz & Stegun eq. 7.1.28, evaluated in fp32)
restated in NumPy float32 with the same operation order, against the exact
erf-GELU (math.erf in float64) of the reference (F.gelu(approximate="none"))."""

import math

import numpy as np

A = [0.0705230784, 0.0422820123, 0.0092705272, 0.0001520143, 0.0002765672, 0.0000430638]


def gelu_as_f32(v):
    v = np.asarray(v, dtype=np.float32)
    u = np.abs(v) * np.float32(0.70710678118654752440)
    q = np.float32(A[5])
    for c in A[4::-1]:
        q = q * u + np.float32(c)
    q = q * u + np.float32(1.0)
    for _ in range(4):
        q = q * q
    with np.errstate(over="ignore", divide="ignore"):
        e = np.copysign(np.float32(1.0) - np.float32(1.0) / q, v)
    hv = np.float32(0.5) * v
    return hv * e + hv


def test_gelu_approximation_error_bound():
    xs = np.linspace(-12.0, 12.0, 240001)
    exact = np.array([0.5 * x * (1.0 + math.erf(x / math.sqrt(2.0))) for x in xs])
    err = np.abs(gelu_as_f32(xs).astype(np.float64) - exact)
    assert err.max() < 2e-6, err.max()
    # far tails: exactly x for large positive, exactly 0 for large negative
    assert gelu_as_f32(np.float32(40.0)) == np.float32(40.0)
    assert gelu_as_f32(np.float32(-40.0)) == np.float32(0.0)


C4 = [0.6931241750717163, 0.24024099111557007, 0.055906426161527634, 0.009582852944731712]


def exp2_poly_f32(x):
    """NumPy float32 restatement of the kernels' exp2_poly (ptx.cuh), same operation order."""
    x = np.maximum(np.asarray(x, np.float32), np.float32(-120.0))
    t = x + np.float32(12582912.0)
    n = t - np.float32(12582912.0)
    f = x - n
    q = np.float32(C4[3]) * f + np.float32(C4[2])
    q = q * f + np.float32(C4[1])
    q = q * f + np.float32(C4[0])
    q = q * f + np.float32(1.0)
    e = t.view(np.int32) - np.int32(0x4B400000)
    return (q.view(np.int32) + (e << 23)).view(np.float32)


def test_softmax_exp2_polynomial_error_bound():
    xs = np.linspace(-60.0, 0.0, 600001).astype(np.float32)
    got = exp2_poly_f32(xs).astype(np.float64)
    ref = np.exp2(xs.astype(np.float64))
    assert (np.abs(got - ref) / ref).max() < 4e-6
    assert exp2_poly_f32(np.float32(-np.inf)) < 1e-35  # masked scores vanish after the fp16 cast
