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

