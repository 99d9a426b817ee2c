"""The GPU kernels' GELU restated in NumPy float32 (TEST INFRASTRUCTURE).

The kernels evaluate the reference's exact erf-GELU (``F.gelu(approximate="none")``,
TTB:161) with erf from Abramowitz & Stegun, Handbook of Mathematical Functions,
eq. 7.1.28 (a published rational approximation, |error of erf| <= 3e-7), in fp32
with the operation order of ``gelu_as`` in the library's ``ptx.cuh``.  This
restatement bounds how far that GELU is from the exact one; it is used by the
CPU test of the bound and by the accuracy block of ``bench.py``.
"""

from __future__ import annotations

import math

import numpy as np

# A&S 7.1.28: erf(u) = 1 - 1 / (1 + a1 u + ... + a6 u^6)^16, u >= 0
A = [0.0705230784, 0.0422820123, 0.0092705272, 0.0001520143, 0.0002765672, 0.0000430638]


def gelu_as_f32(v):
    """GELU with the A&S erf, float32, Horner order as in the kernels."""
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


def gelu_as_max_error(lo: float = -12.0, hi: float = 12.0, n: int = 240001) -> dict:
    """max |gelu_as_f32(v) - exact erf-GELU(v)| over an even grid (exact: math.erf in float64)."""
    xs = np.linspace(lo, hi, n)
    exact = np.array([0.5 * x * (1.0 + math.erf(x / math.sqrt(2.0))) for x in xs])
    err = np.abs(gelu_as_f32(xs).astype(np.float64) - exact)
    i = int(err.argmax())
    return {"max_abs": float(err[i]), "at": float(xs[i]), "grid": f"[{lo}, {hi}], {n} points",
            "method": "erf by Abramowitz & Stegun 7.1.28 in fp32 (ptx.cuh gelu_as) vs exact erf GELU in fp64"}
