"""The GPU kernels' GELU (erf by Abramowitz & Stegun eq. 7.1.28, evaluated in fp32)
restated in NumPy float32 with the same operation order (oracle/kernel_gelu.py),
against the exact erf-GELU (math.erf in float64) of the reference (F.gelu(approximate="none"))."""

import numpy as np

from oracle import gelu_as_f32, gelu_as_max_error


def test_gelu_approximation_error_bound():
    err = gelu_as_max_error()
    assert err["max_abs"] < 2e-6, err
    # far tails: exactly x for large positive, exactly 0 for large negative
    assert gelu_as_f32(np.float32(40.0)) == np.float32(40.0)
    assert gelu_as_f32(np.float32(-40.0)) == np.float32(0.0)
