"""References and seeded inputs for `rope` (Axon kernels/rope/refs.py:20-46).

cos/sin are genuine rotation values drawn from a uniform angle, so |cos|,
|sin| <= 1, exactly as the reference generator does (same draw order:
x_even, x_odd, then the angles).
"""

import numpy as np
from ml_dtypes import bfloat16


def baseline_op(x_even, x_odd, cos, sin):
    return x_even * cos - x_odd * sin, x_odd * cos + x_even * sin


def torch_ref(x_even, x_odd, cos, sin):
    return (x_even * cos - x_odd * sin, x_odd * cos + x_even * sin)


def make_inputs(*, half_d, free, dtype=bfloat16, rng):
    shape = (half_d, free)
    x_even = rng.standard_normal(shape).astype(dtype)
    x_odd = rng.standard_normal(shape).astype(dtype)
    angle = rng.uniform(-np.pi, np.pi, shape)
    return (x_even, x_odd, np.cos(angle).astype(dtype), np.sin(angle).astype(dtype))
