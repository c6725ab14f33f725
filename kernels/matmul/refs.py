"""References and seeded inputs for `matmul` (Axon kernels/matmul/refs.py:20-38).

x is scaled by 1/sqrt(k) so the product stays O(1) (w stays N(0, 1)).
"""

import numpy as np
from ml_dtypes import bfloat16


def baseline_op(x, w):
    return np.matmul(x, w)


def torch_ref(x, w):
    return x @ w


def make_inputs(*, m, n, k, dtype=bfloat16, rng):
    scale = 1.0 / np.sqrt(k)
    return (
        (rng.standard_normal((m, k)) * scale).astype(dtype),
        rng.standard_normal((k, n)).astype(dtype),
    )
