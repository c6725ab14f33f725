"""References and seeded inputs for `softmax_mm` (Axon kernels/softmax_mm/refs.py:16-26)."""

import numpy as np
from ml_dtypes import bfloat16


def baseline_op(a, b):
    e = np.exp(a)
    return np.matmul(e / np.sum(e, axis=1, keepdims=True), b)


def make_inputs(*, m, n, k, dtype=bfloat16, rng):
    return (
        rng.standard_normal((m, k)).astype(dtype),
        rng.standard_normal((k, n)).astype(dtype),
    )
