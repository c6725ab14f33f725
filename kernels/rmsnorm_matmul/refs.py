"""References and seeded inputs for `rmsnorm_matmul` (Axon kernels/rmsnorm_matmul/refs.py:16-29)."""

import numpy as np
from ml_dtypes import bfloat16


def baseline_op(x, w):
    return np.matmul(x / np.sqrt(np.sum(np.square(x), axis=1, keepdims=True)), w)


def make_inputs(*, m, n, k, dtype=bfloat16, rng):
    return (
        rng.standard_normal((m, k)).astype(dtype),
        rng.standard_normal((k, n)).astype(dtype),
    )
