"""References and seeded inputs for `silu_mlp` (Axon kernels/silu_mlp/refs.py:16-30)."""

import numpy as np
from ml_dtypes import bfloat16


def baseline_op(x, w1, w2, w3):
    gate = np.matmul(x, w1)
    up = np.matmul(x, w2)
    return np.matmul(gate / (1 + np.exp(-gate)) * up, w3)


def make_inputs(*, m, n, k, p, dtype=bfloat16, rng):
    return (
        rng.standard_normal((m, k)).astype(dtype),
        rng.standard_normal((k, n)).astype(dtype),
        rng.standard_normal((k, n)).astype(dtype),
        rng.standard_normal((n, p)).astype(dtype),
    )
