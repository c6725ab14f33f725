"""References and seeded inputs for `softmax` (Axon kernels/softmax/refs.py:11-17)."""

import numpy as np


def baseline_op(a):
    e = np.exp(a)
    return e / np.sum(e, axis=1, keepdims=True)


def make_inputs(*, m, n, dtype=np.float32, rng):
    return (rng.standard_normal((m, n)).astype(dtype),)
