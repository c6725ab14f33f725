"""References and seeded inputs for `cumsum` (Axon kernels/cumsum/refs.py:16-26)."""

import numpy as np
import torch


def baseline_op(a):
    return np.cumsum(a, axis=-1)


def torch_ref(x):
    return torch.cumsum(x, dim=-1)


def make_inputs(*, m, n, dtype=np.float32, rng):
    return (rng.standard_normal((m, n)).astype(dtype),)
