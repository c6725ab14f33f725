"""References and seeded inputs for `rmsnorm_llama` (draw order: x, then w)."""

import numpy as np
import torch
from ml_dtypes import bfloat16

EPS = 1e-6


def baseline_op(x, w):
    ms = np.mean(np.square(x), axis=1, keepdims=True)
    return x / np.sqrt(ms + EPS) * w


def torch_ref(x, w):
    return x * torch.rsqrt(torch.mean(x * x, dim=1, keepdim=True) + EPS) * w


def make_inputs(*, m, n, dtype=bfloat16, rng):
    x = rng.standard_normal((m, n)).astype(dtype)
    w = (1.0 + 0.1 * rng.standard_normal((n,))).astype(dtype)
    return (x, w)
