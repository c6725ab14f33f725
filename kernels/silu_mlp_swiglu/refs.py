"""References and seeded inputs for `silu_mlp_swiglu` (draw order x, w1, w2, w3)."""

import numpy as np
import torch
from ml_dtypes import bfloat16

WEIGHT_STD = 0.02


def baseline_op(x, w1, w2, w3):
    gate = np.matmul(x, w1)
    up = np.matmul(x, w2)
    return np.matmul(gate / (1 + np.exp(-gate)) * up, w3)


def torch_ref(x, w1, w2, w3):
    return (torch.nn.functional.silu(x @ w1) * (x @ w2)) @ w3


def make_inputs(*, m, n, k, p, dtype=bfloat16, rng):
    return (
        rng.standard_normal((m, k)).astype(dtype),
        (WEIGHT_STD * rng.standard_normal((k, n))).astype(dtype),
        (WEIGHT_STD * rng.standard_normal((k, n))).astype(dtype),
        (WEIGHT_STD * rng.standard_normal((n, p))).astype(dtype),
    )
