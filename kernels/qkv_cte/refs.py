"""References and seeded inputs for `qkv_cte` (Axon kernels/qkv_cte/refs.py:23-48).

The weight draw is scaled by 1/sqrt(k), and the inputs are drawn in the
order x, mlp_prev, attention_prev, w, as the reference does.
"""

import numpy as np
import torch
from ml_dtypes import bfloat16

EPS = 1e-6


def baseline_op(x, mlp_prev, attention_prev, w):
    h = x + mlp_prev + attention_prev
    return np.matmul(h / np.sqrt(np.mean(h * h, axis=1, keepdims=True) + EPS), w)


def torch_ref(x, mlp_prev, attention_prev, w):
    h = x + mlp_prev + attention_prev
    return torch.matmul(h / torch.sqrt(torch.mean(h * h, dim=1, keepdim=True) + EPS), w)


def make_inputs(*, m, n, k, dtype=bfloat16, rng):
    x = rng.standard_normal((m, k)).astype(dtype)
    mlp_prev = rng.standard_normal((m, k)).astype(dtype)
    attention_prev = rng.standard_normal((m, k)).astype(dtype)
    w = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(dtype)
    return x, mlp_prev, attention_prev, w
