"""References and seeded inputs for `attention_nkilib` (Axon
kernels/attention_nkilib/refs.py:36-65).

Inputs are uniform [0, 1); q carries the softmax scale the reference folds
into it (1.0 for d < 512, 0.5 from d = 512), which keeps max(q @ k_t) under
the fp32 exponential's limit for the bare, unshifted softmax.
"""

import numpy as np
import torch
from ml_dtypes import bfloat16


def baseline_op(q, k_t, v):
    e = np.exp(np.matmul(q, k_t))
    return np.matmul(e / np.sum(e, axis=1, keepdims=True), v)


def torch_ref(q, k_t, v):
    e = torch.exp(torch.matmul(q, k_t))
    return torch.matmul(e / torch.sum(e, dim=1, keepdim=True), v)


def softmax_scale(d):
    return 0.5 if d >= 512 else 1.0


def make_inputs(*, s, d, dtype=bfloat16, rng):
    return (
        (rng.random((s, d)) * softmax_scale(d)).astype(dtype),
        rng.random((d, s)).astype(dtype),
        rng.random((s, d)).astype(dtype),
    )
