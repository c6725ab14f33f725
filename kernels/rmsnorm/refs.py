"""References and seeded inputs for `rmsnorm` (Axon kernels/rmsnorm/refs.py:21-34).

Loadable on its own by path (no relative imports). `torch_ref` receives fp32
torch tensors; the harness casts its result back to the case dtype.
"""

import numpy as np
import torch
from ml_dtypes import bfloat16


def baseline_op(x):
    return x / np.sqrt(np.sum(np.square(x), axis=1, keepdims=True))


def torch_ref(x):
    return x / torch.sqrt(torch.sum(x * x, dim=1, keepdim=True))


def make_inputs(*, m, n, dtype=bfloat16, rng):
    return (rng.standard_normal((m, n)).astype(dtype),)
