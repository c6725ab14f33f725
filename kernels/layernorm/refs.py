"""References and seeded inputs for `layernorm` (Axon kernels/layernorm/refs.py:16-37).

EPS must equal kernel.py's.
"""

import numpy as np
import torch
from ml_dtypes import bfloat16

EPS = 1e-6


def baseline_op(x):
    centred = x - np.mean(x, axis=1, keepdims=True)
    var = np.mean(np.square(centred), axis=1, keepdims=True)
    return centred / np.sqrt(var + EPS)


def torch_ref(x):
    centred = x - torch.mean(x, dim=1, keepdim=True)
    var = torch.mean(centred * centred, dim=1, keepdim=True)
    return centred / torch.sqrt(var + EPS)


def make_inputs(*, m, n, dtype=bfloat16, rng):
    return (rng.standard_normal((m, n)).astype(dtype),)
