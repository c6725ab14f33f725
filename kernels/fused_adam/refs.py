"""References and seeded inputs for `fused_adam` (Axon kernels/fused_adam/refs.py:21-67).

Draw order (param, grad, exp_avg, |exp_avg_sq|, then constant per-row
scalars step_size=1e-3, inv_bc2_sqrt=1.0, wd=0.01) follows the reference.
"""

import numpy as np
import torch
from ml_dtypes import bfloat16

BETA1 = 0.9
BETA2 = 0.999
EPS = 1e-8


def baseline_op(param, grad, exp_avg, exp_avg_sq, step_size, inv_bc2_sqrt, wd):
    g = grad + wd * param
    m = BETA1 * exp_avg + (1.0 - BETA1) * g
    v = BETA2 * exp_avg_sq + (1.0 - BETA2) * (g * g)
    p = param - m / (np.sqrt(v) * inv_bc2_sqrt + EPS) * step_size
    return p, m, v


def torch_ref(param, grad, exp_avg, exp_avg_sq, step_size, inv_bc2_sqrt, wd):
    g = grad + wd * param
    m = BETA1 * exp_avg + (1.0 - BETA1) * g
    v = BETA2 * exp_avg_sq + (1.0 - BETA2) * (g * g)
    p = param - m / (torch.sqrt(v) * inv_bc2_sqrt + EPS) * step_size
    return (p, m, v)


def make_inputs(*, p, f, dtype=bfloat16, rng):
    full, col = (p, f), (p, 1)
    return (
        rng.standard_normal(full).astype(dtype),
        rng.standard_normal(full).astype(dtype),
        rng.standard_normal(full).astype(dtype),
        np.abs(rng.standard_normal(full)).astype(dtype),
        np.full(col, 1e-3, dtype=dtype),
        np.full(col, 1.0, dtype=dtype),
        np.full(col, 0.01, dtype=dtype),
    )
