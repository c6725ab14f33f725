"""References and seeded inputs for `fused_adam_cfg` (draw order: param, grad)."""

import numpy as np
import torch
from ml_dtypes import bfloat16

BETA1 = 0.9
BETA2 = 0.95
EPS = 1e-8
LR = 3e-4
WD = 0.1
STEP = 10


def hyper():
    """(step_size, inv_bc2_sqrt, wd) for the config's step."""
    return (
        LR / (1.0 - BETA1**STEP),
        1.0 / np.sqrt(1.0 - BETA2**STEP),
        WD,
    )


def baseline_op(param, grad, exp_avg, exp_avg_sq, step_size, inv_bc2_sqrt, wd):
    # evaluated in float64: the config's bar is rel 1e-5 against float64
    param, grad, exp_avg, exp_avg_sq, step_size, inv_bc2_sqrt, wd = (
        np.asarray(a, dtype=np.float64) for a in (param, grad, exp_avg, exp_avg_sq, step_size, inv_bc2_sqrt, wd))
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


def make_inputs(*, p, f, dtype=np.float32, rng):
    step_size, inv_bc2_sqrt, wd = hyper()
    full, col = (p, f), (p, 1)
    return (
        (0.02 * rng.standard_normal(full)).astype(dtype),
        (1e-3 * rng.standard_normal(full)).astype(bfloat16),
        np.zeros(full, dtype=dtype),
        np.zeros(full, dtype=dtype),
        np.full(col, step_size, dtype=np.float32),
        np.full(col, inv_bc2_sqrt, dtype=np.float32),
        np.full(col, wd, dtype=np.float32),
    )
