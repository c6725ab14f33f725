"""Spec math for `fused_adam` (Axon kernels/fused_adam/kernel.py:20-45).

beta1 = 0.9, beta2 = 0.999 and eps = 1e-8 are fixed by the spec.
"""

from enzyme_b200.ir import AxonArray

BETA1 = 0.9
BETA2 = 0.999
EPS = 1e-8


def kernel_fused_adam(param, grad, exp_avg, exp_avg_sq, step_size, inv_bc2_sqrt, wd):
    g = grad + wd * param
    m = BETA1 * exp_avg + (1.0 - BETA1) * g
    v = BETA2 * exp_avg_sq + (1.0 - BETA2) * (g * g)
    p = param - m / (v.sqrt() * inv_bc2_sqrt + EPS) * step_size
    return (p, m, v)
