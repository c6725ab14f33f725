"""Spec math for `qkv_cte` (Axon kernels/qkv_cte/kernel.py:18-27): the norm
divides by the square root of the mean of h^2 plus EPS."""

from enzyme_b200.ir import AxonArray

EPS = 1e-6


def kernel_qkv_cte(x: AxonArray, mlp_prev: AxonArray, attention_prev: AxonArray, w: AxonArray) -> AxonArray:
    h = x + mlp_prev + attention_prev
    ms = (h * h).sum(axis=1, keep_dims=True) * (1.0 / x.shape[1])
    return (h / (ms + EPS).sqrt()) @ w
