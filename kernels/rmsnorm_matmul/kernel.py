"""Spec math for `rmsnorm_matmul` (Axon kernels/rmsnorm_matmul/kernel.py:7-16):
sum-based norm, as in `rmsnorm`."""

from enzyme_b200.ir import AxonArray


def kernel_rmsnorm_matmul(x: AxonArray, w: AxonArray) -> AxonArray:
    return (x / (x * x).sum(axis=1, keep_dims=True).sqrt()) @ w
