"""Spec math for `rmsnorm` (kernels/rmsnorm/kernel.py:13-20 of Axon): the row
norm uses the plain sum of squares, not the mean."""

from enzyme_b200.ir import AxonArray


def kernel_rmsnorm(x: AxonArray) -> AxonArray:
    return x / (x * x).sum(axis=1, keep_dims=True).sqrt()
