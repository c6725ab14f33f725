"""Spec math for `matmul` (Axon kernels/matmul/kernel.py:7-8)."""

from enzyme_b200.ir import AxonArray


def kernel_matmul(x: AxonArray, w: AxonArray) -> AxonArray:
    return x @ w
