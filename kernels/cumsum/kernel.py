"""Spec math for `cumsum` (Axon kernels/cumsum/kernel.py:12-13)."""

from enzyme_b200.ir import AxonArray


def kernel_cumsum(x: AxonArray) -> AxonArray:
    return x.cumsum(axis=-1)
