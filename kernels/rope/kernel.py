"""Spec math for `rope` (Axon kernels/rope/kernel.py:27-36)."""

from enzyme_b200.ir import AxonArray


def kernel_rope(x_even: AxonArray, x_odd: AxonArray, cos: AxonArray, sin: AxonArray):
    return (x_even * cos - x_odd * sin, x_odd * cos + x_even * sin)
