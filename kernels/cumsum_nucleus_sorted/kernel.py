"""Spec math for `cumsum_nucleus_sorted`."""

from enzyme_b200.ir import AxonArray


def kernel_cumsum_sorted(x: AxonArray) -> AxonArray:
    return x.cumsum(axis=-1)
