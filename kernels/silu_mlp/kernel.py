"""Spec math for `silu_mlp` (Axon kernels/silu_mlp/kernel.py:7-14)."""

from enzyme_b200.ir import AxonArray


def kernel_silu_mlp_full(x: AxonArray, w1: AxonArray, w2: AxonArray, w3: AxonArray):
    return ((x @ w1).silu() * (x @ w2)) @ w3
