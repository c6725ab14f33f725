"""Spec math for `silu_mlp_swiglu`."""

from enzyme_b200.ir import AxonArray


def kernel_swiglu(x: AxonArray, w1: AxonArray, w2: AxonArray, w3: AxonArray):
    return ((x @ w1).silu() * (x @ w2)) @ w3
