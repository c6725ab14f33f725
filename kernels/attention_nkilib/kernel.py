"""Spec math for `attention_nkilib` (Axon kernels/attention_nkilib/kernel.py:14-21)."""

from enzyme_b200.ir import AxonArray


def kernel_attention_nkilib(q: AxonArray, k_t: AxonArray, v: AxonArray) -> AxonArray:
    e = (q @ k_t).exp()
    return (e / e.sum(axis=1, keep_dims=True)) @ v
