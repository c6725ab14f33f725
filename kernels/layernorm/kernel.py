"""Spec math for `layernorm` (Axon kernels/layernorm/kernel.py:17-25):
`(x - mean) / sqrt(mean((x - mean)^2) + EPS)` with EPS = 1e-6."""

from enzyme_b200.ir import AxonArray

EPS = 1e-6


def kernel_layernorm(x: AxonArray) -> AxonArray:
    inv_n = 1.0 / x.shape[1]
    centred = x - x.sum(axis=1, keep_dims=True) * inv_n
    var = (centred * centred).sum(axis=1, keep_dims=True) * inv_n
    return centred / (var + EPS).sqrt()
