"""Spec math for `rmsnorm_llama`: mean-of-squares RMS norm with eps and weight."""

from enzyme_b200.ir import AxonArray

EPS = 1e-6


def kernel_rmsnorm_llama(x: AxonArray, w: AxonArray) -> AxonArray:
    ms = (x * x).sum(axis=1, keep_dims=True) * (1.0 / x.shape[1])
    return x / (ms + EPS).sqrt() * w
