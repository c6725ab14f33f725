"""Spec math for `rope_gqa`, written with numpy views (AxonArray has no
indexing; the arrays it wraps do)."""

import numpy as np

from enzyme_b200.ir import AxonArray


def _rotate(x: np.ndarray, c: np.ndarray, s: np.ndarray) -> np.ndarray:
    x1, x2 = x[:, :, 0, :], x[:, :, 1, :]
    c, s = c[:, None, :], s[:, None, :]
    return np.stack([x1 * c - x2 * s, x2 * c + x1 * s], axis=2)


def kernel_rope_gqa(q: AxonArray, k: AxonArray, cos: AxonArray, sin: AxonArray):
    return (
        AxonArray(_rotate(q.data, cos.data, sin.data)),
        AxonArray(_rotate(k.data, cos.data, sin.data)),
    )
