"""References and seeded inputs for `rope_gqa`.

Tables: inv_freq[i] = theta ** (-2 i / d) for i < d/2, angle = pos * inv_freq,
evaluated in float64 and stored as fp32. Draw order: q, then k.
"""

import numpy as np
import torch
from ml_dtypes import bfloat16

THETA = 500000.0


def rope_tables(s, half_d, theta=THETA):
    inv_freq = theta ** (-np.arange(half_d, dtype=np.float64) * 2.0 / (2 * half_d))
    angle = np.arange(s, dtype=np.float64)[:, None] * inv_freq[None, :]
    return np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)


def _rotate_np(x, c, s):
    x1, x2 = x[:, :, 0, :], x[:, :, 1, :]
    c, s = c[:, None, :], s[:, None, :]
    return np.stack([x1 * c - x2 * s, x2 * c + x1 * s], axis=2)


def baseline_op(q, k, cos, sin):
    return _rotate_np(q, cos, sin), _rotate_np(k, cos, sin)


def _rotate_t(x, c, s):
    x1, x2 = x[:, :, 0, :], x[:, :, 1, :]
    c, s = c[:, None, :], s[:, None, :]
    return torch.stack([x1 * c - x2 * s, x2 * c + x1 * s], dim=2)


def torch_ref(q, k, cos, sin):
    return (_rotate_t(q, cos, sin), _rotate_t(k, cos, sin))


def make_inputs(*, s, hq, hkv, half_d, dtype=bfloat16, rng):
    q = rng.standard_normal((s, hq, 2, half_d)).astype(dtype)
    k = rng.standard_normal((s, hkv, 2, half_d)).astype(dtype)
    cos, sin = rope_tables(s, half_d)
    return (q, k, cos, sin)
