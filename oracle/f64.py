"""Float64 restatements of each hot-path spec (the parity oracle).

Test infrastructure only (see `oracle/__init__.py`). Every function takes
numpy arrays of any float dtype, widens to float64 and returns float64.
"""

from __future__ import annotations

import numpy as np


def _f(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float64)


def rmsnorm_sum(x):
    """Axon kernels/rmsnorm/refs.py:21-23: x / sqrt(sum(x^2)) per row."""
    x = _f(x)
    return x / np.sqrt(np.sum(x * x, axis=1, keepdims=True))


def rmsnorm_mean(x, w=None, eps=1e-6):
    """BASELINE rmsnorm config: x * rsqrt(mean(x^2) + eps) * w."""
    x = _f(x)
    y = x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + eps)
    return y * _f(w) if w is not None else y


def layernorm(x, eps=1e-6):
    """Axon kernels/layernorm/refs.py:19-23 (EPS 1e-6 at :16)."""
    x = _f(x)
    c = x - x.mean(axis=1, keepdims=True)
    return c / np.sqrt(np.mean(c * c, axis=1, keepdims=True) + eps)


def softmax(x):
    """Axon kernels/softmax/refs.py:11-13 (evaluated max-shifted, same value)."""
    x = _f(x)
    e = np.exp(x - x.max(axis=1, keepdims=True))
    return e / e.sum(axis=1, keepdims=True)


def rope_split(x_even, x_odd, cos, sin):
    """Axon kernels/rope/refs.py:20-23."""
    xe, xo, c, s = map(_f, (x_even, x_odd, cos, sin))
    return xe * c - xo * s, xo * c + xe * s


def rope_rotate_half(x, cos, sin):
    """Rotate-half rope on x [s, h, 2, half_d] with tables [s, half_d]
    (the BASELINE layout); the pointwise math is Axon kernels/rope/kernel.py:34-35."""
    x = _f(x)
    c, s = _f(cos)[:, None, :], _f(sin)[:, None, :]
    x1, x2 = x[:, :, 0, :], x[:, :, 1, :]
    return np.stack([x1 * c - x2 * s, x2 * c + x1 * s], axis=2)


def cumsum(x):
    """Axon kernels/cumsum/refs.py:16-17: inclusive scan on the last axis."""
    return np.cumsum(_f(x), axis=-1)


def adam(param, grad, exp_avg, exp_avg_sq, step_size, inv_bc2_sqrt, wd,
         beta1=0.9, beta2=0.999, eps=1e-8):
    """Axon kernels/fused_adam/refs.py:28-35 (betas/eps defaults at :21-23)."""
    p, g, m, v = map(_f, (param, grad, exp_avg, exp_avg_sq))
    ss, ib, wd = map(_f, (step_size, inv_bc2_sqrt, wd))
    g = g + wd * p
    m = beta1 * m + (1.0 - beta1) * g
    v = beta2 * v + (1.0 - beta2) * (g * g)
    p = p - m / (np.sqrt(v) * ib + eps) * ss
    return p, m, v


def matmul(x, w):
    """Axon kernels/matmul/refs.py:20-21."""
    return _f(x) @ _f(w)


def silu_mlp(x, w1, w2, w3):
    """Axon kernels/silu_mlp/refs.py:16-21."""
    x = _f(x)
    gate = x @ _f(w1)
    up = x @ _f(w2)
    return (gate / (1.0 + np.exp(-gate)) * up) @ _f(w3)


def rmsnorm_matmul(x, w):
    """Axon kernels/rmsnorm_matmul/refs.py:16-22 (sum-based norm)."""
    return rmsnorm_sum(x) @ _f(w)


def qkv_cte(x, mlp_prev, attention_prev, w, eps=1e-6):
    """Axon kernels/qkv_cte/refs.py:23-27: residual add, mean-RMS norm, projection."""
    h = _f(x) + _f(mlp_prev) + _f(attention_prev)
    return (h / np.sqrt(np.mean(h * h, axis=1, keepdims=True) + eps)) @ _f(w)


def softmax_mm(x, w):
    """Axon kernels/softmax_mm/refs.py:16-19: bare-exponential softmax, then @ w."""
    e = np.exp(_f(x))
    return (e / e.sum(axis=1, keepdims=True)) @ _f(w)


def attention(q, k_t, v):
    """Axon kernels/attention_nkilib/refs.py:36-40: softmax(q @ k_t) @ v with a
    bare exponential (q @ k_t stays below the exponential's float64 limit)."""
    e = np.exp(_f(q) @ _f(k_t))
    return (e / e.sum(axis=1, keepdims=True)) @ _f(v)


# spec name -> oracle over the spec's positional inputs
ORACLES = {
    "rmsnorm": rmsnorm_sum,
    "rmsnorm_llama": lambda x, w: rmsnorm_mean(x, w, 1e-6),
    "layernorm": layernorm,
    "softmax": softmax,
    "rope": rope_split,
    "rope_gqa": lambda q, k, c, s: (rope_rotate_half(q, c, s), rope_rotate_half(k, c, s)),
    "cumsum": cumsum,
    "cumsum_nucleus_sorted": cumsum,
    "fused_adam": adam,
    "fused_adam_cfg": lambda *a: adam(*a, beta1=0.9, beta2=0.95, eps=1e-8),
    "matmul": matmul,
    "silu_mlp": silu_mlp,
    "silu_mlp_swiglu": silu_mlp,
    "rmsnorm_matmul": rmsnorm_matmul,
    "qkv_cte": qkv_cte,
    "softmax_mm": softmax_mm,
    "attention_nkilib": attention,
}


def evaluate(spec_name: str, *inputs) -> tuple[np.ndarray, ...]:
    out = ORACLES[spec_name](*inputs)
    return out if isinstance(out, tuple) else (out,)
