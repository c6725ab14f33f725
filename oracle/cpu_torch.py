"""fp32 torch forms of the specs' reference CPU path -- TEST/BASELINE ONLY.

These are what the reference runs on host cores when it has no device: each
spec's `torch_ref` (inputs coerced to fp32 torch, as Axon's case harness does
in src/axon/case_gen.py:190-201), or its numpy `baseline_op` restated in
torch where the spec has no `torch_ref`. `bench.py` times them as the CPU
baseline; nothing in `enzyme_b200` imports this module.
"""

from __future__ import annotations

import torch


def rmsnorm_mean(x, w, eps=1e-6):
    return x * torch.rsqrt(torch.mean(x * x, dim=1, keepdim=True) + eps) * w


def rmsnorm_sum(x):
    return x / torch.sqrt(torch.sum(x * x, dim=1, keepdim=True))


def layernorm(x, eps=1e-6):
    c = x - torch.mean(x, dim=1, keepdim=True)
    return c / torch.sqrt(torch.mean(c * c, dim=1, keepdim=True) + eps)


def softmax(x):
    e = torch.exp(x)
    return e / torch.sum(e, dim=1, keepdim=True)


def rope_rotate_half(x, cos, sin):
    x1, x2 = x[:, :, 0, :], x[:, :, 1, :]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.stack([x1 * c - x2 * s, x2 * c + x1 * s], dim=2)


def cumsum(x):
    return torch.cumsum(x, dim=-1)


def adam(p, g, m, v, step_size, inv_bc2_sqrt, wd, beta1=0.9, beta2=0.999, eps=1e-8):
    g = g + wd * p
    m = beta1 * m + (1.0 - beta1) * g
    v = beta2 * v + (1.0 - beta2) * (g * g)
    p = p - m / (torch.sqrt(v) * inv_bc2_sqrt + eps) * step_size
    return p, m, v


def silu_mlp(x, w1, w2, w3):
    return (torch.nn.functional.silu(x @ w1) * (x @ w2)) @ w3


def qkv_cte(x, mlp_prev, attention_prev, w, eps=1e-6):
    h = x + mlp_prev + attention_prev
    return (h / torch.sqrt(torch.mean(h * h, dim=1, keepdim=True) + eps)) @ w


def softmax_mm(x, w):
    e = torch.exp(x)
    return (e / torch.sum(e, dim=1, keepdim=True)) @ w


def attention(q, k_t, v):
    e = torch.exp(q @ k_t)
    return (e / torch.sum(e, dim=1, keepdim=True)) @ v


def matmul(x, w):
    return x @ w


def rmsnorm_matmul(x, w):
    return rmsnorm_sum(x) @ w
