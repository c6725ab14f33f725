"""References and seeded inputs for `cumsum_nucleus_sorted`.

logits ~ N(0, 2) (standard deviation 2), softmax per row in float64, sorted
descending, stored as `dtype` (fp32 by default).
"""

import numpy as np
import torch


def baseline_op(a):
    # the config's bar is rel 1e-5 against float64: a float32 running sum over
    # 128256 columns is itself ~7e-5 off, so the reference evaluates in float64
    return np.cumsum(np.asarray(a, dtype=np.float64), axis=-1)


def torch_ref(x):
    return torch.cumsum(x, dim=-1)


def make_inputs(*, m, n, dtype=np.float32, rng):
    logits = 2.0 * rng.standard_normal((m, n))
    e = np.exp(logits - logits.max(axis=1, keepdims=True))
    probs = e / e.sum(axis=1, keepdims=True)
    return (-np.sort(-probs, axis=1)).astype(dtype),
