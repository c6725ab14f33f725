"""`AxonArray`: an eager, solver-free stand-in for Axon's tracing array.

Axon's `AxonArray` (src/axon/ir.py:27-160) records a graph for e-graph
synthesis. The CUDA backend has no synthesis stage, so the spec packages'
`kernel.py` math only needs to *run*: this class evaluates the same operator
vocabulary (`+ - * / @`, `sum(axis, keep_dims)`, `sqrt`, `exp`, `transpose`,
`relu`, `silu`, `softmax`, `cumsum`) eagerly in float64 numpy. Running a
spec's `axon_kernel` on wrapped inputs therefore gives a third, independent
evaluation of the spec math next to `baseline_op` and `torch_ref`.
"""

from __future__ import annotations

from typing import Any

import numpy as np


def _unwrap(v: Any) -> Any:
    return v.data if isinstance(v, AxonArray) else v


class AxonArray:
    __slots__ = ("data",)

    def __init__(self, data: Any):
        self.data = np.asarray(data, dtype=np.float64)

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self.data.shape)

    def __add__(self, o: Any) -> AxonArray:
        return AxonArray(self.data + _unwrap(o))

    __radd__ = __add__

    def __sub__(self, o: Any) -> AxonArray:
        return AxonArray(self.data - _unwrap(o))

    def __rsub__(self, o: Any) -> AxonArray:
        return AxonArray(_unwrap(o) - self.data)

    def __mul__(self, o: Any) -> AxonArray:
        return AxonArray(self.data * _unwrap(o))

    __rmul__ = __mul__

    def __truediv__(self, o: Any) -> AxonArray:
        return AxonArray(self.data / _unwrap(o))

    def __rtruediv__(self, o: Any) -> AxonArray:
        return AxonArray(_unwrap(o) / self.data)

    def __neg__(self) -> AxonArray:
        return AxonArray(-self.data)

    def __matmul__(self, o: Any) -> AxonArray:
        if not isinstance(o, AxonArray) or self.data.ndim != 2 or o.data.ndim != 2:
            raise ValueError("matmul expects two rank-2 AxonArrays")
        return AxonArray(self.data @ o.data)

    def sum(self, axis: Any = None, keep_dims: bool = False) -> AxonArray:
        return AxonArray(np.sum(self.data, axis=axis, keepdims=keep_dims))

    def sqrt(self) -> AxonArray:
        return AxonArray(np.sqrt(self.data))

    def exp(self) -> AxonArray:
        return AxonArray(np.exp(self.data))

    def transpose(self) -> AxonArray:
        return AxonArray(self.data.T)

    def relu(self) -> AxonArray:
        return AxonArray(np.maximum(self.data, 0.0))

    def silu(self) -> AxonArray:
        return AxonArray(self.data / (1.0 + np.exp(-self.data)))

    def softmax(self, axis: int = -1) -> AxonArray:
        e = np.exp(self.data - self.data.max(axis=axis, keepdims=True))
        return AxonArray(e / e.sum(axis=axis, keepdims=True))

    def cumsum(self, axis: int = -1) -> AxonArray:
        return AxonArray(np.cumsum(self.data, axis=axis))

    def numpy(self) -> np.ndarray:
        return self.data


def evaluate(kernel, *inputs: Any) -> tuple[np.ndarray, ...]:
    """Run a spec's `axon_kernel` eagerly; always returns a tuple of arrays."""
    out = kernel(*[AxonArray(np.asarray(a, dtype=np.float64)) for a in inputs])
    if isinstance(out, tuple):
        return tuple(o.data for o in out)
    return (out.data,)
