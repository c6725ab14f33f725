"""Multi-GPU paths: column/row tensor-parallel SwiGLU and parameter-sharded Adam.

Both follow the reference's sharding laws (src/axon/sharding.py):

* SwiGLU. The intermediate axis is one axis class shared by W_gate/W_up
  (columns) and W_down (rows). Sharding that class puts the first two GEMMs
  in S (each rank owns a column slice: no communication) and makes the down
  projection a contraction over a sharded class, hence Partial("+")
  (sharding.py:380-384), which a terminal AllReduce resolves (:514-522). Here
  the all-reduce is NCCL over NVLink/NVSwitch via torch.distributed, on fp32
  partials so the sum adds no bf16 rounding.
* Adam. Every tensor is split along the same (flattened parameter) axis: the
  update is elementwise, so the plan is S everywhere with no combine step
  beyond a barrier (the reference's row-shard "P" plan).

The per-rank compute is this library's CUDA kernels. `TPSwiGLU` splits the
tokens into m-slabs and issues each slab's all-reduce asynchronously as soon
as its partial is written, so the collective of slab i overlaps the GEMMs of
slab i+1. The kernel calls are injected (`ops`), so the host logic -- shard
ranges, slab schedule, collectives -- is testable on CPU ranks over gloo.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

# Sharding labels in the reference's vocabulary: R = replicated, S(axis) =
# sharded along that axis of the tensor, P(+) = partial sum pending a combine.
SWIGLU_PLAN = {
    "x": "R",
    "w_gate": "S(1)",
    "w_up": "S(1)",
    "w_down": "S(0)",
    "activation": "S(1)",
    "y_partial": "P(+)",
    "y": "R (after AllReduce(+))",
}
ADAM_PLAN = {name: "S(0)" for name in ("param", "grad", "exp_avg", "exp_avg_sq")}


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous near-even split: the first total % world ranks get one more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_swiglu(w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, rank: int, world: int):
    """This rank's (w_gate[:, s], w_up[:, s], w_down[s, :]) for its slice s of
    the intermediate axis, contiguous."""
    inter = w_gate.shape[1]
    if w_up.shape != w_gate.shape or w_down.shape[0] != inter:
        raise ValueError("w_gate/w_up must be [hidden, inter] and w_down [inter, hidden]")
    a, b = shard_range(inter, rank, world)
    return (w_gate[:, a:b].contiguous(), w_up[:, a:b].contiguous(), w_down[a:b, :].contiguous())


@dataclass
class _CudaOps:
    """The CUDA kernels a TP step runs (enzyme_b200.ops). `tune` goes to both
    GEMMs: capping `max_ctas` below the SM count (and/or using fewer stages)
    leaves room on some SMs for NCCL's kernels, so a slab's all-reduce really
    runs while the next slab's GEMMs do."""

    tune: dict | None = None

    def cast(self, src, dtype, out):
        from . import ops

        return ops.cast(src, dtype, out=out)

    def gate_up(self, x, w_gate, w_up, out):
        from . import _native as N
        from . import ops

        return ops.gemm(x, w_gate, b2=w_up, epilogue=N.AXON_EPI_SILU_GATE, out=out, tune=self.tune)

    def down(self, act, w_down, out):
        from . import ops

        return ops.gemm(act, w_down, out=out, tune=self.tune)


class TPSwiGLU:
    """One rank's shard of y = (silu(x @ W_gate) * (x @ W_up)) @ W_down.

    forward(x) returns the full fp32 output on every rank. Per step: one f16
    copy of the W_down shard, then per m-slab the SiLU-gate GEMM (f16
    activation) and the down GEMM into an fp32 partial, whose all-reduce is
    issued asynchronously before the next slab starts.
    """

    def __init__(self, w_gate, w_up, w_down, *, group=None, slabs: int = 4, ops=None,
                 act_dtype=torch.float16):
        self.w_gate, self.w_up, self.w_down = w_gate, w_up, w_down
        self.group = group
        self.slabs = max(1, int(slabs))
        self.ops = ops or _CudaOps()
        self.act_dtype = act_dtype
        self._w_down_h = None
        self._act = None

    def _buffers(self, m: int):
        dev = self.w_gate.device
        if self._w_down_h is None or self._w_down_h.device != dev:
            self._w_down_h = torch.empty(self.w_down.shape, dtype=self.act_dtype, device=dev)
        if self._act is None or self._act.shape[0] < m:
            self._act = torch.empty((m, self.w_gate.shape[1]), dtype=self.act_dtype, device=dev)
        return self._w_down_h, self._act[:m]

    def slab_bounds(self, m: int) -> list[tuple[int, int]]:
        # slabs of whole 128-row tiles, so no tile is split between two GEMMs
        tiles = -(-m // 128)
        per = -(-tiles // self.slabs)
        out = []
        for s in range(0, tiles, per):
            a, b = s * 128, min(m, (s + per) * 128)
            if a < b:
                out.append((a, b))
        return out

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        m = x.shape[0]
        w_down_h, act = self._buffers(m)
        y = out if out is not None else torch.empty((m, self.w_down.shape[1]), dtype=torch.float32, device=x.device)
        self.ops.cast(self.w_down, self.act_dtype, w_down_h)
        works = []
        for a, b in self.slab_bounds(m):
            self.ops.gate_up(x[a:b], self.w_gate, self.w_up, act[a:b])
            self.ops.down(act[a:b], w_down_h, y[a:b])
            if dist.is_initialized() and dist.get_world_size(self.group) > 1:
                works.append(dist.all_reduce(y[a:b], op=dist.ReduceOp.SUM, group=self.group, async_op=True))
        for w in works:
            w.wait()
        return y


def adam_shard(total: int, rank: int, world: int) -> slice:
    """The contiguous slice of a flat parameter vector this rank updates."""
    a, b = shard_range(total, rank, world)
    return slice(a, b)
