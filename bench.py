"""Benchmark of the Axon B200 backend on the BASELINE configs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl axon|reference]

One JSON line on rank 0. The headline workload is the SwiGLU MLP config
(m 4096, hidden 4096, intermediate 14336, bf16): on one
GPU the two tcgen05 GEMMs, on N GPUs the column/row tensor-parallel step whose
output all-reduce is fused with the down projection over NVLink peer memory
(enzyme_b200.tp.FusedTPSwiGLU), so the 1 -> N values trace the one path with
a collective. After the timed region the headline's output is checked on
sampled rows against the float64 oracle (rtol = atol = 1e-2) and across ranks
(every rank holds the same bits); the result is the line's "parity" record and
a miss exits non-zero. The other BASELINE configs (rope, rmsnorm, nucleus
cumsum, 1e9-parameter Adam), the remaining specs at their reference eval cases
plus a roofline-scale shape (layernorm, softmax, matmul, rmsnorm_matmul) and
the GEMM-backed neighbour specs (qkv_cte, softmax_mm, attention_nkilib) are
measured in the same run and reported, compactly, under "workloads" unless
--no-extra is given.

A step is one pass of the hot path over one batch of synthetic input. Timing:
W untimed steps, then exactly K steps (replayed from a CUDA graph on one GPU),
bracketed by a barrier and torch.cuda.synchronize() on both sides, CUDA
events on the launching stream, max over ranks; that K-step region is
repeated (at least 3 times, more until the headline's timed windows add up to
tens of milliseconds) and the median repeat is reported. Memory-bound
workloads rotate over enough input/output sets that the working set exceeds
2 x L2 (126 MB), so every launch reads HBM. `e2e` times the same step
through the public API with pinned host inputs copied in and the result
copied back inside the timed loop.

--impl reference times the reference's CPU path for the same workload (the
specs' torch references, restated in oracle/cpu_torch.py) on all host cores.
Multi-GPU (torchrun): memory-bound and GEMM workloads run as replicas (weak
scaling); Adam shards the 1e9 parameters across ranks with no collective; the
SwiGLU MLP runs tensor-parallel (strong scaling).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from enzyme_b200 import _native as N  # noqa: E402
from enzyme_b200 import ops, roofline, timing  # noqa: E402

THETA = 500000.0
HEADLINE = "silu_mlp"


def _sig(x, digits=4):
    if x is None or not math.isfinite(x) or x == 0:
        return x
    return round(x, digits - 1 - int(math.floor(math.log10(abs(x)))))


# ---------------------------------------------------------------------------------
# workloads
#
# Each workload is built with dev=None for the reference arm: then only its
# sizes and CPU sample exist, no device memory is touched.


class Workload:
    name = ""
    spec = ""
    kind = "hbm"
    dtype = "bf16"
    launches_per_step = 1
    use_graph = True
    scaling = "weak"
    itemsize = 2
    nsets = 1

    def __init__(self, dev, rank, world):
        self.dev, self.rank, self.world = dev, rank, world
        if dev is not None:
            self.gen = torch.Generator(device=dev).manual_seed(42 + rank)

    @property
    def unit(self):
        return "GB/s" if self.kind == "hbm" else "TFLOP/s"

    def metric(self):
        return ("HBM GB/s" if self.kind == "hbm" else "bf16 TFLOP/s") + f" ({self.name})"

    def per_step_work(self) -> float:  # bytes or flops per rank per step
        return roofline.work(self.spec, self.dims, self.itemsize)[1]

    def job_work(self) -> float:  # whole-job work per step (all ranks)
        return self.per_step_work() * self.world

    # End to end through the public call for workloads whose step reads
    # `e2e_inputs()` and writes `e2e_output()` (single set): the inputs come
    # from pinned host memory and the output goes back to it inside the
    # timed loop. Workloads with rotating sets define their own.
    def e2e_inputs(self):
        raise NotImplementedError

    def e2e_output(self):
        raise NotImplementedError

    def e2e_setup(self):
        ins = self.e2e_inputs()
        self.h = [t.cpu().pin_memory() for t in ins]
        out = self.e2e_output()
        self.ho = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        self.h2d = sum(t.numel() * t.element_size() for t in self.h)
        self.d2h = self.ho.numel() * self.ho.element_size()

    def e2e_step(self, i):
        for d, h in zip(self.e2e_inputs(), self.h):
            d.copy_(h, non_blocking=True)
        self.launch(0)
        self.ho.copy_(self.e2e_output(), non_blocking=True)

    def _randn(self, *shape, dtype=torch.bfloat16, scale=1.0):
        t = torch.randn(*shape, device=self.dev, generator=self.gen)
        if scale != 1.0:
            t.mul_(scale)
        return t.to(dtype)


class SwiGLU(Workload):
    """The SwiGLU MLP config; tensor-parallel over the intermediate axis at N > 1."""

    name, spec = "silu_mlp", "silu_mlp_swiglu"
    kind = "tensor"
    M, H, INTER = 4096, 4096, 14336
    # parity rows: every 97th token (43 rows), checked against float64
    PARITY_STRIDE = 97
    # the fused path's knobs (enzyme_b200.tp.FusedTPSwiGLU); measured per step
    # on 2 and 8 B200s in section 6 of the design notes
    SLABS = 1
    TP_TUNE = None
    REDUCE_CTAS = 32
    # "slabs" (default): the GEMMs with the reduce-scatter in the down
    # projection's epilogue, then the owner reduce + all-gather push;
    # "whole": the step in one kernel, reduction warps beside the tiles;
    # "nvls": the same with the all-reduce by the NVLink switch; "auto":
    # nvls where every rank's GPU supports multicast, else slabs. Measured at
    # 8 ranks: slabs 275 us, whole 274, nvls 335 per step.
    TP_MODE = os.environ.get("AXON_BENCH_TP_MODE", "slabs")

    def __init__(self, dev, rank, world):
        super().__init__(dev, rank, world)
        m, h, inter = self.M, self.H, self.INTER
        if inter % world:
            raise SystemExit(f"intermediate {inter} not divisible by {world} ranks")
        self.shard = inter // world
        self.dims = dict(m=m, n=inter, k=h, p=h)
        self.scaling = "strong" if world > 1 else "weak"
        if dev is None:
            return
        g = torch.Generator(device=dev).manual_seed(42)  # the same tokens on every rank
        # x rotates over two buffers so a step's inputs and outputs exceed L2
        self.xs = [torch.randn(m, h, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
        self.nsets = 2
        self.w1 = self._randn(h, self.shard, scale=0.02)
        self.w2 = self._randn(h, self.shard, scale=0.02)
        self.w3 = self._randn(self.shard, h, scale=0.02)
        # The activation is stored as f16 (precision 5: the f16 copy of W_down
        # is made once here, as a serving stack converts weights at load time).
        # One bf16 term misses the config's 1e-2 tolerance on ~1e4 outputs;
        # f16 meets it.
        if world > 1:
            # column/row tensor parallel: W_gate/W_up column shard, W_down row
            # shard; the down GEMM scatters f16 partial rows to their owner
            # ranks over NVLink, owners reduce and push bf16 rows to every rank
            from enzyme_b200.tp import FusedTPSwiGLU, multicast_supported

            mode = self.TP_MODE
            if mode == "auto":
                ok = torch.tensor([1 if multicast_supported(dev) else 0], device=dev)
                dist.all_reduce(ok, op=dist.ReduceOp.MIN)  # every rank takes the same path
                mode = "nvls" if ok.item() else "slabs"
            self.tp_mode = mode
            self.tp = FusedTPSwiGLU(self.w1, self.w2, self.w3, m=m, slabs=self.SLABS, tune=self.TP_TUNE,
                                    reduce_ctas=self.REDUCE_CTAS, whole_step=mode in ("nvls", "whole"),
                                    multicast_gather=mode == "nvls")
            self.y = self.tp.y
            self.use_graph = False  # each step carries a new epoch for the peer flags
            self.launches_per_step = self.tp.launches_per_step()
        else:
            self.w3h = ops.cast(self.w3, torch.float16)
            self.tune = {"precision": 5}
            ws = ops.silu_mlp_workspace_bytes(m, self.shard, h, N.AXON_BF16, self.tune)
            self.act = torch.empty(ws, dtype=torch.uint8, device=dev)
            self.y = torch.empty(m, h, dtype=torch.bfloat16, device=dev)
            self.launches_per_step = 2  # gate/up GEMM with the SiLU-gate epilogue, down GEMM
        torch.cuda.synchronize(dev)

    def per_step_work(self):
        m, n, k, p = self.M, self.shard, self.H, self.H
        return 2.0 * m * k * n * 2 + 2.0 * m * n * p

    def job_work(self):
        return roofline.work(self.spec, self.dims)[1]

    def launch(self, i):
        x = self.xs[i % 2]
        if self.world > 1:
            self.tp.forward(x)
        else:
            ops.silu_mlp(x, self.w1, self.w2, self.w3h, out=self.y, workspace=self.act, tune=self.tune)

    def check(self):
        if self.world > 1:
            self.tp.status()

    def close(self):
        if self.world > 1:
            torch.cuda.synchronize()
            dist.barrier()  # no rank unmaps a peer buffer while another still writes it
            self.tp.close()
            dist.barrier()

    def parity(self) -> dict:
        """Sampled rows of one fresh step against the float64 oracle of the
        unsharded MLP, plus a bitwise cross-rank comparison. Every rank takes
        the same collective steps; rank 0 evaluates. Outside any timed region."""
        self.launch(0)
        torch.cuda.synchronize()
        self.check()
        y = self.y.clone()
        # every rank's copy of the output has the same bits (a checksum of the raw words)
        words = y.view(torch.int16).to(torch.int64)
        sums = torch.stack([words.sum(), (words * torch.arange(1, words.shape[1] + 1, device=y.device)).sum()])
        same = True
        if self.world > 1:
            allsums = [torch.empty_like(sums) for _ in range(self.world)]
            dist.all_gather(allsums, sums)
            same = all(bool(torch.equal(a, allsums[0])) for a in allsums)
            shards = []
            for w in (self.w1, self.w2, self.w3):
                parts = [torch.empty_like(w) for _ in range(self.world)]
                dist.all_gather(parts, w.contiguous())
                shards.append(parts)
            w1 = torch.cat(shards[0], dim=1)
            w2 = torch.cat(shards[1], dim=1)
            w3 = torch.cat(shards[2], dim=0)
        else:
            w1, w2, w3 = self.w1, self.w2, self.w3
        rec = {"rows": 0, "worst_err_over_tol": None, "ranks_identical": same,
               "tol": "rtol=atol=1e-2 vs oracle.f64.silu_mlp"}
        if self.rank == 0:
            import numpy as np

            from oracle import f64

            rows = torch.arange(0, self.M, self.PARITY_STRIDE, device=y.device)
            x = self.xs[0][rows].float().cpu().numpy()
            want = f64.silu_mlp(x, w1.float().cpu().numpy(), w2.float().cpu().numpy(), w3.float().cpu().numpy())
            got = y[rows].float().cpu().numpy().astype(np.float64)
            ratio = np.abs(got - want) / (1e-2 + 1e-2 * np.abs(want))
            rec.update(rows=int(rows.numel()), worst_err_over_tol=float(ratio.max()),
                       finite=bool(torch.isfinite(y.float()).all()))
        del w1, w2, w3
        return rec

    def e2e_setup(self):
        self.h = self.xs[0].cpu().pin_memory()
        self.ho = torch.empty(self.y.shape, dtype=self.y.dtype).pin_memory()
        self.h2d = self.h.numel() * 2
        self.d2h = self.ho.numel() * self.ho.element_size()

    def e2e_step(self, i):
        self.xs[0].copy_(self.h, non_blocking=True)
        self.launch(0)
        self.ho.copy_(self.y, non_blocking=True)

    def cpu_step(self):
        from oracle import cpu_torch

        rows = 64
        if not hasattr(self, "_cpu"):
            g = torch.Generator().manual_seed(1)
            self._cpu = (torch.randn(rows, 4096, generator=g), 0.02 * torch.randn(4096, 14336, generator=g),
                         0.02 * torch.randn(4096, 14336, generator=g), 0.02 * torch.randn(14336, 4096, generator=g))
        cpu_torch.silu_mlp(*self._cpu)
        return roofline.work(self.spec, dict(m=rows, n=14336, k=4096, p=4096))[1], \
            f"{rows} of 4096 tokens (fp32 torch, same weights shape)"

    def config(self):
        how = {"nvls": "one kernel per step: GEMM tiles beside reduction warps, all-reduce by the NVLink switch "
                       "(multimem.ld_reduce + multimem.st)",
               "whole": "one kernel per step: GEMM tiles beside reduction warps, reduce-scatter into owners' "
                        "inboxes, all-gather by peer stores",
               "slabs": "reduce-scatter in the down GEMM over NVLink, owner reduce + all-gather push"}
        par = "tp1" if self.world == 1 else f"tp{self.world} ({how[self.tp_mode]})"
        ws = (self.M * self.H * 2 * 2 + 3 * self.H * self.shard * 2 + self.M * self.shard * 2) / 2**20
        return {"workload": "silu_mlp_swiglu: m 4096, h 4096, inter 14336, bf16, W ~ N(0, 0.02), f16 act",
                "parallelism": par, "l2": f"x over 2 buffers; {ws:.0f} MiB touched per GPU per step > L2"}


class Rope(Workload):
    name, spec = "rope", "rope_gqa"

    def __init__(self, dev, rank, world):
        super().__init__(dev, rank, world)
        self.dims = dict(s=4096, hq=32, hkv=8, half_d=64)
        s, h = 4096, 64
        inv = THETA ** (-torch.arange(h, dtype=torch.float64) * 2 / 128)
        ang = torch.arange(s, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos_h, self.sin_h = torch.cos(ang).float(), torch.sin(ang).float()
        if dev is None:
            return
        set_bytes = int(self.per_step_work())
        self.nsets = timing.sets_to_defeat_l2(set_bytes)
        self.sets = []
        for _ in range(self.nsets):
            q = self._randn(s, 32, 128)
            k = self._randn(s, 8, 128)
            self.sets.append((q, k, self.cos_h.to(dev), self.sin_h.to(dev), torch.empty_like(q), torch.empty_like(k)))
        self.working_set = set_bytes * self.nsets

    def launch(self, i):
        q, k, c, s, qo, ko = self.sets[i % self.nsets]
        ops.rope_rotate_half(q, k, c, s, q_out=qo, k_out=ko)

    def e2e_setup(self):
        q, k, c, s, qo, ko = self.sets[0]
        self.h = [t.cpu().pin_memory() for t in (q, k, c, s)]
        self.ho = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (qo, ko)]
        self.h2d = sum(t.numel() * t.element_size() for t in self.h)
        self.d2h = sum(t.numel() * t.element_size() for t in self.ho)

    def e2e_step(self, i):
        q, k, c, s, qo, ko = self.sets[i % self.nsets]
        for d, h in zip((q, k, c, s), self.h):
            d.copy_(h, non_blocking=True)
        ops.rope_rotate_half(q, k, c, s, q_out=qo, k_out=ko)
        self.ho[0].copy_(qo, non_blocking=True)
        self.ho[1].copy_(ko, non_blocking=True)

    def cpu_step(self):
        from oracle import cpu_torch

        tok = 256
        if not hasattr(self, "_cpu"):
            g = torch.Generator().manual_seed(1)
            self._cpu = (torch.randn(tok, 32, 2, 64, generator=g), torch.randn(tok, 8, 2, 64, generator=g),
                         self.cos_h[:tok].clone(), self.sin_h[:tok].clone())
        q, k, c, s = self._cpu
        cpu_torch.rope_rotate_half(q, c, s)
        cpu_torch.rope_rotate_half(k, c, s)
        return self.per_step_work() * tok / 4096, f"{tok} of 4096 tokens (q 32 heads + k 8 heads, fp32 torch_ref)"

    def config(self):
        return {"workload": "rope_gqa: q [4096,32,128] + k [4096,8,128] bf16, fp32 cos/sin [4096,64], theta 5e5",
                "rotating_sets": self.nsets, "l2": f"inputs rotate over {self.working_set / 2**20:.0f} MiB > 2x L2"}


class RowCase(Workload):
    """A row-wise spec (rmsnorm_llama, layernorm, softmax) at one shape, with
    its inputs rotated past 2 x L2."""

    op = ""

    def __init__(self, dev, rank, world, m, n, dtype=torch.bfloat16, case=""):
        self.name = f"{self.op}_{case}" if case else self.op
        super().__init__(dev, rank, world)
        self.m, self.n, self.tdtype = m, n, dtype
        self.itemsize = torch.empty(0, dtype=dtype).element_size()
        self.dtype = "f32" if dtype == torch.float32 else "bf16"
        self.dims = dict(m=m, n=n)
        self.case = case
        if dev is None:
            return
        self.nsets = timing.sets_to_defeat_l2(int(self.per_step_work()))
        self.sets = []
        for _ in range(self.nsets):
            x = self._randn(m, n, dtype=dtype)
            w = (1 + 0.1 * torch.randn(n, device=dev, generator=self.gen)).to(dtype) if self.op == "rmsnorm" else None
            self.sets.append((x, w, torch.empty_like(x)))

    def _run(self, x, w, y):
        if self.op == "rmsnorm":
            ops.rmsnorm(x, w, scale=1.0 / self.n, eps=1e-6, out=y)
        elif self.op == "layernorm":
            ops.layernorm(x, eps=1e-6, out=y)
        else:
            ops.softmax(x, out=y)

    def launch(self, i):
        self._run(*self.sets[i % self.nsets])

    def e2e_setup(self):
        x, w, y = self.sets[0]
        self.h = [x.cpu().pin_memory()] + ([w.cpu().pin_memory()] if w is not None else [])
        self.ho = torch.empty(y.shape, dtype=y.dtype).pin_memory()
        self.h2d = sum(t.numel() * t.element_size() for t in self.h)
        self.d2h = self.ho.numel() * self.ho.element_size()

    def e2e_step(self, i):
        x, w, y = self.sets[i % self.nsets]
        x.copy_(self.h[0], non_blocking=True)
        if w is not None:
            w.copy_(self.h[1], non_blocking=True)
        self._run(x, w, y)
        self.ho.copy_(y, non_blocking=True)

    def cpu_step(self):
        from oracle import cpu_torch

        rows = min(self.m, 256)
        if not hasattr(self, "_cpu"):
            g = torch.Generator().manual_seed(1)
            self._cpu = (torch.randn(rows, self.n, generator=g), 1 + 0.1 * torch.randn(self.n, generator=g))
        x, w = self._cpu
        if self.op == "rmsnorm":
            cpu_torch.rmsnorm_mean(x, w)
        elif self.op == "layernorm":
            cpu_torch.layernorm(x)
        else:
            cpu_torch.softmax(x)
        return self.per_step_work() * rows / self.m, f"{rows} of {self.m} rows (fp32 torch reference)"

    def config(self):
        return {"workload": f"{self.spec}: x [{self.m},{self.n}] {self.dtype}" + (f" ({self.case})" if self.case else ""),
                "rotating_sets": self.nsets}


class RmsNorm(RowCase):
    op, spec = "rmsnorm", "rmsnorm_llama"

    def __init__(self, dev, rank, world):
        super().__init__(dev, rank, world, 2048, 4096)

    def config(self):
        return {"workload": "rmsnorm_llama: x [2048,4096] bf16, w [4096], eps 1e-6, mean form",
                "rotating_sets": self.nsets}


class LayerNorm(RowCase):
    op, spec = "layernorm", "layernorm"


class Softmax(RowCase):
    op, spec = "softmax", "softmax"


class Cumsum(Workload):
    name, spec = "cumsum", "cumsum_nucleus_sorted"
    dtype = "f32"
    itemsize = 4
    # the library default: at 256 aligned rows it runs the row-streaming scan
    TUNE = None

    def __init__(self, dev, rank, world):
        super().__init__(dev, rank, world)
        self.dims = dict(m=256, n=128256)
        if dev is None:
            logits = 2.0 * torch.randn(32, 128256, generator=torch.Generator().manual_seed(1))
            self._cpu = torch.sort(torch.softmax(logits, dim=1), dim=1, descending=True).values.contiguous()
            return
        self.nsets = timing.sets_to_defeat_l2(int(self.per_step_work()))
        self.sets = []
        for _ in range(self.nsets):
            logits = 2.0 * torch.randn(256, 128256, device=dev, generator=self.gen)
            x = torch.sort(torch.softmax(logits, dim=1), dim=1, descending=True).values.contiguous()
            nbytes = ops.cumsum_workspace_bytes(256, 128256, self.TUNE)
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev) if nbytes else None
            self.sets.append((x, torch.empty_like(x), ws))

    def launch(self, i):
        x, y, ws = self.sets[i % self.nsets]
        ops.cumsum(x, out=y, workspace=ws, tune=self.TUNE)

    def check(self):
        for _, _, ws in self.sets:
            if ws is not None:
                ops.cumsum_status(ws)
        N.check(N.lib().axon_cumsum_status(None, torch.cuda.current_stream().cuda_stream))

    def e2e_setup(self):
        x, y, _ = self.sets[0]
        self.h = x.cpu().pin_memory()
        self.ho = torch.empty(y.shape, dtype=y.dtype).pin_memory()
        self.h2d = self.h.numel() * 4
        self.d2h = self.ho.numel() * 4

    def e2e_step(self, i):
        x, y, ws = self.sets[i % self.nsets]
        x.copy_(self.h, non_blocking=True)
        ops.cumsum(x, out=y, workspace=ws, tune=self.TUNE)
        self.ho.copy_(y, non_blocking=True)

    def cpu_step(self):
        from oracle import cpu_torch

        rows = 32
        if not hasattr(self, "_cpu"):
            self._cpu = self.sets[0][0][:rows].cpu()
        cpu_torch.cumsum(self._cpu)
        return self.per_step_work() * rows / 256, f"{rows} of 256 rows (fp32 torch.cumsum)"

    def config(self):
        return {"workload": "cumsum_nucleus_sorted: 256 x 128256 fp32 sorted softmax rows", "rotating_sets": self.nsets}


class Adam(Workload):
    name, spec = "fused_adam", "fused_adam_cfg"
    dtype = "f32"
    TOTAL = 1_000_000_000

    def __init__(self, dev, rank, world):
        super().__init__(dev, rank, world)
        n = self.TOTAL // world
        self.n = n
        self.scaling = "strong"
        self.dims = dict(p=1, f=n)
        self.ss = 3e-4 / (1 - 0.9 ** 10)
        self.ib = 1 / math.sqrt(1 - 0.95 ** 10)
        if dev is None:
            return
        self.p = torch.randn(n, device=dev, generator=self.gen).mul_(0.02)
        self.g = torch.randn(n, device=dev, generator=self.gen).mul_(1e-3).to(torch.bfloat16)
        self.m = torch.zeros(n, device=dev)
        self.v = torch.zeros(n, device=dev)

    def per_step_work(self):
        return 26.0 * self.n

    def launch(self, i):
        ops.adam(self.p, self.g, self.m, self.v, step_size=self.ss, inv_bc2_sqrt=self.ib, wd=0.1, beta1=0.9,
                 beta2=0.95, eps=1e-8, out=(self.p, self.m, self.v))

    def e2e_setup(self):
        # end to end at this size is a PCIe stream of 26 GB per step; time a
        # 1e8-parameter slice through the same call and scale per byte.
        self.e2e_n = min(self.n, 100_000_000)
        sl = slice(0, self.e2e_n)
        self.h = [t[sl].cpu().pin_memory() for t in (self.p, self.g, self.m, self.v)]
        self.ho = [torch.empty(self.e2e_n).pin_memory() for _ in range(3)]
        self.h2d = sum(t.numel() * t.element_size() for t in self.h)
        self.d2h = 12 * self.e2e_n
        self.e2e_scale = self.e2e_n / self.n

    def e2e_step(self, i):
        sl = slice(0, self.e2e_n)
        dst = (self.p[sl], self.g[sl], self.m[sl], self.v[sl])
        for d, h in zip(dst, self.h):
            d.copy_(h, non_blocking=True)
        ops.adam(*dst, step_size=self.ss, inv_bc2_sqrt=self.ib, wd=0.1, beta1=0.9, beta2=0.95,
                 out=(dst[0], dst[2], dst[3]))
        for h, d in zip(self.ho, (dst[0], dst[2], dst[3])):
            h.copy_(d, non_blocking=True)

    def cpu_step(self):
        from oracle import cpu_torch

        n = 10_000_000
        if not hasattr(self, "_cpu"):
            g = torch.Generator().manual_seed(1)
            self._cpu = (0.02 * torch.randn(n, generator=g), 1e-3 * torch.randn(n, generator=g),
                         torch.zeros(n), torch.zeros(n))
        cpu_torch.adam(*self._cpu, self.ss, self.ib, 0.1, beta1=0.9, beta2=0.95)
        return 26.0 * n, "1e7 of 1e9 parameters (fp32 torch_ref)"

    def config(self):
        return {"workload": f"fused_adam_cfg: 1e9 fp32 params (+bf16 grads), {self.n} per rank, in place",
                "l2": "working set 26 GB >> L2"}


class GemmCase(Workload):
    """matmul or rmsnorm_matmul (sum-based norm, row-scale epilogue) at one shape."""

    kind = "tensor"
    op = ""

    def __init__(self, dev, rank, world, m, n, k, case=""):
        self.name = f"{self.op}_{case}" if case else self.op
        self.spec = self.op
        super().__init__(dev, rank, world)
        self.m, self.n, self.k, self.case = m, n, k, case
        self.dims = dict(m=m, n=n, k=k)
        self.launches_per_step = 2 if self.op == "rmsnorm_matmul" else 1
        if dev is None:
            return
        set_bytes = (m * k + k * n + m * n) * 2
        self.nsets = timing.sets_to_defeat_l2(set_bytes)
        self.sets = []
        for _ in range(self.nsets):
            x = self._randn(m, k, scale=1.0 / math.sqrt(k) if self.op == "matmul" else 1.0)
            w = self._randn(k, n)
            ws = torch.empty(max(16, 4 * m), dtype=torch.uint8, device=dev) if self.op == "rmsnorm_matmul" else None
            self.sets.append((x, w, torch.empty(m, n, dtype=torch.bfloat16, device=dev), ws))
        self.working_set = set_bytes * self.nsets

    def _run(self, x, w, y, ws):
        if self.op == "matmul":
            ops.gemm(x, w, out=y)
        else:
            ops.rmsnorm_matmul(x, w, out=y, workspace=ws)

    def launch(self, i):
        self._run(*self.sets[i % self.nsets])

    def e2e_setup(self):
        x, w, y, _ = self.sets[0]
        self.h = [x.cpu().pin_memory(), w.cpu().pin_memory()]
        self.ho = torch.empty(y.shape, dtype=y.dtype).pin_memory()
        self.h2d = sum(t.numel() * 2 for t in self.h)
        self.d2h = self.ho.numel() * 2

    def e2e_step(self, i):
        x, w, y, ws = self.sets[i % self.nsets]
        x.copy_(self.h[0], non_blocking=True)
        w.copy_(self.h[1], non_blocking=True)
        self._run(x, w, y, ws)
        self.ho.copy_(y, non_blocking=True)

    def cpu_step(self):
        from oracle import cpu_torch

        rows = min(self.m, 256)
        if not hasattr(self, "_cpu"):
            g = torch.Generator().manual_seed(1)
            self._cpu = (torch.randn(rows, self.k, generator=g), torch.randn(self.k, self.n, generator=g))
        getattr(cpu_torch, self.op)(*self._cpu)
        return self.per_step_work() * rows / self.m, f"{rows} of {self.m} rows (fp32 torch reference)"

    def config(self):
        return {"workload": f"{self.op}: m {self.m}, n {self.n}, k {self.k} bf16" + (f" ({self.case})" if self.case else ""),
                "rotating_sets": self.nsets, "l2": f"operands rotate over {self.working_set / 2**20:.0f} MiB"}


class Matmul(GemmCase):
    op = "matmul"


class RmsNormMatmul(GemmCase):
    op = "rmsnorm_matmul"


class QkvCte(Workload):
    """qkv_cte at its eval/sizes.json llama70b case: residual add, norm and
    fused QKV projection in one kernel; HBM-bound (the three inputs)."""

    name, spec = "qkv_cte", "qkv_cte"
    M, N, K = 16384, 512, 8192

    def __init__(self, dev, rank, world):
        super().__init__(dev, rank, world)
        m, n, k = self.M, self.N, self.K
        self.dims = dict(m=m, n=n, k=k)
        if dev is None:
            return
        self.ins = [self._randn(m, k) for _ in range(3)]  # 805 MB per step: past L2 with one set
        self.w = self._randn(k, n, scale=1.0 / k ** 0.5)
        self.y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        nbytes = int(N.lib().axon_qkv_cte_workspace_bytes(m, n, k, None))
        self.ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)

    def launch(self, i):
        ops.qkv_cte(*self.ins, self.w, out=self.y, workspace=self.ws)

    def e2e_inputs(self):
        return [*self.ins, self.w]

    def e2e_output(self):
        return self.y

    def cpu_step(self):
        from oracle import cpu_torch

        rows = 256
        if not hasattr(self, "_cpu"):
            g = torch.Generator().manual_seed(1)
            self._cpu = [torch.randn(rows, self.K, generator=g) for _ in range(3)] + \
                [torch.randn(self.K, self.N, generator=g) / self.K ** 0.5]
        cpu_torch.qkv_cte(*self._cpu)
        return self.per_step_work() * rows / self.M, f"{rows} of {self.M} rows (fp32 torch_ref)"

    def config(self):
        return {"workload": "qkv_cte llama70b (eval/sizes.json): m 16384, n 512, k 8192 bf16, one kernel",
                "l2": "inputs 805 MB >> L2"}


class SoftmaxMM(Workload):
    """softmax_mm at 4096^3: exp row pass, then the row-scaled GEMM."""

    name, spec = "softmax_mm", "softmax_mm"
    kind = "tensor"
    launches_per_step = 2
    M = N_ = K = 4096

    def __init__(self, dev, rank, world):
        super().__init__(dev, rank, world)
        m, n, k = self.M, self.N_, self.K
        self.dims = dict(m=m, n=n, k=k)
        if dev is None:
            return
        self.nsets = 2  # 2 x 128 MB (x, w, exp(x), y) rotate past L2
        self.sets = []
        for _ in range(self.nsets):
            x = self._randn(m, k)
            w = self._randn(k, n)
            ws = torch.empty(int(N.lib().axon_softmax_mm_workspace_bytes(m, k)), dtype=torch.uint8, device=dev)
            self.sets.append((x, w, torch.empty(m, n, dtype=torch.bfloat16, device=dev), ws))

    def launch(self, i):
        x, w, y, ws = self.sets[i % self.nsets]
        ops.softmax_mm(x, w, out=y, workspace=ws)

    def e2e_inputs(self):
        return list(self.sets[0][:2])

    def e2e_output(self):
        return self.sets[0][2]

    def cpu_step(self):
        from oracle import cpu_torch

        rows = 256
        if not hasattr(self, "_cpu"):
            g = torch.Generator().manual_seed(1)
            self._cpu = (torch.randn(rows, self.K, generator=g), torch.randn(self.K, self.N_, generator=g))
        cpu_torch.softmax_mm(*self._cpu)
        return self.per_step_work() * rows / self.M, f"{rows} of {self.M} rows (fp32 baseline_op in torch)"

    def config(self):
        return {"workload": "softmax_mm: m = n = k = 4096 bf16 (exp row pass + row-scaled tcgen05 GEMM)",
                "rotating_sets": self.nsets, "l2": "inputs rotate over 256 MB > 2 x L2"}


class Attention(Workload):
    """attention_nkilib at its s8k_d128 case (eval/sizes.json)."""

    name, spec = "attention", "attention_nkilib"
    kind = "tensor"
    launches_per_step = 2  # the fused kernel and its split-key reduce
    S, D = 8192, 128

    def __init__(self, dev, rank, world):
        super().__init__(dev, rank, world)
        s, d = self.S, self.D
        self.dims = dict(s=s, d=d)
        if dev is None:
            return
        self.q = torch.rand(s, d, device=dev, generator=self.gen).to(torch.bfloat16)
        self.kt = torch.rand(d, s, device=dev, generator=self.gen).to(torch.bfloat16)
        self.v = torch.rand(s, d, device=dev, generator=self.gen).to(torch.bfloat16)
        self.y = torch.empty(s, d, dtype=torch.bfloat16, device=dev)
        nbytes = int(N.lib().axon_attention_workspace_bytes(s, d, None))
        self.ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)

    def launch(self, i):
        ops.attention(self.q, self.kt, self.v, out=self.y, workspace=self.ws)

    def e2e_inputs(self):
        return [self.q, self.kt, self.v]

    def e2e_output(self):
        return self.y

    def cpu_step(self):
        from oracle import cpu_torch

        rows = 256
        if not hasattr(self, "_cpu"):
            g = torch.Generator().manual_seed(1)
            self._cpu = (torch.rand(rows, self.D, generator=g), torch.rand(self.D, self.S, generator=g),
                         torch.rand(self.S, self.D, generator=g))
        cpu_torch.attention(*self._cpu)
        return self.per_step_work() * rows / self.S, f"{rows} of {self.S} query rows (fp32 torch_ref)"

    def config(self):
        return {"workload": "attention_nkilib s8k_d128 (eval/sizes.json): s 8192, d 128 bf16, uniform [0, 1), "
                            "one kernel (scores stay on chip)",
                "l2": "q, k_t, v (6 MB) stay L2-resident across steps: the kernel is tensor-bound, not HBM-bound"}


def _case(cls, **kw):
    def make(dev, rank, world):
        return cls(dev, rank, world, **kw)

    make.cls = cls
    return make


# name -> constructor(dev, rank, world); dev=None builds the CPU-only form
WORKLOADS = {
    "silu_mlp": SwiGLU,
    "rope": Rope,
    "rmsnorm": RmsNorm,
    "cumsum": Cumsum,
    "fused_adam": Adam,
    # reference eval cases (eval/sizes.json) and one roofline-scale shape each
    "layernorm_llama70b": _case(LayerNorm, m=128, n=8192, case="llama70b"),
    "layernorm_2048x8192": _case(LayerNorm, m=2048, n=8192, case="2048x8192"),
    "softmax_sq1k": _case(Softmax, m=1024, n=1024, dtype=torch.float32, case="sq1k"),
    "softmax_4096x32768": _case(Softmax, m=4096, n=32768, dtype=torch.float32, case="4096x32768"),
    "matmul_sq1k": _case(Matmul, m=1024, n=1024, k=1024, case="sq1k"),
    "matmul_4096": _case(Matmul, m=4096, n=4096, k=4096, case="4096"),
    "rmsnorm_matmul_sq1k": _case(RmsNormMatmul, m=1024, n=1024, k=1024, case="sq1k"),
    "rmsnorm_matmul_h8192": _case(RmsNormMatmul, m=1024, n=8192, k=8192, case="h8192"),
    "qkv_cte": QkvCte,
    "softmax_mm": SoftmaxMM,
    "attention": Attention,
}
# long steps: fewer timed steps among the extras
LONG = {"fused_adam", "silu_mlp", "qkv_cte", "softmax_mm", "attention", "matmul_4096", "rmsnorm_matmul_h8192",
        "softmax_4096x32768"}


# ---------------------------------------------------------------------------------
# measurement


def barrier():
    if dist.is_initialized():
        dist.barrier()


def max_over_ranks(v: float, dev) -> float:
    if not dist.is_initialized():
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure(w: Workload, steps: int, warmup: int, sampler_gpu: int | None, window_ms: float):
    """Median over repeats of the K-step timed region (each: barrier + sync,
    events around exactly K steps, sync + barrier; max over ranks). Repeats:
    at least 3, more until the timed windows add up to `window_ms`. Returns
    (ms for K steps, repeats, clocks summary or None)."""
    if w.use_graph:
        if steps >= w.nsets:
            chunk = min(steps, 64 * w.nsets) // w.nsets * w.nsets
            reps, rem = divmod(steps, chunk)
            graph = timing.capture_graph(w.launch, chunk)
            tail = timing.capture_graph(lambda i: w.launch(reps * chunk + i), rem) if rem else None
            plans = [(graph, reps, tail)]
        else:
            # fewer steps than input sets: one K-step graph per starting set,
            # cycled over the repeats, so every set is used in turn and none
            # is still in L2 when it comes round again
            plans = [(timing.capture_graph(lambda i, o=o: w.launch(o + i), steps), 1, None)
                     for o in range(0, w.nsets, steps)]
        wchunk = max(1, min(warmup, steps, w.nsets))
        wgraph = timing.capture_graph(w.launch, wchunk)
        turn = [0]

        def run_timed():
            graph, reps, tail = plans[turn[0] % len(plans)]
            turn[0] += 1
            for _ in range(reps):
                graph.replay()
            if tail is not None:
                tail.replay()

        def run_warm():
            for _ in range(math.ceil(warmup / wchunk)):
                wgraph.replay()

        soak = run_timed
    else:
        def run_timed():
            for i in range(steps):
                w.launch(i)

        def run_warm():
            for i in range(warmup):
                w.launch(i)

        def soak():
            w.launch(0)

    sampler = timing.ClockSampler(sampler_gpu) if sampler_gpu is not None else None
    # keep the GPU busy so clocks settle (and the sampler sees the load); the
    # stop decision is taken on rank 0 and shared, so every rank soaks alike
    t_end = time.time() + 0.6
    if sampler:
        sampler.__enter__()
    while True:
        soak()
        torch.cuda.synchronize()
        more = torch.tensor([1.0 if time.time() < t_end else 0.0], device=w.dev)
        if dist.is_initialized():
            dist.broadcast(more, 0)
        if more.item() == 0.0:
            break
    run_warm()
    torch.cuda.synchronize()

    def one():
        barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        run_timed()
        end.record()
        end.synchronize()
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(start.elapsed_time(end), w.dev)

    times = [one()]
    want = max(3, min(25, math.ceil(window_ms / max(times[0], 1e-3))))
    while len(times) < want:
        times.append(one())
    clocks = None
    if sampler:
        sampler.__exit__(None, None, None)
        clocks = sampler.summary()
        clocks["window"] = "soak + warmup + timed repeats"
    return statistics.median(times), len(times), clocks


def measure_e2e(w: Workload, steps: int):
    w.e2e_setup()
    iters = max(3, min(steps, 20))
    w.e2e_step(0)
    torch.cuda.synchronize()
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(iters):
        w.e2e_step(i)
    end.record()
    end.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), w.dev) / iters
    scale = getattr(w, "e2e_scale", 1.0)
    work = w.job_work() * scale
    val = work / (ms / 1e3) / (1e9 if w.kind == "hbm" else 1e12)
    return {"value": val, "unit": w.unit, "h2d_bytes_per_step": int(w.h2d), "d2h_bytes_per_step": int(w.d2h),
            "ms_per_step": ms, "steps": iters,
            **({"note": f"measured on a {scale:.0%} slice of the step, same call"} if scale != 1.0 else {})}


def cpu_baseline(w: Workload, seconds: float):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w.cpu_step()  # warm
    done, t0 = 0.0, time.perf_counter()
    sample = ""
    while time.perf_counter() - t0 < seconds:
        work, sample = w.cpu_step()
        done += work
    dt = time.perf_counter() - t0
    val = done / dt / (1e9 if w.kind == "hbm" else 1e12)
    return {"value": val, "unit": w.unit, "cores": threads, "kind": "port", "sample": sample,
            "seconds": round(dt, 2)}


def load_traffic() -> dict:
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.is_file():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return {}
    return {}


def run_workload(name, dev, rank, world, steps, warmup, sampler_gpu, *, window_ms, with_e2e=True,
                 with_parity=False):
    w = WORKLOADS[name](dev, rank, world)
    ms, repeats, clocks = measure(w, steps, warmup, sampler_gpu, window_ms)
    if hasattr(w, "check"):
        w.check()
    ops.gemm_status()
    per_step_ms = ms / steps
    value = w.job_work() / (per_step_ms / 1e3) / (1e9 if w.kind == "hbm" else 1e12)
    # per rank: the step's algorithmic work over the step's device time; the
    # timed loop follows a soak of the same steps, so a tensor-bound step
    # runs at the power-capped (sustained) clock
    roof = roofline.fraction(w.kind, w.per_step_work(), per_step_ms / 1e3, sustained=w.kind == "tensor")
    tr = load_traffic().get(w.spec)
    roof["traffic"] = tr.get("bytes_per_launch") if tr else None
    roof["traffic_source"] = tr.get("source") if tr else None
    roof["traffic_kind"] = tr.get("kind") if tr else None
    res = {"metric": w.metric(), "value": value, "unit": w.unit, "ms_per_step": per_step_ms, "dtype": w.dtype,
           "scaling": w.scaling, "roofline": roof, "config": w.config(), "clocks": clocks,
           "gpu_launches": steps * w.launches_per_step * repeats, "repeats": repeats,
           "timed_window_ms": ms * repeats}
    if with_parity and hasattr(w, "parity"):
        res["parity"] = w.parity()
    if with_e2e:
        res["e2e"] = measure_e2e(w, steps)
    if hasattr(w, "close"):
        w.close()
    return w, res


def compact(r: dict) -> dict:
    """One extra workload in a few keys, so every workload fits the kept tail."""
    c = {r["unit"]: _sig(r["value"]), "ms_per_step": _sig(r["ms_per_step"]), "frac": round(r["roofline"]["frac"], 3)}
    if r["clocks"] and r["clocks"].get("sm_mhz"):
        c["mhz"] = int(r["clocks"]["sm_mhz"])
        bad = [x for x in r["clocks"].get("reasons", []) if x != "sw_power_cap"]
        if bad:
            c["throttle"] = bad
    return c


def reference_arm(args, rank) -> int:
    """The reference's CPU path for the same workload; under torchrun only
    rank 0 runs it."""
    if rank != 0:
        return 0
    w = WORKLOADS[args.workload](None, 0, 1)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    for _ in range(args.warmup):
        w.cpu_step()
    t0 = time.perf_counter()
    work = 0.0
    sample = ""
    for _ in range(args.steps):
        a, sample = w.cpu_step()
        work += a
    dt = time.perf_counter() - t0
    val = work / dt / (1e9 if w.kind == "hbm" else 1e12)
    line = {"impl": "reference", "metric": w.metric(), "value": val, "unit": w.unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "config": {"workload": w.name + " (bounded CPU sample per step)"},
            "cpu_baseline": {"value": val, "unit": w.unit, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": val, "unit": w.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=HEADLINE)
    ap.add_argument("--impl", choices=("axon", "reference"), default="axon")
    ap.add_argument("--no-extra", action="store_true", help="skip the other workloads")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(args, rank)

    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    sampler_gpu = local if rank == 0 else None

    head, res = run_workload(args.workload, dev, rank, world, args.steps, args.warmup, sampler_gpu, window_ms=40.0,
                             with_parity=True)
    line = {
        "metric": res["metric"], "value": res["value"], "unit": res["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
        "higher_is_better": True, "scaling": res["scaling"], "vs_baseline": None, "dtype": res["dtype"],
        "data": "synthetic (seeded randn on device; no dataset)",
        "config": {**res["config"], "parallelism": res["config"].get("parallelism", f"replicas x{world}"),
                   "timing": f"median of {res['repeats']} x {args.steps} steps ({res['timed_window_ms']:.1f} ms)"},
        "roofline": res["roofline"], "clocks": res["clocks"], "e2e": res["e2e"],
        "gpu_launches": res["gpu_launches"],
    }
    parity = res.get("parity")
    if parity is not None:
        line["parity"] = parity
    if rank == 0 and world == 1:
        line["cpu_baseline"] = cpu_baseline(head, args.cpu_seconds)
    del head
    torch.cuda.empty_cache()
    if not args.no_extra:
        extra = {}
        for name in WORKLOADS:
            if name == args.workload:
                continue
            k = max(3, min(args.steps, 20 if name in LONG else args.steps))
            w, r = run_workload(name, dev, rank, world, k, args.warmup, sampler_gpu, window_ms=10.0,
                                with_e2e=False)
            extra[name] = compact(r)
            del w
            torch.cuda.empty_cache()
        line["workloads"] = extra
    failed = False
    if parity is not None and rank == 0:
        worst = parity.get("worst_err_over_tol")
        failed = not parity["ranks_identical"] or worst is None or worst > 1.0 or not parity.get("finite", True)
    if rank == 0:
        print(json.dumps(line))
    if dist.is_initialized():
        flag = torch.tensor([1 if failed else 0], device=dev)
        dist.broadcast(flag, 0)
        failed = bool(flag.item())
        dist.barrier()
        dist.destroy_process_group()
    if failed:
        print(f"bench: parity check of {args.workload} failed: {parity}", file=sys.stderr)
        return 3
    return 0


if __name__ == "__main__":
    sys.exit(main())
