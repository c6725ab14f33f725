"""Multi-GPU paths: column/row tensor-parallel SwiGLU and parameter-sharded Adam.

Both follow the reference's sharding laws (src/axon/sharding.py):

* SwiGLU. The intermediate axis is one axis class shared by W_gate/W_up
  (columns) and W_down (rows). Sharding that class puts the first two GEMMs
  in S (each rank owns a column slice: no communication) and makes the down
  projection a contraction over a sharded class, hence Partial("+")
  (sharding.py:380-384), which a terminal AllReduce resolves (:514-522).
  `FusedTPSwiGLU` (the path bench.py runs) resolves it without NCCL: the down
  GEMM's epilogue scatters f16 partial rows to their owner ranks over NVLink
  peer memory, owners sum them in fp32 and push the bf16 rows to every rank
  (or store them once through an NVLink multicast address). `TPSwiGLU` keeps
  the plain form -- an NCCL all-reduce of fp32 partials per slab -- for
  comparison.
* Adam. Every tensor is split along the same (flattened parameter) axis: the
  update is elementwise, so the plan is S everywhere with no combine step
  beyond a barrier (the reference's row-shard "P" plan).

The per-rank compute is this library's CUDA kernels. `TPSwiGLU` splits the
tokens into m-slabs and issues each slab's all-reduce asynchronously as soon
as its partial is written, so the collective of slab i overlaps the GEMMs of
slab i+1; its kernel calls are injected (`ops`), so that host logic -- shard
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


# ---- fused path: reduce-scatter in the down GEMM's epilogue, over peer memory ----


def fused_slabs(m: int, world: int, slabs: int) -> list[tuple[int, int]]:
    """Token slabs for the fused path: contiguous, each a multiple of `world`
    rows so every rank owns the same number of rows of every slab."""
    if m % world:
        raise ValueError(f"m={m} must be a multiple of world={world}")
    slabs = max(1, min(int(slabs), m // world))
    unit = m // world
    per = -(-unit // slabs) * world
    return [(a, min(m, a + per)) for a in range(0, m, per)]


@dataclass(frozen=True)
class PeerLayout:
    """Byte offsets inside each rank's shared buffer: the f16 inboxes (slab i
    at its first row: [world][rows_i / world][hidden]), the output [m, hidden]
    and int32 flags (arrive[i][world], done[i][world])."""

    m: int
    hidden: int
    world: int
    nslabs: int
    out_itemsize: int

    @property
    def inbox_bytes(self) -> int:
        return self.m * self.hidden * 2

    @property
    def y_offset(self) -> int:
        return _round_up(self.inbox_bytes, 256)

    @property
    def flags_offset(self) -> int:
        return _round_up(self.y_offset + self.m * self.hidden * self.out_itemsize, 256)

    @property
    def counts_offset(self) -> int:
        """Whole-step kernel: arrival counts [m / 256] then the done count."""
        return _round_up(self.flags_offset + 2 * self.nslabs * self.world * 4, 256)

    @property
    def done_count_offset(self) -> int:
        return self.counts_offset + _round_up(-(-self.m // 256) * 4, 16)

    @property
    def total_bytes(self) -> int:
        return _round_up(self.done_count_offset + 16, 256)

    def inbox_offset(self, slab_start: int) -> int:
        return slab_start * self.hidden * 2

    def arrive_offset(self, i: int) -> int:
        return self.flags_offset + (2 * i) * self.world * 4

    def done_offset(self, i: int) -> int:
        return self.flags_offset + (2 * i + 1) * self.world * 4


def _round_up(x: int, a: int) -> int:
    return -(-x // a) * a


class PeerBuffers:
    """One zeroed device buffer per rank (PeerLayout), mapped into every other
    rank with CUDA IPC; `bases[d]` is rank d's buffer as seen from this rank."""

    def __init__(self, layout: PeerLayout, device, group=None):
        import ctypes

        from . import _native as N

        self.layout = layout
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world != layout.world:
            raise ValueError("layout world size differs from the process group")
        self.buf = torch.zeros(layout.total_bytes, dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)
        handle = ctypes.create_string_buffer(N.AXON_IPC_HANDLE_BYTES)
        off = ctypes.c_int64(0)
        N.check(N.lib().axon_ipc_handle(ctypes.c_void_p(self.buf.data_ptr()), handle, ctypes.byref(off)))
        mine = (bytes(handle.raw), int(off.value))
        everyone = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(everyone, mine, group=group)
        else:
            everyone = [mine]
        self._opened = []
        self.bases = []
        for d, (h, o) in enumerate(everyone):
            if d == self.rank:
                self.bases.append(self.buf.data_ptr())
                continue
            p = ctypes.c_void_p()
            N.check(N.lib().axon_ipc_open(h, o, ctypes.byref(p)))
            self._opened.append((p.value, o))
            self.bases.append(p.value)
        if self.world > 1:
            dist.barrier(group=group)

    def close(self) -> None:
        from . import _native as N

        for p, o in self._opened:
            N.lib().axon_ipc_close(p, o)
        self._opened = []

    def output(self, dtype) -> torch.Tensor:
        lo = self.layout
        nbytes = lo.m * lo.hidden * lo.out_itemsize
        return self.buf[lo.y_offset:lo.y_offset + nbytes].view(dtype).view(lo.m, lo.hidden)


def multicast_supported(device) -> bool:
    """True where symmetric memory on this CUDA device can be bound to an
    NVLink multicast object (GPUs behind an NVSwitch with multicast enabled)."""
    from torch._C._distributed_c10d import _SymmetricMemory

    dev = torch.device(device)
    try:
        return bool(_SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA, dev.index or 0))
    except (RuntimeError, AttributeError):
        return False


def multicast_output(m: int, hidden: int, dtype, device, group=None):
    """An [m, hidden] output in symmetric memory whose ranks' copies are bound
    to one NVLink multicast object: returns (this rank's tensor, the multicast
    address of its first element, the symmetric-memory handle that keeps the
    mapping alive). Raises RuntimeError where the GPUs or the group give no
    multicast address (no NVSwitch multicast support)."""
    from torch.distributed import _symmetric_memory as symm

    y = symm.empty((m, hidden), dtype=dtype, device=device)
    handle = symm.rendezvous(y, group if group is not None else dist.group.WORLD)
    mc = int(handle.multicast_ptr or 0)
    if not mc:
        raise RuntimeError("no NVLink multicast address for this group's symmetric memory")
    # the tensor's offset inside the rank's mapping, applied to the multicast
    # mapping of the same allocation
    off = y.data_ptr() - int(handle.buffer_ptrs[handle.rank])
    if not 0 <= off <= int(handle.buffer_size) - y.numel() * y.element_size():
        raise RuntimeError("symmetric-memory output lies outside its handle's buffer")
    return y, mc + off, handle


class FusedTPSwiGLU:
    """Tensor-parallel SwiGLU whose down-projection all-reduce is fused into
    the GEMMs over NVLink peer memory (csrc/tp.cu):

    per slab: SiLU-gate GEMM -> f16 activation; down GEMM whose epilogue
    stores each f16 partial row into its owner rank's inbox (with one slab,
    both GEMMs run as one kernel, axon_tp_mlp_partial); a release of the
    slab's arrival flags; on a side stream the owner waits for every rank's
    partials, sums them in fp32, rounds once to bf16 and pushes its rows into
    every rank's output, then raises the done flags. forward() ends with a
    bounded wait on every owner's done flag, so the returned [m, hidden]
    tensor (a view of the shared buffer, valid until the next forward) holds
    the full output on every rank. The output is one rounding of the fp32 sum
    of world f16-rounded partials.

    whole_step=True runs the step as one kernel (axon_tp_mlp_step): rows are
    owned in 8-row granules dealt to the ranks in turn, so every owner's rows
    complete while the down projection is still running; two reduction warps
    in every CTA, beside the GEMM roles, reduce and push this rank's rows of
    each 256-row block as soon as every rank's partials of that block have
    arrived, overlapped with the GEMM tiles that follow; one wait for the
    done count ends the step. tune["rows_per_cta"] sets the row blocks per
    group of the kernel's tile order (default 4).

    whole_step=True with multicast_gather=True runs the same kernel with the
    all-reduce done by the NVLink switch (axon_tp_mlp_step_multicast): the
    partials stay in each rank's own buffer, the reduction warps read every
    owned packet once through the partials' multicast address with
    multimem.ld_reduce and store the bf16 sum once, with multimem.st, to the
    output's multicast address. Each byte crosses NVLink once each way
    instead of twice. Needs GPUs behind an NVSwitch with multicast
    (multicast_supported).

    multicast_gather=True puts the output in symmetric memory bound to an
    NVLink multicast object and has each owner store its summed rows once, to
    the multicast address (axon_tp_reduce_multicast): the switch writes them
    into every rank's output, so the all-gather leaves each GPU once instead
    of world - 1 times. The returned tensor is then that symmetric-memory
    output.
    """

    def __init__(self, w_gate, w_up, w_down, m: int, *, group=None, slabs: int = 2, tune=None,
                 reduce_ctas: int = 16, out_dtype=torch.bfloat16, whole_step: bool = False,
                 fused_kernel: bool | None = None, copy_engine_gather: bool = False,
                 multicast_gather: bool = False):
        self.w_gate, self.w_up, self.w_down = w_gate, w_up, w_down
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.m = m
        self.hidden = w_down.shape[1]
        self.slabs = fused_slabs(m, self.world, slabs)
        self.tune = dict(tune or {})
        self.reduce_ctas = int(reduce_ctas)
        self.out_dtype = out_dtype
        dev = w_gate.device
        self.layout = PeerLayout(m, self.hidden, self.world, len(self.slabs), torch.empty(0, dtype=out_dtype).element_size())
        self.peers = PeerBuffers(self.layout, dev, group)
        self.y = self.peers.output(out_dtype)
        # the shard's W_down is fixed for the object's life: one f16 copy, made
        # here (the down projection runs f16 x f16 on the f16 activation)
        from . import _native as N
        from . import ops

        self.w_down_h = ops.cast(w_down, torch.float16)

        # activation [m, n] f16 followed by the fused kernel's counters
        n = w_gate.shape[1]
        self.ws = torch.empty(int(N.lib().axon_tp_mlp_workspace_bytes(m, n)), dtype=torch.uint8, device=dev)
        self.act = self.ws[:m * n * 2].view(torch.float16).view(m, n)
        self.side = torch.cuda.Stream(device=dev)
        self.epoch = 0
        # Both GEMMs in one kernel pays while the shard's gate/up GEMM is a
        # few waves of 256 x 128 tiles (the rule axon_silu_mlp's default
        # applies: fewer than 320 tiles, e.g. 8 ranks at the BASELINE config);
        # larger shards run the two GEMMs as separate launches.
        self.fused_kernel = (-(-m // 256) * -(-n // 128) < 320) if fused_kernel is None else bool(fused_kernel)
        # all-gather by the copy engines (cudaMemcpyAsync to each peer) instead
        # of bulk copies issued by the reducing SMs
        self.copy_engine_gather = bool(copy_engine_gather)
        # all-gather through one multicast store per output packet
        self.multicast_gather = bool(multicast_gather)
        self._y_mc, self._symm = 0, None
        self._part, self._part_mc, self._part_symm = None, 0, None
        if self.multicast_gather:
            if copy_engine_gather:
                raise ValueError("multicast_gather replaces the copy-engine all-gather")
            self.y, self._y_mc, self._symm = multicast_output(m, self.hidden, out_dtype, dev, group)
            if whole_step:
                # each rank's f16 partial of y, bound to its own multicast object
                self._part, self._part_mc, self._part_symm = multicast_output(m, self.hidden, torch.float16, dev,
                                                                              group)
        # one kernel per step (axon_tp_mlp_step): both GEMMs and the reduction
        self.whole_step = bool(whole_step)
        if self.whole_step:
            if out_dtype != torch.bfloat16 or m % 256 or self.world not in (1, 2, 4, 8):
                raise ValueError("whole_step needs bf16 output, m % 256 == 0 and 1, 2, 4 or 8 ranks")
            self.done_per_epoch = int(N.lib().axon_tp_step_done_per_epoch(self.world, m, self.hidden))

    def launches_per_step(self) -> int:
        """Kernels this library launches per forward() (copy-engine transfers
        not counted)."""
        if self.whole_step:
            return 2  # the step kernel, the wait on the done count
        if len(self.slabs) == 1 and self.fused_kernel:
            return 5  # fused GEMMs, signal, reduce + push, signal, wait
        # per slab: gate/up GEMM, scattering down GEMM, signal, reduce, signal;
        # then one wait per slab
        return 6 * len(self.slabs)

    def close(self) -> None:
        torch.cuda.synchronize(self.w_gate.device)
        self.peers.close()
        if self._symm is not None:
            # every rank done with the multicast buffers before any unmaps them
            if self.world > 1:
                dist.barrier(group=self.group)
            self.y, self._symm, self._y_mc = None, None, 0
            self._part, self._part_symm, self._part_mc = None, None, 0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        import ctypes

        from . import _native as N
        from . import ops

        if x.shape[0] != self.m:
            raise ValueError(f"built for {self.m} tokens, got {x.shape[0]}")
        lib, lo, W = N.lib(), self.layout, self.world
        self.epoch += 1
        e = self.epoch
        main = torch.cuda.current_stream(x.device)
        ptrs = lambda vals: (ctypes.c_void_p * W)(*vals)  # noqa: E731
        tune = N.Tune.of(self.tune)
        out_code = {torch.bfloat16: N.AXON_BF16, torch.float16: N.AXON_F16, torch.float32: N.AXON_F32}[self.out_dtype]
        y_ptrs = ptrs([b + lo.y_offset for b in self.peers.bases])
        mine = self.peers.bases[self.rank]
        if self.whole_step and self._part is not None:
            bases = self.peers.bases
            N.check(lib.axon_tp_mlp_step_multicast(
                x.data_ptr(), self.w_gate.data_ptr(), self.w_up.data_ptr(), self.w_down_h.data_ptr(),
                self.ws.data_ptr(), self.ws.numel(), self._part.data_ptr(), ctypes.c_void_p(self._part_mc),
                ctypes.c_void_p(self._y_mc), ptrs([b + lo.counts_offset for b in bases]),
                ptrs([b + lo.done_count_offset for b in bases]), W, self.rank, e, self.m, self.act.shape[1],
                x.shape[1], self.hidden, tune, main.cuda_stream))
            target = (e * self.done_per_epoch + 2 ** 31) % 2 ** 32 - 2 ** 31  # int32 wrap, as the counters
            N.check(lib.axon_tp_wait_count(mine + lo.done_count_offset, target, main.cuda_stream))
            return self.y
        if self.whole_step:
            bases = self.peers.bases
            N.check(lib.axon_tp_mlp_step(
                x.data_ptr(), self.w_gate.data_ptr(), self.w_up.data_ptr(), self.w_down_h.data_ptr(),
                self.ws.data_ptr(), self.ws.numel(), mine + lo.inbox_offset(0),
                ptrs([b + lo.inbox_offset(0) for b in bases]), ptrs([b + lo.counts_offset for b in bases]),
                ptrs([b + lo.done_count_offset for b in bases]), y_ptrs, W, self.rank, e, self.m,
                self.act.shape[1], x.shape[1], self.hidden, tune, main.cuda_stream))
            target = (e * self.done_per_epoch + 2 ** 31) % 2 ** 32 - 2 ** 31  # int32 wrap, as the counters
            N.check(lib.axon_tp_wait_count(mine + lo.done_count_offset, target, main.cuda_stream))
            return self.y
        if len(self.slabs) == 1 and self.fused_kernel:
            # one slab: both GEMMs in one kernel, the down projection's rows
            # scattered to the owners as its tiles finish
            rows = self.m // W
            inboxes = ptrs([base + lo.inbox_offset(0) for base in self.peers.bases])
            N.check(lib.axon_tp_mlp_partial(x.data_ptr(), self.w_gate.data_ptr(), self.w_up.data_ptr(),
                                            self.w_down_h.data_ptr(), self.ws.data_ptr(), self.ws.numel(), inboxes,
                                            W, self.rank, self.m, self.act.shape[1], x.shape[1], self.hidden, rows,
                                            tune, main.cuda_stream))
            N.check(lib.axon_tp_signal(ptrs([base + lo.arrive_offset(0) for base in self.peers.bases]), W,
                                       self.rank, e, main.cuda_stream))
            self._reduce(lib, mine + lo.inbox_offset(0), y_ptrs, mine + lo.arrive_offset(0), e, rows, 0, out_code,
                         0, main)
            N.check(lib.axon_tp_signal(ptrs([base + lo.done_offset(0) for base in self.peers.bases]), W,
                                       self.rank, e, main.cuda_stream))
            N.check(lib.axon_tp_wait(mine + lo.done_offset(0), W, e, main.cuda_stream))
            return self.y
        for i, (a, b) in enumerate(self.slabs):
            rows = (b - a) // W
            ops.gemm(x[a:b], self.w_gate, b2=self.w_up, epilogue=N.AXON_EPI_SILU_GATE, out=self.act[a:b],
                     tune=self.tune)
            inboxes = ptrs([base + lo.inbox_offset(a) for base in self.peers.bases])
            N.check(lib.axon_tp_down_partial(self.act[a:b].data_ptr(), self.w_down_h.data_ptr(), inboxes, W,
                                             self.rank, b - a, self.hidden, self.act.shape[1], rows, N.AXON_F16,
                                             tune, main.cuda_stream))
            N.check(lib.axon_tp_signal(ptrs([base + lo.arrive_offset(i) for base in self.peers.bases]), W,
                                       self.rank, e, main.cuda_stream))
            # earlier slabs reduce on a side stream with a small grid, beside
            # the next slab's GEMMs; the last slab has the whole GPU
            last = i == len(self.slabs) - 1
            st = main if last else self.side
            if not last:
                self.side.wait_stream(main)
            self._reduce(lib, mine + lo.inbox_offset(a), y_ptrs, mine + lo.arrive_offset(i), e, rows, a, out_code,
                         0 if last else self.reduce_ctas, st)
            N.check(lib.axon_tp_signal(ptrs([base + lo.done_offset(i) for base in self.peers.bases]), W,
                                       self.rank, e, st.cuda_stream))
        main.wait_stream(self.side)
        for i in range(len(self.slabs)):
            N.check(lib.axon_tp_wait(mine + lo.done_offset(i), W, e, main.cuda_stream))
        return self.y

    def _reduce(self, lib, inbox, y_ptrs, arrive, e, rows, row0, out_code, ctas, stream) -> None:
        """Owner side of a slab: sum this rank's rows and put them into every
        rank's output (bulk copies from the reducing SMs, or a local write
        and then one copy-engine transfer per peer)."""
        import ctypes

        from . import _native as N

        W = self.world
        if self._y_mc:
            N.check(lib.axon_tp_reduce_multicast(inbox, ctypes.c_void_p(self._y_mc), arrive, W, self.rank, e, rows,
                                                 self.hidden, row0, self.hidden, out_code, ctas, stream.cuda_stream))
            return
        if not self.copy_engine_gather:
            N.check(lib.axon_tp_reduce_gather(inbox, y_ptrs, arrive, W, self.rank, e, rows, self.hidden, row0,
                                              self.hidden, out_code, ctas, stream.cuda_stream))
            return
        first = (row0 + self.rank * rows) * self.hidden * self.y.element_size()
        nbytes = rows * self.hidden * self.y.element_size()
        N.check(lib.axon_tp_reduce_local(inbox, ctypes.c_void_p(y_ptrs[self.rank]), arrive, W, self.rank, e, rows,
                                         self.hidden, row0, self.hidden, out_code, ctas, stream.cuda_stream))
        dsts = (ctypes.c_void_p * W)(*[y_ptrs[d] + first for d in range(W)])
        N.check(lib.axon_tp_push_rows(ctypes.c_void_p(y_ptrs[self.rank] + first), dsts, nbytes, W, self.rank,
                                      stream.cuda_stream))

    def status(self) -> None:
        from . import _native as N

        N.check(N.lib().axon_tp_status(torch.cuda.current_stream(self.w_gate.device).cuda_stream))
