"""Host logic of the multi-GPU paths on CPU ranks (gloo, world size 2).

The CUDA kernels are replaced by float64 numpy stand-ins of the same three
calls (cast, SiLU-gate GEMM, down GEMM) so the shard ranges, the slab
schedule and the asynchronous all-reduces run exactly as on GPUs; the result
must equal the unsharded float64 oracle.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from enzyme_b200 import tp


class _CpuOps:
    def cast(self, src, dtype, out):
        out.copy_(src.to(out.dtype))
        return out

    def gate_up(self, x, w_gate, w_up, out):
        h1 = x.double() @ w_gate.double()
        h2 = x.double() @ w_up.double()
        out.copy_((h1 / (1 + torch.exp(-h1)) * h2).to(out.dtype))
        return out

    def down(self, act, w_down, out):
        out.copy_((act.double() @ w_down.double()).to(out.dtype))
        return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, h, inter, slabs, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(m, h, generator=g, dtype=torch.float64)
        wg = 0.1 * torch.randn(h, inter, generator=g, dtype=torch.float64)
        wu = 0.1 * torch.randn(h, inter, generator=g, dtype=torch.float64)
        wd = 0.1 * torch.randn(inter, h, generator=g, dtype=torch.float64)
        shards = tp.shard_swiglu(wg, wu, wd, rank, world)
        mod = tp.TPSwiGLU(*shards, slabs=slabs, ops=_CpuOps(), act_dtype=torch.float64)
        y = mod.forward(x, out=torch.empty(m, h, dtype=torch.float64))
        h1, h2 = x @ wg, x @ wu
        want = (h1 / (1 + torch.exp(-h1)) * h2) @ wd
        q.put((rank, float((y.double() - want).abs().max()), len(mod.slab_bounds(m))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("slabs", [1, 3])
def test_tp_swiglu_two_ranks_matches_unsharded(slabs):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 300, 16, 24, slabs, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, err, nslabs in res:
        assert err < 1e-10, (rank, err)
        assert nslabs == min(slabs, 3)


def test_shard_ranges_cover_exactly_once():
    for total in (0, 1, 7, 14336, 1_000_000_000):
        for world in (1, 2, 3, 4, 8):
            spans = [tp.shard_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    assert tp.adam_shard(1_000_000_000, 7, 8) == slice(875_000_000, 1_000_000_000)
    with pytest.raises(ValueError):
        tp.shard_range(10, 2, 2)


def test_slab_bounds_are_whole_tiles():
    mod = tp.TPSwiGLU(torch.zeros(4, 8), torch.zeros(4, 8), torch.zeros(8, 4), slabs=4, ops=_CpuOps())
    b = mod.slab_bounds(4096)
    assert b == [(0, 1024), (1024, 2048), (2048, 3072), (3072, 4096)]
    assert mod.slab_bounds(300) == [(0, 128), (128, 256), (256, 300)]


def test_plans_follow_the_reference_laws():
    # the contraction over the sharded intermediate class is a partial sum
    assert tp.SWIGLU_PLAN["w_down"] == "S(0)" and tp.SWIGLU_PLAN["y_partial"] == "P(+)"
    assert tp.SWIGLU_PLAN["w_gate"] == tp.SWIGLU_PLAN["w_up"] == "S(1)"
    assert set(tp.ADAM_PLAN.values()) == {"S(0)"}


def _adam_worker(rank, world, port, n, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import f64

        rng = np.random.default_rng(1)
        p = 0.02 * rng.standard_normal(n)
        g = 1e-3 * rng.standard_normal(n)
        z = np.zeros(n)
        sl = tp.adam_shard(n, rank, world)
        mine = f64.adam(p[sl], g[sl], z[sl], z[sl], 1e-3, 1.2, 0.1, beta1=0.9, beta2=0.95)[0]
        full = torch.zeros(n, dtype=torch.float64)
        full[sl] = torch.from_numpy(mine)
        dist.all_reduce(full)  # test-side gather only; the step itself has no collective
        want = f64.adam(p, g, z, z, 1e-3, 1.2, 0.1, beta1=0.9, beta2=0.95)[0]
        q.put(float(np.abs(full.numpy() - want).max()))
    finally:
        dist.destroy_process_group()


def test_sharded_adam_two_ranks_equals_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_adam_worker, args=(r, 2, port, 1001, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert max(q.get(timeout=5) for _ in range(2)) == 0.0


def test_fused_slabs_and_layout():
    assert tp.fused_slabs(4096, 8, 2) == [(0, 2048), (2048, 4096)]
    assert tp.fused_slabs(1024, 2, 3) == [(0, 342), (342, 684), (684, 1024)]
    for m, w, s in [(4096, 8, 4), (1000, 4, 3), (64, 8, 16)]:
        sl = tp.fused_slabs(m, w, s)
        assert sl[0][0] == 0 and sl[-1][1] == m
        assert all(b > a and (b - a) % w == 0 for a, b in sl)
        assert all(sl[i][1] == sl[i + 1][0] for i in range(len(sl) - 1))
    with pytest.raises(ValueError):
        tp.fused_slabs(1001, 4, 2)
    lo = tp.PeerLayout(m=4096, hidden=4096, world=8, nslabs=2, out_itemsize=2)
    assert lo.inbox_bytes == 4096 * 4096 * 2
    assert lo.y_offset % 256 == 0 and lo.y_offset >= lo.inbox_bytes
    assert lo.flags_offset >= lo.y_offset + 4096 * 4096 * 2
    # slab regions of the inbox do not overlap and end inside it
    assert lo.inbox_offset(2048) == 2048 * 4096 * 2
    assert lo.inbox_offset(4096) == lo.inbox_bytes
    flags = {lo.arrive_offset(0), lo.done_offset(0), lo.arrive_offset(1), lo.done_offset(1)}
    assert len(flags) == 4 and max(flags) + 8 * 4 <= lo.counts_offset
    # whole-step counts: one per 256-row block, then the done count
    assert lo.counts_offset % 256 == 0
    assert lo.done_count_offset >= lo.counts_offset + 16 * 4
    assert lo.done_count_offset + 4 <= lo.total_bytes
