"""Multi-GPU paths on real GPUs (two ranks over NCCL; skipped on a 1-GPU box).

* Tensor-parallel SwiGLU: two ranks, each with its column/row shard, slabbed
  all-reduce of fp32 partials; the full output is checked on sampled rows
  against the float64 oracle of the unsharded MLP.
* Parameter-sharded Adam: each rank updates its contiguous slice; the
  gathered result equals a one-GPU update of the whole vector.
* Fused tensor-parallel SwiGLU: the down GEMM's epilogue scatters f16
  partial rows into the owners' inboxes over peer memory, owners reduce and
  push bf16 rows to every rank (bulk copies, copy engines, or one multicast
  store per packet through the NVLink switch); checked against the oracle,
  across ranks and over repeated steps (epoch flags), and on one rank
  without a process group.
* The whole step in one kernel, its reduction warps resolving the
  all-reduce beside the GEMM tiles, through the owners' inboxes or through
  the NVLink switch (multimem.ld_reduce of the partials, multimem.st of the
  sums).
* The BASELINE SwiGLU config on every GPU of the box (the largest power of
  two up to 8), default path and whole step.
* A flag wait that nobody satisfies gives up with AXON_E_TIMEOUT and the
  context stays usable.
NVLS is off (NCCL_NVLS_ENABLE=0) and the process group has a short timeout.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from enzyme_b200 import ops, tp

        dev = torch.device("cuda", rank)
        g = torch.Generator().manual_seed(0)
        m, h, inter = 512, 1024, 2048
        x = torch.randn(m, h, generator=g).bfloat16()
        wg = (0.02 * torch.randn(h, inter, generator=g)).bfloat16()
        wu = (0.02 * torch.randn(h, inter, generator=g)).bfloat16()
        wd = (0.02 * torch.randn(inter, h, generator=g)).bfloat16()
        shards = [s.to(dev) for s in tp.shard_swiglu(wg, wu, wd, rank, world)]
        y = tp.TPSwiGLU(*shards, slabs=3).forward(x.to(dev))
        torch.cuda.synchronize()
        ops.gemm_status()
        # adam: 10_000_003 params, each rank its slice
        n = 10_000_003
        gen = torch.Generator().manual_seed(1)
        p = 0.02 * torch.randn(n, generator=gen)
        gr = (1e-3 * torch.randn(n, generator=gen)).bfloat16()
        sl = tp.adam_shard(n, rank, world)
        pd, gd = p[sl].to(dev), gr[sl].to(dev)
        md, vd = torch.zeros_like(pd), torch.zeros_like(pd)
        ops.adam(pd, gd, md, vd, step_size=1e-3, inv_bc2_sqrt=1.2, wd=0.1, beta1=0.9, beta2=0.95, out=(pd, md, vd))
        full = torch.zeros(n, device=dev)
        full[sl] = pd
        dist.all_reduce(full)  # gather for the check only
        whole = p.to(dev)
        zm, zv = torch.zeros_like(whole), torch.zeros_like(whole)
        ops.adam(whole, gr.to(dev), zm, zv, step_size=1e-3, inv_bc2_sqrt=1.2, wd=0.1, beta1=0.9, beta2=0.95,
                 out=(whole, zm, zv))
        q.put((rank, y.cpu().numpy(), bool(torch.equal(full, whole))))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_swiglu_and_sharded_adam_two_gpus():
    import torch.multiprocessing as mp

    from oracle import f64

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    g = torch.Generator().manual_seed(0)
    m, h, inter = 512, 1024, 2048
    x = torch.randn(m, h, generator=g).bfloat16().float().numpy()
    wg = (0.02 * torch.randn(h, inter, generator=g)).bfloat16().float().numpy()
    wu = (0.02 * torch.randn(h, inter, generator=g)).bfloat16().float().numpy()
    wd = (0.02 * torch.randn(inter, h, generator=g)).bfloat16().float().numpy()
    rows = np.arange(0, m, 7)
    want = f64.silu_mlp(x[rows], wg, wu, wd)
    for rank, y, adam_equal in res:
        assert adam_equal, f"rank {rank}: sharded Adam differs from the one-GPU update"
        np.testing.assert_allclose(y[rows], want, rtol=1e-2, atol=1e-2)
    np.testing.assert_array_equal(res[0][1], res[1][1])  # every rank holds the same reduced output


def _swiglu_case(m, h, inter, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, h, generator=g).bfloat16()
    wg = (0.02 * torch.randn(h, inter, generator=g)).bfloat16()
    wu = (0.02 * torch.randn(h, inter, generator=g)).bfloat16()
    wd = (0.02 * torch.randn(inter, h, generator=g)).bfloat16()
    return x, wg, wu, wd


def _fused_rank(rank, world, port, q, whole_step=False, ce=False, mc=False):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from enzyme_b200 import ops, tp

        dev = torch.device("cuda", rank)
        x, wg, wu, wd = _swiglu_case(1024, 1024, 2048, 3)
        shards = [s.to(dev) for s in tp.shard_swiglu(wg, wu, wd, rank, world)]
        xd = x.to(dev)
        if mc and not tp.multicast_supported(dev):
            q.put((rank, None, None))  # every rank sees the same GPUs, so all skip
            return
        # whole_step + mc: the all-reduce by the switch (multimem.ld_reduce / multimem.st)
        f = tp.FusedTPSwiGLU(*shards, m=1024, slabs=2, tune={"max_ctas": 132}, whole_step=whole_step,
                             copy_engine_gather=ce, multicast_gather=mc)
        try:
            y1 = f.forward(xd).clone()
            y2 = f.forward(xd).clone()  # second epoch reuses inboxes, output and flags
            torch.cuda.synchronize()
        finally:
            f.close()  # with multicast: a barrier first, so no rank unmaps while another still stores
        f.status()
        ops.gemm_status()
        same = bool(torch.equal(y1, y2))
        if mc and not whole_step:  # the multicast all-gather carries the bits of the bulk-copy push
            plain = tp.FusedTPSwiGLU(*shards, m=1024, slabs=2, tune={"max_ctas": 132})
            same = same and bool(torch.equal(y1, plain.forward(xd)))
            plain.close()
        q.put((rank, y1.float().cpu().numpy(), same))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("whole_step,ce,mc", [(False, False, False), (True, False, False), (False, True, False),
                                              (False, False, True), (True, False, True)])
def test_fused_tp_swiglu_two_gpus(whole_step, ce, mc):
    import torch.multiprocessing as mp

    from oracle import f64

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_rank, args=(r, 2, port, q, whole_step, ce, mc)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    if any(y is None for _, y, _ in res):
        pytest.skip("no NVLink multicast on these GPUs")
    x, wg, wu, wd = (t.float().numpy() for t in _swiglu_case(1024, 1024, 2048, 3))
    rows = np.arange(0, 1024, 5)
    want = f64.silu_mlp(x[rows], wg, wu, wd)
    for rank, y, repeat_equal in res:
        assert repeat_equal, f"rank {rank}: a second step gave different bits"
        np.testing.assert_allclose(y[rows], want, rtol=1e-2, atol=1e-2)
    np.testing.assert_array_equal(res[0][1], res[1][1])


@pytest.mark.parametrize("slabs,whole_step,fused_kernel", [(2, False, None), (1, False, True), (1, False, False),
                                                        (1, True, None)])
def test_fused_tp_single_rank(slabs, whole_step, fused_kernel, cuda_device):
    """world = 1: the same kernels with the inbox and output local; twice, so
    the whole-step kernel's accumulating counts are exercised."""
    from enzyme_b200 import ops, tp
    from oracle import f64

    x, wg, wu, wd = _swiglu_case(512, 512, 1024, 4)
    f = tp.FusedTPSwiGLU(wg.to(cuda_device), wu.to(cuda_device), wd.to(cuda_device), m=512, slabs=slabs,
                         whole_step=whole_step, fused_kernel=fused_kernel)
    y1 = f.forward(x.to(cuda_device)).clone()
    y = f.forward(x.to(cuda_device))
    torch.cuda.synchronize()
    f.status()
    ops.gemm_status()
    assert torch.equal(y1, y)
    rows = np.arange(0, 512, 3)
    want = f64.silu_mlp(*(t.float().numpy() for t in (x[rows], wg, wu, wd)))
    np.testing.assert_allclose(y.float().cpu().numpy()[rows], want, rtol=1e-2, atol=1e-2)
    f.close()


def test_tp_flag_wait_times_out(cuda_device):
    """Flags nobody raises: the bounded wait gives up, reports AXON_E_TIMEOUT,
    and the context keeps working."""
    from enzyme_b200 import _native as N
    from enzyme_b200 import ops

    flags = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    N.check(N.lib().axon_tp_wait(flags.data_ptr(), 4, 1, s))
    with pytest.raises(N.AxonError) as e:
        N.check(N.lib().axon_tp_status(s))
    assert e.value.code == N.AXON_E_TIMEOUT
    N.check(N.lib().axon_tp_status(s))  # the record was cleared
    a = torch.randn(256, 256, device=cuda_device).bfloat16()
    assert torch.isfinite(ops.gemm(a, a, out_dtype=torch.float32)).all()


CONFIG_ROW_STRIDE = 61


def _config_tensors(dev):
    """x [4096, 4096] and the full W_gate, W_up [4096, 14336], W_down [14336, 4096]
    (bf16, N(0, 0.02) weights), drawn from one seeded generator on `dev`."""
    m, h, inter = 4096, 4096, 14336
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(m, h, device=dev, generator=g).bfloat16()
    full = [(0.02 * torch.randn(*shape, device=dev, generator=g)).bfloat16()
            for shape in ((h, inter), (h, inter), (inter, h))]
    return x, full


def _config_rank(rank, world, port, q, whole_step=False, mc=False):
    """One rank of the fused path at the BASELINE SwiGLU config (m 4096,
    hidden 4096, inter 14336): the same seeded full weights on every rank,
    this rank's column/row shard, three steps; returns the sampled rows and a
    checksum of the raw output bits."""
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from enzyme_b200 import ops, tp

        dev = torch.device("cuda", rank)
        m, h = 4096, 4096
        x, full = _config_tensors(dev)
        shards = tp.shard_swiglu(*full, rank, world)
        if mc and not tp.multicast_supported(dev):
            q.put((rank, None, True, None))  # every rank sees the same GPUs, so all skip
            return
        f = tp.FusedTPSwiGLU(*shards, m=m, slabs=1, whole_step=whole_step, multicast_gather=mc)
        try:
            ys = [f.forward(x).clone() for _ in range(3)]
            torch.cuda.synchronize()
        finally:
            f.close()
        f.status()
        ops.gemm_status()
        repeat_equal = all(torch.equal(ys[0], y) for y in ys[1:])
        words = ys[0].view(torch.int16).to(torch.int64)
        checksum = (int(words.sum()), int((words * torch.arange(1, h + 1, device=dev)).sum()))
        rows = torch.arange(0, m, CONFIG_ROW_STRIDE, device=dev)
        q.put((rank, ys[0][rows].float().cpu().numpy(), repeat_equal, checksum))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("whole_step,mc", [(False, False), (True, False), (True, True)])
def test_fused_tp_swiglu_config_shape_all_gpus(whole_step, mc):
    """The fused tensor-parallel path at the BASELINE config on every GPU of
    the box (the largest power of two up to 8): sampled rows against the
    float64 oracle of the unsharded MLP at rtol = atol = 1e-2, bit-identical
    outputs on every rank and over repeated steps."""
    import torch.multiprocessing as mp

    from oracle import f64

    world = 1 << (min(torch.cuda.device_count(), 8).bit_length() - 1)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_config_rank, args=(r, world, port, q, whole_step, mc)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=600) for _ in range(world)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    if any(y is None for _, y, _, _ in res):
        pytest.skip("no NVLink multicast on these GPUs")
    x, full = _config_tensors(torch.device("cuda", 0))  # the same draws as every rank's
    rows = torch.arange(0, x.shape[0], CONFIG_ROW_STRIDE, device=x.device)
    want = f64.silu_mlp(x[rows].float().cpu().numpy(), *(w.float().cpu().numpy() for w in full))
    del x, full
    for rank, y, repeat_equal, checksum in res:
        assert repeat_equal, f"rank {rank}: repeated steps gave different bits"
        assert checksum == res[0][3], f"rank {rank} holds a different output than rank 0"
        np.testing.assert_allclose(y, want, rtol=1e-2, atol=1e-2)
