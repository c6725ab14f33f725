"""Failure detection without a GPU fault.

The device side: every wait in the kernels is bounded. The diagnostic entry
point runs the same bounded waits on an mbarrier nothing arrives on and on a
flag nothing sets; both must give up with AXON_E_TIMEOUT after about the
limit, and the context must stay usable. The host side: a worker that fails
becomes an error row (tested in test_bench_runner.py); a rank that never
joins ends the others' collective with an error after a short process-group
timeout (CPU ranks over gloo, below).
"""

from __future__ import annotations

import os
import socket
import time

import pytest
import torch

from enzyme_b200 import _native as N


@pytest.mark.gpu
def test_bounded_waits_time_out_and_the_context_survives(cuda_device):
    status = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = N.lib().axon_selftest_bounded_wait(200_000_000, status.data_ptr(), flag.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == N.AXON_OK, N.last_error()
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert status.tolist() == [N.AXON_E_TIMEOUT, N.AXON_E_TIMEOUT]
    assert 0.35 <= elapsed < 10.0  # two waits of 0.2 s each gave up, then the kernel returned
    # the context still works
    from enzyme_b200 import ops

    x = torch.randn(4, 256, device=cuda_device)
    torch.testing.assert_close(ops.softmax(x), torch.softmax(x, dim=1), rtol=1e-5, atol=1e-6)


@pytest.mark.gpu
def test_set_flag_is_seen(cuda_device):
    status = torch.full((2,), 99, dtype=torch.int32, device=cuda_device)
    flag = torch.ones(1, dtype=torch.int32, device=cuda_device)
    rc = N.lib().axon_selftest_bounded_wait(50_000_000, status.data_ptr(), flag.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == N.AXON_OK
    torch.cuda.synchronize()
    assert status.tolist() == [N.AXON_E_TIMEOUT, N.AXON_OK]


def test_selftest_limits_checked_on_host():
    assert N.lib().axon_selftest_bounded_wait(0, None, None, None) == N.AXON_E_ARG
    fake = 0x1000
    assert N.lib().axon_selftest_bounded_wait(10 * 10**9, fake, fake, None) == N.AXON_E_ARG


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=3))
    try:
        if rank == 1:
            q.put((1, "left"))  # leaves between steps: never enters the collective
            return
        t = torch.ones(4)
        t0 = time.time()
        try:
            dist.all_reduce(t)
            q.put((0, "completed"))
        except Exception as e:  # the short timeout ends the wait with an error
            q.put((0, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_missing_rank_ends_collective_with_error():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    got = dict(q.get(timeout=5) for _ in range(2))
    assert got[1] == "left"
    assert got[0].startswith("error after"), got[0]
