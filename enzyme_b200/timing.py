"""Device timing: CUDA events on the launching stream, CUDA graphs for
launch-bound loops, and an nvidia-smi clock sampler for the timed region."""

from __future__ import annotations

import csv
import io
import statistics
import subprocess
import time
from collections.abc import Callable

import torch

L2_BYTES = 126 * 1024 * 1024  # B200 L2


def sets_to_defeat_l2(set_bytes: int, factor: float = 2.0) -> int:
    """How many distinct buffer sets a rotation needs so that the working set
    exceeds `factor` x L2 (each launch then reads from HBM)."""
    if set_bytes <= 0:
        return 1
    return max(1, int(-(-factor * L2_BYTES // set_bytes)))


def capture_graph(fn: Callable[[int], None], launches: int, stream: torch.cuda.Stream | None = None):
    """Capture `fn(i)` for i in range(launches) into one CUDA graph."""
    g = torch.cuda.CUDAGraph()
    s = stream or torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(0)  # warm the launch path outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=s):
        for i in range(launches):
            fn(i)
    torch.cuda.synchronize()
    return g


def time_graph(g: torch.cuda.CUDAGraph, reps: int = 1) -> float:
    """Milliseconds of `reps` replays, events recorded on the current stream."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(reps):
        g.replay()
    end.record()
    end.synchronize()
    return start.elapsed_time(end)


def time_calls(fn: Callable[[int], None], iters: int) -> list[float]:
    """Per-call milliseconds of `fn(i)` (events around each call)."""
    out = []
    for i in range(iters):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn(i)
        b.record()
        b.synchronize()
        out.append(a.elapsed_time(b))
    return out


QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """Samples SM clocks and throttle reasons every 200 ms while active."""

    def __init__(self, gpu_index: int = 0):
        self.gpu = gpu_index
        self.proc = None
        self.t0 = 0.0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        self.t0 = time.time()
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            # make sure at least one sample landed inside the region
            if time.time() - self.t0 < 0.3:
                time.sleep(0.3 - (time.time() - self.t0))
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()
        return False

    def summary(self) -> dict:
        rows = [r for r in csv.reader(io.StringIO(self.out or "")) if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons,
            "samples": len(rows),
        }
