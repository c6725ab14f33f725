"""bench.py's reference arm on CPU: every workload's bounded CPU sample runs
without a GPU and reports positive work, and the --impl reference line keeps
the contract's keys."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


@pytest.mark.parametrize("name", sorted(bench.WORKLOADS))
def test_cpu_sample_runs_without_gpu(name):
    cls = bench.WORKLOADS[name]
    w = cls.__new__(cls)
    w.dev, w.rank, w.world = None, 0, 1
    bench._prepare_cpu_only(w)
    work, sample = w.cpu_step()
    assert work > 0 and sample


@pytest.mark.parametrize("name", ["qkv_cte", "attention"])
def test_reference_line(name):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", name,
                          "--steps", "2", "--warmup", "3"], capture_output=True, text=True, timeout=300, check=True)
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    for key in ("metric", "unit", "cpu_baseline", "e2e", "higher_is_better", "config"):
        assert key in line
    assert line["e2e"]["h2d_bytes_per_step"] == 0
