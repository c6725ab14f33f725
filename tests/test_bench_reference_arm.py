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
    w = bench.WORKLOADS[name](None, 0, 1)  # dev=None: sizes and the CPU sample only
    work, sample = w.cpu_step()
    assert work > 0 and sample
    assert w.metric().endswith(f"({w.name})") and w.unit in ("GB/s", "TFLOP/s")


def test_headline_is_the_tensor_parallel_mlp():
    assert bench.HEADLINE == "silu_mlp"
    w = bench.WORKLOADS[bench.HEADLINE](None, 0, 8)
    assert w.shard == 14336 // 8 and w.scaling == "strong" and w.kind == "tensor"
    # whole-job work is the unsharded chain's 6 m h i FLOPs at any rank count
    assert w.job_work() == 6.0 * 4096 * 4096 * 14336


def test_line_with_every_workload_fits_the_kept_tail():
    """The driver keeps about 3000 characters of stdout: a realistic line
    with every extra workload in compact form stays under that."""
    r = {"value": 5933.82424, "unit": "GB/s", "ms_per_step": 0.0144927993, "clocks": {"sm_mhz": 1965.0, "reasons": ["sw_power_cap"]},
         "roofline": {"frac": 0.91093434}}
    extra = {name: bench.compact(r) for name in bench.WORKLOADS if name != bench.HEADLINE}
    head = {"metric": "bf16 TFLOP/s (silu_mlp)", "value": 1395.09321, "unit": "TFLOP/s", "n_gpus": 8, "steps": 20,
            "warmup": 5, "ms_per_step": 1.03441762, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded randn on device; no dataset)",
            "config": {"workload": "silu_mlp_swiglu: m 4096, h 4096, inter 14336, bf16, W ~ N(0, 0.02), f16 act",
                       "parallelism": "tp8 (reduce-scatter in the down GEMM over NVLink, owner reduce + "
                                      "all-gather push)",
                       "l2": "x over 2 buffers; 155 MiB touched per GPU per step > L2",
                       "timing": "median of 8 x 20 steps (43.2 ms)"},
            "roofline": {"bound": "tensor", "achieved": 1395.093210576428, "peak": 1353.4, "unit": "TFLOP/s",
                         "frac": 1.0308062735159065, "peak_source": "measured", "peak_kind": "sustained",
                         "frac_of_burst": 0.8388510676305863, "traffic": 607000000,
                         "traffic_source": "profiles/gemm_tcgen05_pair__swiglu_4096x4096x14336.md",
                         "traffic_kind": "dram read+write of one launch"},
            "clocks": {"sm_mhz": 1957.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 31,
                       "window": "soak + warmup + timed repeats"},
            "e2e": {"value": 612.3456, "unit": "TFLOP/s", "h2d_bytes_per_step": 33554432,
                    "d2h_bytes_per_step": 33554432, "ms_per_step": 2.3566, "steps": 20},
            "gpu_launches": 800,
            "parity": {"rows": 43, "worst_err_over_tol": 0.3612345, "ranks_identical": True,
                       "tol": "rtol=atol=1e-2 vs oracle.f64.silu_mlp", "finite": True},
            "cpu_baseline": {"value": 1.5123, "unit": "TFLOP/s", "cores": 32, "kind": "port",
                             "sample": "64 of 4096 tokens (fp32 torch, same weights shape)", "seconds": 12.0},
            "workloads": extra}
    assert len(json.dumps(head)) < 2900, len(json.dumps(head))


@pytest.mark.parametrize("name", ["qkv_cte", "attention"])
def test_reference_line(name):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", name,
                          "--steps", "2", "--warmup", "3"], capture_output=True, text=True, timeout=300, check=True)
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    for key in ("metric", "unit", "cpu_baseline", "e2e", "higher_is_better", "config"):
        assert key in line
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_every_workload_has_an_end_to_end_path():
    """`python bench.py --workload NAME` reports `e2e` for any workload: each
    class either defines its own end-to-end step or names the inputs and the
    output the generic one copies."""
    import bench

    for name, make in bench.WORKLOADS.items():
        cls = getattr(make, "cls", make)
        own = "e2e_setup" in vars(cls) or any("e2e_setup" in vars(b) for b in cls.__mro__[1:-1]
                                              if b is not bench.Workload)
        generic = "e2e_inputs" in vars(cls) and "e2e_output" in vars(cls)
        assert own or generic, name
