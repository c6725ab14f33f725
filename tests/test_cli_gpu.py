"""The drop-in leg on a B200: `python -m enzyme_b200 kernels/<spec> --sizes ...`
end to end through real CUDA launches, and the case driver on the
reference's eval cases.

This is the path Axon's `axon kernels/<name> --sizes ...` takes
(src/axon/cli.py:1042-1126 `_run`, src/axon/bench_runner.py:576-825
`run_nki_bench`, :144-223 the device bench, :703-717 the on-device check):
variant modules are written, every selected tile key is benched in a spawned
device worker (CUDA graph, L2 flushed per iteration), its outputs are checked
against the spec's reference, the per-variant CSV is published and the
fastest correct row is exported with its provenance. Each run happens in a
subprocess, as a user would start it.
"""

from __future__ import annotations

import ast
import os
import subprocess
import sys
from pathlib import Path

import pandas as pd
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from enzyme_b200.bench_runner import result_columns, tile_cols  # noqa: E402
from enzyme_b200.specs import load_spec  # noqa: E402

pytestmark = pytest.mark.gpu


def _reference_columns(spec) -> list[str]:
    """Axon's CSV columns in order (src/axon/bench_runner.py:364-388)."""
    return [*spec.dim_vars, "lnc", "sharding", "hw_variant", "tile_variant", *tile_cols(spec.tile_args),
            "mean_ms", "median_ms", "min_ms", "max_ms", "std_dev_ms", "correct", "max_abs_err", "error", "mode"]


def _env():
    env = dict(os.environ)
    env["PYTHONPATH"] = str(ROOT) + os.pathsep + env.get("PYTHONPATH", "")
    return env


def _provenance(path: Path) -> dict:
    for line in path.read_text().splitlines():
        if line.startswith("WINNER_PROVENANCE = "):
            return ast.literal_eval(line.split("=", 1)[1].strip())
    raise AssertionError(f"no WINNER_PROVENANCE in {path}")


# spec, sizes, rtol, atol, case id, rows that must be correct (None: every row)
CLI_CASES = [
    ("rmsnorm_llama", [2048, 4096], 1e-2, 1e-2, "config", None),
    # rel 1e-5 against float64 (the spec's baseline_op evaluates in float64)
    ("cumsum_nucleus_sorted", [256, 128256], 1e-5, 1e-7, "config", None),
    # a small SwiGLU: one bf16 activation term (hw_variant 0) may miss 1e-2 at
    # N(0, 0.02) weights; the f16 activation variants (3, 4) must not
    ("silu_mlp_swiglu", [512, 2048, 1024, 1024], 1e-2, 1e-2, "small", (3, 4)),
]


@pytest.mark.parametrize("name,sizes,rtol,atol,case,must", CLI_CASES, ids=[c[0] for c in CLI_CASES])
def test_cli_drop_in_leg_on_gpu(name, sizes, rtol, atol, case, must, tmp_path):
    out = tmp_path / f"{name}_{case}.csv"
    cmd = [sys.executable, "-m", "enzyme_b200", str(ROOT / "kernels" / name), "--sizes", *map(str, sizes),
           "--rtol", repr(rtol), "--atol", repr(atol), "--out", str(out), "--warmup", "3", "--bench", "10"]
    r = subprocess.run(cmd, cwd=tmp_path, env=_env(), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    spec = load_spec(ROOT / "kernels" / name)
    df = pd.read_csv(out)
    # the reference's columns first, in order, then this backend's
    assert list(df.columns) == result_columns(spec)
    assert list(df.columns)[:len(_reference_columns(spec))] == _reference_columns(spec)
    assert len(df) >= 2 and df["error"].isna().all(), df[["hw_variant", "tile_variant", "error"]].to_string()
    assert df["median_ms"].notna().all() and (df["median_ms"] > 0).all()
    assert (df["mode"] == "device").all() and (df["n_gpus"] == 1).all()
    correct = df["correct"].astype(str).str.lower() == "true"
    if must is None:
        assert correct.all(), df[["hw_variant", "tile_variant", "correct", "max_abs_err"]]
    else:
        assert correct[df["hw_variant"].isin(must)].all(), df[["hw_variant", "correct", "max_abs_err"]]
    # the exported winner: the fastest correct row, with the device recorded
    winner = tmp_path / "winners" / f"{name}_{case}.py"
    assert winner.is_file() and (tmp_path / "winners" / f"{name}_{case}_case.py").is_file()
    prov = _provenance(winner)
    assert "B200" in prov["device"], prov
    best = df[correct].sort_values("median_ms").iloc[0]
    assert prov["hw_variant"] == int(best["hw_variant"]) and prov["median_ms"] == pytest.approx(best["median_ms"])


# one reference eval case (eval/sizes.json) per implemented spec family, run
# the way `make <kernel>_<case>` runs it
DRIVER_CASES = ["rmsnorm_h4096", "layernorm_llama70b", "softmax_sq1k", "rope_llama3_8b", "cumsum_nucleus",
                "fused_adam_opt_1m", "matmul_sq1k", "rmsnorm_matmul_sq1k", "qkv_cte_vision_l4",
                "softmax_mm_sq1k", "attention_nkilib_d128"]


@pytest.mark.parametrize("case", DRIVER_CASES)
def test_case_driver_on_gpu(case, tmp_path):
    from enzyme_b200 import cases

    kernel, cid, c = cases.resolve(case)
    r = subprocess.run([sys.executable, "-m", "enzyme_b200.cases", "run", case, "--warmup", "3", "--bench", "10"],
                       cwd=tmp_path, env=_env(), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    df = pd.read_csv(tmp_path / "out" / f"{kernel}_{cid}.csv")
    assert df["median_ms"].notna().any()
    assert (df["correct"].astype(str).str.lower() == "true").any(), df[["hw_variant", "correct", "max_abs_err"]]
    if "rtol" in c:  # head-to-head: the winner, its harness and the specialized deliverable
        assert (tmp_path / "out" / "winners" / f"{kernel}_{cid}.py").is_file()
        assert (tmp_path / "out" / "winners" / f"{kernel}_{cid}_case.py").is_file()
        text = (tmp_path / "winners" / f"{kernel}_{cid}.py").read_text()
        assert "measured on   : NVIDIA B200" in text and "us median (on-device, correct" in text


def test_case_driver_fails_loud_on_silu_mlp_sq1k(tmp_path):
    """silu_mlp sq1k (eval/sizes.json: m = n = k = p = 1024, every input
    N(0, 1)) is a bench-only case checked at Axon's permissive default
    rtol = atol = 2e-2 (src/axon/cli.py:59-62). Its outputs have a standard
    deviation of about 23000 and arise from sums of 1024 terms of about 700,
    so a few outputs near zero carry an fp32 accumulation error of a few
    hundredths: every variant, including the three-term (near-fp32)
    activation, is verified wrong at the 0.02 absolute floor. Axon's winner
    rule then fails the case loudly (src/axon/winner.py pick_winner: "Only
    when every timed variant is verified incorrect does this fail loud");
    the case driver must do the same, after benching and publishing every
    key."""
    kernel, cid = "silu_mlp", "sq1k"
    r = subprocess.run([sys.executable, "-m", "enzyme_b200.cases", "run", f"{kernel}_{cid}", "--warmup", "3",
                        "--bench", "10"], cwd=tmp_path, env=_env(), capture_output=True, text=True, timeout=900)
    assert r.returncode != 0
    assert "failed on-device correctness" in r.stdout + r.stderr, r.stdout[-3000:] + r.stderr[-3000:]
    df = pd.read_csv(tmp_path / "out" / f"{kernel}_{cid}.csv")
    assert len(df) >= 5 and df["error"].isna().all(), df[["hw_variant", "tile_variant", "error"]].to_string()
    assert df["median_ms"].notna().all() and (df["median_ms"] > 0).all()
    assert not (df["correct"].astype(str).str.lower() == "true").any()
