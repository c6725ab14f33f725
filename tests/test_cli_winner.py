"""CLI binding, run paths, candidate filter and winner selection (host only).

Mirrors the behaviours Axon pins in tests/test_cli_sizes.py,
tests/test_candidate_filter.py and tests/test_export_winner.py.
"""

from __future__ import annotations

import csv
import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import KERNELS, load_spec
from enzyme_b200 import cli
from enzyme_b200.bench_runner import result_columns
from enzyme_b200.candidate_filter import (TileConstraint, manifest_literal, read_manifest, rejection_reason,
                                          select_diverse)
from enzyme_b200.case_gen import generate_case_module
from enzyme_b200.paths import run_paths
from enzyme_b200.winner import WinnerRow, export_winner, pick_winner

# ---- CLI ---------------------------------------------------------------------------


def _parse(*argv):
    return cli.build_parser().parse_args([str(a) for a in argv])


def test_sizes_count_mismatch_exits_2(capsys):
    with pytest.raises(SystemExit) as e:
        cli.run(_parse(KERNELS / "rmsnorm", "--sizes", 64))
    assert e.value.code == 2
    assert "expects 2 values" in capsys.readouterr().err


def test_missing_spec_exits_2(tmp_path):
    with pytest.raises(SystemExit) as e:
        cli.run(_parse(tmp_path / "nope", "--sizes", 1))
    assert e.value.code == 2


@pytest.mark.parametrize("flag,value", [("--bench", 0), ("--warmup", -1), ("--rtol", 0), ("--atol", "nan"),
                                        ("--candidate-budget", -2)])
def test_bad_flag_values_rejected(flag, value):
    with pytest.raises(SystemExit):
        _parse(KERNELS / "rmsnorm", "--sizes", 1, 2, flag, value)


def test_head_to_head_stem_must_name_the_kernel(tmp_path, capsys):
    with pytest.raises(SystemExit) as e:
        cli.run(_parse(KERNELS / "rmsnorm", "--sizes", 64, 256, "--rtol", 1e-2, "--atol", 1e-2, "--phase", "emit",
                       "--out", tmp_path / "out/other_case.csv"))
    assert e.value.code == 2
    assert "rmsnorm_<case_id>" in capsys.readouterr().err


def test_emit_phase_writes_variant_modules(tmp_path):
    rc = cli.run(_parse(KERNELS / "rmsnorm", "--sizes", 64, 512, "--phase", "emit", "--out",
                        tmp_path / "out/rmsnorm_h512"))
    assert rc == 0
    mods = sorted((tmp_path / "out/rmsnorm_h512").glob("rmsnorm__v*_t*.py"))
    assert [m.name for m in mods] == ["rmsnorm__v0_t0.py", "rmsnorm__v1_t0.py", "rmsnorm__v2_t0.py"]
    cons = read_manifest(mods[0])
    assert {c.tile_arg for c in cons} == {"TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"}


def test_bench_phase_without_modules_exits_2(tmp_path):
    with pytest.raises(SystemExit) as e:
        cli.run(_parse(KERNELS / "rmsnorm", "--sizes", 64, 512, "--phase", "bench", "--out", tmp_path / "out/x"))
    assert e.value.code == 2


def test_spec_default_dtype():
    assert cli.spec_default_dtype(load_spec("rmsnorm")) == "bfloat16"
    assert cli.spec_default_dtype(load_spec("cumsum")) == "float32"


def test_run_paths_forms(tmp_path, monkeypatch):
    spec = load_spec("matmul")
    monkeypatch.chdir(tmp_path)
    assert run_paths(spec, None).csv == tmp_path / "out" / "nki_matmul.csv"
    assert run_paths(spec, "out/matmul_sq1k").csv == run_paths(spec, "out/matmul_sq1k.csv").csv
    assert run_paths(spec, "res/").csv == tmp_path / "res" / "nki_matmul.csv"
    p = run_paths(spec, "out/matmul_sq1k")
    assert p.run_dir == tmp_path / "out" / "matmul_sq1k"
    assert p.results == p.run_dir / "results.csv"
    assert p.baseline_csv == tmp_path / "out" / "baseline_matmul_sq1k.csv"
    assert p.variant_module("matmul", 2, 3).name == "matmul__v2_t3.py"
    assert p.winner_case("matmul_sq1k").name == "matmul_sq1k_case.py"


# ---- candidate filter ---------------------------------------------------------------


def test_constraint_rules():
    c = TileConstraint("T", extent=1024, tile_size=128, require_divisible=True)
    assert c.rejection_reason(0) and c.rejection_reason(16) and c.rejection_reason(3)
    assert c.rejection_reason(4) is None
    a = TileConstraint("T", extent=8, tile_size=1, require_divisible=True, allowed=(2, 4))
    assert a.rejection_reason(1) and a.rejection_reason(8) and a.rejection_reason(2) is None


def test_manifest_round_trip_and_fail_open(tmp_path):
    cons = [TileConstraint("TILES_IN_BLOCK_N", 512, 64, True, (1, 2)), TileConstraint("TILES_IN_BLOCK_M", 1, 1, True)]
    p = tmp_path / "m.py"
    p.write_text(f"__axon_tile_constraints__ = {manifest_literal(cons)}\n")
    assert sorted(read_manifest(p), key=lambda c: c.tile_arg) == sorted(cons, key=lambda c: c.tile_arg)
    p.write_text("__axon_tile_constraints__ = make()\n")
    assert read_manifest(p) == ()
    assert read_manifest(tmp_path / "missing.py") == ()


def test_rejection_reason_matches_by_name():
    cons = [TileConstraint("B", 4, 1, True)]
    assert rejection_reason(["A", "B"], [32, 4], cons) is None
    assert rejection_reason(["A", "B"], [1, 8], cons) is not None


def test_select_diverse_is_bounded_and_deterministic():
    keys = [(a, b) for a in (1, 2, 4, 8, 16) for b in (1, 2, 4, 8, 16)]
    s1 = select_diverse(keys, budget=6, seed=42)
    assert s1 == select_diverse(list(reversed(keys)), budget=6, seed=42)
    assert len(s1) == 6 and (1, 1) in s1 and (16, 16) in s1
    assert select_diverse(keys, budget=0, seed=1) == sorted(keys)


# ---- winner ---------------------------------------------------------------------------


def _write_csv(path, spec, rows):
    cols = result_columns(spec)
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=cols)
        w.writeheader()
        for r in rows:
            base = {c: "" for c in cols}
            base.update({"m": 64, "n": 512, "lnc": 1, "sharding": "cuda", "TILES_M": 1, "TILES_N": 2,
                         "mean_ms": r["ms"], "min_ms": r["ms"], "max_ms": r["ms"], "std_dev_ms": 0, "mode": "device"})
            base.update({k: v for k, v in r.items() if k != "ms"})
            base["median_ms"] = r["ms"]
            w.writerow(base)


def test_pick_winner_rules(tmp_path, capsys):
    spec = load_spec("rmsnorm")
    p = tmp_path / "r.csv"
    assert pick_winner(p, spec, "median", rtol=1e-2, atol=1e-2) is None
    _write_csv(p, spec, [{"hw_variant": 0, "tile_variant": 0, "ms": 1.0, "correct": False, "max_abs_err": 9},
                         {"hw_variant": 1, "tile_variant": 0, "ms": 2.0, "correct": True},
                         {"hw_variant": 2, "tile_variant": 0, "ms": 3.0, "correct": False}])
    w = pick_winner(p, spec, "median", rtol=1e-2, atol=1e-2)
    assert (w.hw_variant, w.median_ms) == (1, 2.0)
    assert "skipped 1 faster but incorrect" in capsys.readouterr().out
    _write_csv(p, spec, [{"hw_variant": 0, "tile_variant": 0, "ms": 1.0, "correct": False, "max_abs_err": 9},
                         {"hw_variant": 1, "tile_variant": 0, "ms": 2.0, "correct": ""}])
    w = pick_winner(p, spec, "median", rtol=1e-2, atol=1e-2)
    assert w.hw_variant == 1 and "unverified" in capsys.readouterr().out
    _write_csv(p, spec, [{"hw_variant": 0, "tile_variant": 0, "ms": 1.0, "correct": False, "max_abs_err": 9}])
    with pytest.raises(AssertionError, match="failed on-device correctness"):
        pick_winner(p, spec, "median", rtol=1e-2, atol=1e-2)


def test_export_winner_writes_kernel_and_case(tmp_path):
    spec = load_spec("rmsnorm")
    paths = run_paths(spec, str(tmp_path / "out/rmsnorm_h512"))
    from enzyme_b200 import catalogue

    catalogue.emit_variant_modules(spec, {"m": 64, "n": 512}, 2, paths)
    w = WinnerRow(hw_variant=0, tile_variant=0, mean_ms=1.0, median_ms=1.0, min_ms=1.0, sizes=(64, 512),
                  tile_values=(1, 2))
    export_winner(spec, w, case_id="h512", kernel_path=KERNELS / "rmsnorm", paths=paths, dtype="bfloat16",
                  rtol=1e-2, atol=1e-2)
    assert paths.winner_kernel("rmsnorm_h512").is_file()
    case = paths.winner_case("rmsnorm_h512")
    s = importlib.util.spec_from_file_location("_case_under_test", case)
    mod = importlib.util.module_from_spec(s)
    s.loader.exec_module(mod)
    assert mod.CASE["entry_point"] == "rmsnorm" and mod.CASE["shape_args"]["TILES_IN_BLOCK_N"] == 2
    import ast

    tree = ast.parse(paths.winner_kernel("rmsnorm_h512").read_text())
    prov = next(ast.literal_eval(n.value) for n in tree.body if isinstance(n, ast.Assign)
                and getattr(n.targets[0], "id", "") == "WINNER_PROVENANCE")
    assert prov["case"] == "h512" and prov["median_ms"] == 1.0 and prov["tiles"]["TILES_IN_BLOCK_N"] == 2
    ins = mod.make_inputs(m=64, n=512, TILES_IN_BLOCK_M=1, TILES_IN_BLOCK_N=2)
    assert ins["x"].shape == (64, 512) and ins["TILES_IN_BLOCK_N"] == 2
    out = mod.torch_ref(ins["x"], 1, 2)
    assert set(out) == {"output_0"} and str(out["output_0"].dtype) == "torch.bfloat16"
    assert set(mod.output_tensors(ins)) == {"output_0"}
    with pytest.raises(FileNotFoundError):
        export_winner(spec, WinnerRow(5, 0, 1.0, 1.0, 1.0, (64, 512), (1, 1)), case_id="x",
                      kernel_path=KERNELS / "rmsnorm", paths=paths, dtype="bfloat16", rtol=1e-2, atol=1e-2)


def test_case_module_needs_torch_ref():
    spec = load_spec("softmax")
    with pytest.raises(ValueError, match="torch_ref"):
        generate_case_module(spec, KERNELS / "softmax", "float32", Path("/tmp/x_case.py"), name="softmax_x",
                             entry_point="softmax", shape_args={}, rtol=1e-2, atol=1e-2)


# ---- case catalogue ---------------------------------------------------------------


def test_case_catalogue_builds_the_make_target_command():
    from enzyme_b200 import cases

    a = cases.argv("rmsnorm_h4096")
    assert a[0].endswith("kernels/rmsnorm") and a[1:4] == ["--sizes", "1024", "4096"]
    assert a[a.index("--rtol") + 1] == "0.01" and a[-2:] == ["--out", "out/rmsnorm_h4096.csv"]
    a = cases.argv("matmul_ck_16k_l2")
    assert a[a.index("--dtype") + 1] == "float32" and a[a.index("--gpus") + 1] == "2"
    assert "--rtol" not in cases.argv("matmul_sq1k")
    # kernel names with underscores resolve to the longest matching spec
    assert cases.resolve("rmsnorm_matmul_sq1k")[0] == "rmsnorm_matmul"
    assert cases.resolve("silu_mlp_swiglu_config")[0] == "silu_mlp_swiglu"
    with pytest.raises(KeyError):
        cases.resolve("rmsnorm_nope")


def test_every_case_parses_and_matches_its_spec():
    from enzyme_b200 import cases

    for case in cases.all_cases():
        kernel, _, c = cases.resolve(case)
        spec = load_spec(kernel)
        assert len(c["sizes"]) == len(spec.dim_vars), case
        args = cli.build_parser().parse_args(cases.argv(case))
        assert args.sizes == c["sizes"]


def test_every_case_resolves_and_binds_its_spec():
    """Each named case splits back into its own kernel and case id (kernel
    names share prefixes: softmax / softmax_mm, rmsnorm / rmsnorm_matmul),
    names a spec package that loads, and gives one size per dim_var."""
    from enzyme_b200 import cases

    for name in cases.all_cases():
        kernel, cid, c = cases.resolve(name)
        assert f"{kernel}_{cid}" == name
        spec = load_spec(kernel)
        assert len(c["sizes"]) == len(spec.dim_vars), name
        args = cases.argv(name)
        assert args[0].endswith(f"kernels/{kernel}") and args[-1].endswith(f"{kernel}_{cid}.csv")
