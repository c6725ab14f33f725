"""The winners/ deliverable on CPU: the specialized module binds the fastest
correct row's tile key, and the keep-faster rule of the reference
(tools/specialize_winner.py:351-373) decides whether a re-run replaces it."""

from __future__ import annotations

import ast
import csv

import pytest

from enzyme_b200 import catalogue
from enzyme_b200.bench_runner import result_columns
from enzyme_b200.paths import RunPaths
from enzyme_b200.specialize import KeptExisting, SpecializeError, decide_write, recorded_measurement, specialize

from conftest import load_spec

STEM = "rmsnorm_llama_config"


def _run_dir(tmp_path, rows):
    """An out/ tree as the CLI leaves it: the variant modules and a CSV."""
    spec = load_spec("rmsnorm_llama")
    out = tmp_path / "out"
    paths = RunPaths(csv=out / f"{STEM}.csv")
    catalogue.emit_variant_modules(spec, {"m": 2048, "n": 4096}, 2, paths)
    cols = result_columns(spec)
    with paths.csv.open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=cols)
        w.writeheader()
        for hw, tn, med, ok in rows:
            w.writerow({"m": 2048, "n": 4096, "lnc": 1, "sharding": "cuda", "hw_variant": hw, "tile_variant": 0,
                        "TILES_M": 1, "TILES_N": tn, "mean_ms": med, "median_ms": med, "min_ms": med * 0.9,
                        "max_ms": med * 1.1, "std_dev_ms": 0.0, "correct": ok, "max_abs_err": 1e-3, "error": "",
                        "mode": "device"})
    return out


def test_specialized_module_binds_the_fastest_correct_row(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    out = _run_dir(tmp_path, [(0, 4, 0.0100, True), (2, 8, 0.0061, True), (1, 8, 0.0050, False)])
    p = specialize(STEM, out_root=out, winners_dir=tmp_path / "winners")
    text = p.read_text()
    tree = ast.parse(text)
    fn = [n for n in tree.body if isinstance(n, ast.FunctionDef)][0]
    assert fn.name == "rmsnorm_llama" and [a.arg for a in fn.args.args] == ["x", "w"]
    assert not fn.args.kwonlyargs  # the tile key is bound, not a parameter
    assert "HW_VARIANT = 2" in text and "'TILES_IN_BLOCK_N': 8" in text  # the faster wrong row lost
    assert recorded_measurement(p) == pytest.approx(6.10)
    assert "out/rmsnorm_llama_config.csv" in text and "/root" not in text


def test_keep_faster_rule(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    winners = tmp_path / "winners"
    out = _run_dir(tmp_path, [(2, 8, 0.0061, True)])
    specialize(STEM, out_root=out, winners_dir=winners)
    slower = _run_dir(tmp_path, [(2, 8, 0.0070, True)])
    with pytest.raises(KeptExisting, match="slower"):
        specialize(STEM, out_root=slower, winners_dir=winners)
    tie = _run_dir(tmp_path, [(2, 8, 0.006101, True)])  # equal at the stored two decimals
    with pytest.raises(KeptExisting, match="tie"):
        specialize(STEM, out_root=tie, winners_dir=winners)
    assert recorded_measurement(winners / f"{STEM}.py") == pytest.approx(6.10)
    faster = _run_dir(tmp_path, [(0, 4, 0.0055, True)])
    specialize(STEM, out_root=faster, winners_dir=winners)
    assert recorded_measurement(winners / f"{STEM}.py") == pytest.approx(5.50)
    forced = _run_dir(tmp_path, [(2, 8, 0.0090, True)])
    specialize(STEM, out_root=forced, winners_dir=winners, force=True)
    assert recorded_measurement(winners / f"{STEM}.py") == pytest.approx(9.00)


def test_measured_only(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    out = _run_dir(tmp_path, [(2, 8, 0.0061, False), (0, 4, 0.0100, "")])
    with pytest.raises(SpecializeError, match="no benched row passed"):
        specialize(STEM, out_root=out, winners_dir=tmp_path / "winners")


def test_decide_write_unmeasured_artifact_is_superseded(tmp_path):
    p = tmp_path / "w.py"
    assert decide_write(p, 5.0, False) is None  # absent
    p.write_text('"""hand written"""\n')
    assert decide_write(p, 50.0, False) is None  # no measurement recorded


def test_source_commit_off_git_comes_from_the_environment(tmp_path, monkeypatch):
    """A checkout copied without its history (as to a GPU host) records the
    commit it was copied from, when the caller names it."""
    from enzyme_b200 import specialize

    monkeypatch.setenv("AXON_SOURCE_COMMIT", "abc1234")
    assert specialize.source_commit(tmp_path) == "abc1234"
    monkeypatch.delenv("AXON_SOURCE_COMMIT")
    assert specialize.source_commit(tmp_path) == "unknown"
