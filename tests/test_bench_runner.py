"""Host behaviour of the CUDA bench runner, with the device worker stubbed.

Mirrors the contract Axon's tests/test_bench_resume.py pins for its NEFF
pipeline: the column layout, one terminal row per key, publication only on
exact coverage, candidate filtering, failures as rows, interruption and
resume, torn-tail truncation and a damaged store. No GPU is touched: the
device pool is an in-process thread pool and `bench_fn` is a stub.
"""

from __future__ import annotations

import csv
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from conftest import KERNELS, load_spec
from enzyme_b200 import bench_runner as br
from enzyme_b200 import catalogue
from enzyme_b200.kernel_spec import SEED
from enzyme_b200.paths import run_paths
from enzyme_b200.specs import safe_name

DIMS = {"m": 8, "n": 256}


def _setup(tmp_path, name="rmsnorm"):
    spec = load_spec(name)
    paths = run_paths(spec, str(tmp_path / f"out/{name}_t"))
    mods = catalogue.emit_variant_modules(spec, DIMS, 2, paths)
    return spec, paths, mods


def _ref_outputs(spec):
    ins = spec.make_inputs(**DIMS, rng=np.random.default_rng(SEED))
    return br.compute_ref_outputs(spec, ins)[0]


def _good_stub(spec):
    refs = _ref_outputs(spec)

    def stub(args):
        return br.BenchStats.from_times([1.0, 2.0, 3.0], refs)

    return stub


def _run(spec, paths, module, stub, **kw):
    return br.run_cuda_bench(spec, DIMS, hw_variant=0, tile_variant=0, module_path=str(module),
                             function_name=safe_name(spec.name), spec_path=str(KERNELS / spec.name), warmup=1,
                             bench=3, paths=paths, rtol=1e-2, atol=1e-2, pools=[ThreadPoolExecutor(1)],
                             bench_fn=stub, **kw)


def _rows(path):
    with open(path, newline="") as f:
        return list(csv.DictReader(f))


def test_column_layout_and_key_columns():
    spec = load_spec("matmul")
    cols = br.result_columns(spec)
    assert cols[:3] == ["m", "n", "k"]
    assert cols[3:7] == br.KEY_PREFIX_COLS
    assert cols[7:10] == ["TILES_M", "TILES_N", "TILES_K"]
    assert cols[-len(br.EXTRA_COLS):] == br.EXTRA_COLS
    assert br.key_columns(spec) == [*br.KEY_PREFIX_COLS, "TILES_M", "TILES_N", "TILES_K"]


def test_missing_store_reads_as_empty(tmp_path):
    spec = load_spec("rmsnorm")
    assert br.read_result_keys(spec, tmp_path / "nope.csv") == set()


def test_full_case_publishes_one_row_per_key(tmp_path):
    spec, paths, mods = _setup(tmp_path)
    expected = _run(spec, paths, mods[0], _good_stub(spec))
    br.publish_results(spec, paths, expected)
    rows = _rows(paths.csv)
    assert len(rows) == len(expected) > 0
    assert all(r["correct"] == "True" for r in rows)
    assert all(r["median_ms"] == "2.0" for r in rows)
    assert all(r["unit"] == "GB/s" and float(r["achieved"]) > 0 for r in rows)


def test_publish_is_noop_without_expected_keys(tmp_path):
    spec, paths, _ = _setup(tmp_path)
    br.publish_results(spec, paths, set())
    assert not paths.csv.exists()


def test_candidate_filter_prunes_illegal_keys(tmp_path):
    spec, paths, mods = _setup(tmp_path)
    seen = []
    stub0 = _good_stub(spec)

    def stub(args):
        seen.append(args[2])
        return stub0(args)

    _run(spec, paths, mods[0], stub)
    # TILES_IN_BLOCK_M must be 1 for row kernels; n=256 bf16 admits N in {1}
    assert seen and all(tv[0] == 1 for tv in seen)
    assert len(seen) <= 8


def test_candidate_filter_can_be_disabled(tmp_path):
    spec, paths, mods = _setup(tmp_path)
    n = []
    stub0 = _good_stub(spec)

    def stub(args):
        n.append(1)
        return stub0(args)

    _run(spec, paths, mods[0], stub, candidate_filter=False)
    assert len(n) == len(spec.tile_options) ** len(spec.tile_args)


def test_wrong_outputs_are_marked_incorrect(tmp_path):
    spec, paths, mods = _setup(tmp_path)
    refs = _ref_outputs(spec)

    def stub(args):
        return br.BenchStats.from_times([1.0], tuple(r + 1.0 for r in refs))

    expected = _run(spec, paths, mods[0], stub)
    br.publish_results(spec, paths, expected)
    rows = _rows(paths.csv)
    assert all(r["correct"] == "False" and float(r["max_abs_err"]) >= 1.0 for r in rows)


def test_bench_failure_writes_exactly_one_terminal_row(tmp_path):
    spec, paths, mods = _setup(tmp_path)

    def stub(args):
        raise RuntimeError("launch failed: boom")

    expected = _run(spec, paths, mods[0], stub)
    rows = _rows(paths.results)
    assert len(rows) == len(expected)
    assert all(r["error"].startswith("RuntimeError: launch failed") and r["median_ms"] == "" for r in rows)


def test_interruption_keeps_rows_and_resume_runs_only_the_rest(tmp_path, monkeypatch):
    spec, paths, mods = _setup(tmp_path)
    stub = _good_stub(spec)
    real = br.append_result_row
    count = {"n": 0}

    def flaky(path, cols, row):
        if count["n"] == 1:
            raise KeyboardInterrupt
        count["n"] += 1
        real(path, cols, row)

    # the first filter-selected key set has one key for this case; use the
    # unfiltered sweep so there are several keys to interrupt
    monkeypatch.setattr(br, "append_result_row", flaky)
    with pytest.raises(KeyboardInterrupt):
        _run(spec, paths, mods[0], stub, candidate_filter=False)
    assert len(_rows(paths.results)) == 1
    monkeypatch.setattr(br, "append_result_row", real)
    ran = []

    def counting(args):
        ran.append(args[2])
        return stub(args)

    expected = _run(spec, paths, mods[0], counting, candidate_filter=False)
    assert len(ran) == len(expected) - 1
    br.publish_results(spec, paths, expected)
    assert len(_rows(paths.csv)) == len(expected)


def test_torn_final_record_is_truncated(tmp_path):
    spec, paths, mods = _setup(tmp_path)
    expected = _run(spec, paths, mods[0], _good_stub(spec), candidate_filter=False)
    text = paths.results.read_text()
    lines = text.splitlines(keepends=True)
    paths.results.write_text("".join(lines[:-1]) + lines[-1][:10])  # cut the last record mid-line
    keys = br.read_result_keys(spec, paths.results)
    assert len(keys) == len(expected) - 1
    assert paths.results.read_text().endswith("\n")
    # resume fills the gap and publication then succeeds
    expected = _run(spec, paths, mods[0], _good_stub(spec), candidate_filter=False)
    br.publish_results(spec, paths, expected)


@pytest.mark.parametrize("damage,message", [("header", "column drift"), ("fields", "malformed record"),
                                            ("dup", "duplicate key")])
def test_damaged_store_stops_publication(tmp_path, damage, message):
    spec, paths, mods = _setup(tmp_path)
    expected = _run(spec, paths, mods[0], _good_stub(spec))
    lines = paths.results.read_text().splitlines(keepends=True)
    if damage == "header":
        lines[0] = lines[0].replace("median_ms", "p50_ms")
    elif damage == "fields":
        lines.append("1,2,3\n")
    else:
        lines.append(lines[-1])
    paths.results.write_text("".join(lines))
    with pytest.raises(AssertionError, match=message):
        br.publish_results(spec, paths, expected)


def test_incomplete_coverage_stops_publication(tmp_path):
    spec, paths, mods = _setup(tmp_path)
    expected = _run(spec, paths, mods[0], _good_stub(spec))
    with pytest.raises(AssertionError, match="missing"):
        br.publish_results(spec, paths, expected | {("1", "cuda", "9", "9", "1", "1")})


def test_stream_bench_spreads_over_pools_and_yields_each_task_once():
    import threading

    used = set()

    def stub(args):
        used.add(threading.current_thread().name)
        return br.BenchStats.from_times([float(args)])

    pools = [ThreadPoolExecutor(1, thread_name_prefix=f"gpu{i}") for i in range(3)]
    got = dict(br.stream_bench([((i,), i + 1) for i in range(9)], pools=pools, bench_fn=stub))
    assert sorted(got) == [(i,) for i in range(9)]
    assert {k: v.median_ms for k, v in got.items()} == {(i,): float(i + 1) for i in range(9)}
    assert len(used) >= 2


def test_baseline_timing_writes_csv(tmp_path):
    spec = load_spec("rmsnorm")
    paths = run_paths(spec, str(tmp_path / "out/rmsnorm_t"))
    out = br.run_baseline(spec, {"m": 16, "n": 128}, warmup=1, bench=2, paths=paths)
    rows = _rows(out)
    assert rows[0]["ref"] == "torch_ref" and int(rows[0]["cores"]) >= 1 and float(rows[0]["median_ms"]) > 0


@pytest.mark.parametrize("name,dims", [("qkv_cte", {"m": 578, "n": 264, "k": 1408}),
                                       ("softmax_mm", {"m": 1024, "n": 1024, "k": 1024}),
                                       ("attention_nkilib", {"s": 1024, "d": 128})])
def test_neighbour_specs_emit_every_variant(tmp_path, name, dims):
    """The GEMM-backed neighbour specs emit one loadable module per catalogue
    variant, each with a manifest whose feasible tile key maps to a tune."""
    import importlib.util

    spec = load_spec(name)
    paths = run_paths(spec, str(tmp_path / f"out/{name}_t"))
    mods = catalogue.emit_variant_modules(spec, dims, 2, paths)
    assert len(mods) == len(catalogue.variants(name))
    for var, mod in zip(catalogue.variants(name), mods):
        m = importlib.util.module_from_spec(importlib.util.spec_from_file_location(f"_m_{name}_{var.hw_variant}", mod))
        m.__spec__.loader.exec_module(m)
        assert callable(getattr(m, safe_name(name)))
        cons = catalogue.constraints(name, var.hw_variant, dims, 2, spec.tile_args)
        tiles = {c.tile_arg: (c.allowed[-1] if c.allowed else 1) for c in cons}
        tune = catalogue.tune_for(name, var.hw_variant, tiles)
        assert isinstance(tune, dict) and tune.get("variant", 0) in (0, 1, 2, 3)


# ---- workers that raise or die -----------------------------------------------------

def _raise_axon_error(args):
    """A device worker whose launch the library refused (an infeasible tile)."""
    from enzyme_b200 import _native as N

    raise N.AxonError(N.AXON_E_SHAPE, f"tile {args} does not fit")


def _die_on_key(args):
    """A device worker that dies outright on key 'die'; others succeed."""
    import os

    if args == "die":
        os._exit(3)
    return br.BenchStats.from_times([1.0])


def test_axon_error_survives_the_worker_boundary():
    import pickle

    from enzyme_b200 import _native as N

    e = pickle.loads(pickle.dumps(N.AxonError(N.AXON_E_SHAPE, "rows too long")))
    assert e.code == N.AXON_E_SHAPE and "rows too long" in str(e)


def test_refused_launch_in_a_process_worker_is_an_error_row():
    import multiprocessing
    from concurrent.futures import ProcessPoolExecutor

    pool = ProcessPoolExecutor(1, mp_context=multiprocessing.get_context("spawn"))
    out = list(br.stream_bench([(("k1",), "a"), (("k2",), "b")], pools=[pool], bench_fn=_raise_axon_error))
    assert [k for k, _ in out] == [("k1",), ("k2",)]
    assert all(isinstance(r, br.BenchError) and "AXON_E_SHAPE" in r.message for _, r in out)


def test_a_worker_that_dies_costs_only_its_key():
    import multiprocessing
    from concurrent.futures import ProcessPoolExecutor

    ctx = multiprocessing.get_context("spawn")
    tasks = [(("k1",), "ok"), (("k2",), "die"), (("k3",), "ok"), (("k4",), "ok")]
    out = dict(br.stream_bench(tasks, pools=[ProcessPoolExecutor(1, mp_context=ctx)], bench_fn=_die_on_key,
                               respawn=lambda pool: ProcessPoolExecutor(1, mp_context=ctx)))
    assert isinstance(out[("k2",)], br.BenchError) and "died" in out[("k2",)].message
    assert all(isinstance(out[k], br.BenchStats) for k in (("k1",), ("k3",), ("k4",)))


def test_reference_outputs_are_float64():
    spec = load_spec("cumsum")
    (ref,) = br.compute_ref_outputs(spec, spec.make_inputs(m=4, n=32768, rng=np.random.default_rng(SEED)))[0]
    assert ref.dtype == np.float64
