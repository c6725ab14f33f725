"""Benchmark every tile key of a variant module on the GPU and keep a durable
per-key CSV row store -- the CUDA replacement of Axon's compile + bench leg.

Behavioural contract kept from Axon (src/axon/bench_runner.py):
* seeded inputs from the spec's `make_inputs(..., rng=default_rng(SEED))`
  (:607-611), the tile-option product filtered by the module's manifest and
  a diverse budgeted selection (:613-630);
* one terminal row per key, appended with fsync (:437-458); a torn final
  record is truncated on resume and finished keys are skipped (:400-434,
  :671-679); the published CSV is replaced atomically only on exact key
  coverage (:461-479);
* correctness: every output against `baseline_op` (evaluated here in float64
  rather than on fp32 inputs: the oracle of the checks), `np.allclose(rtol,
  atol)` plus `max_abs_err` (:562-573, :703-717); a failing launch becomes an
  `error` row, never an exception in the CLI (:534-554), and a worker process
  that dies costs only its key's row (a fresh worker takes the rest).

What differs: there is no compile stage (the kernels are built ahead of time
into libaxon_b200.so), and a "device worker" is a process pinned to one GPU
with CUDA_VISIBLE_DEVICES. Timing is CUDA events around a CUDA-graph replay
of one launch, with L2 flushed (a 256 MiB memset) before every timed
iteration. Columns appended after Axon's: achieved throughput, its unit, the
roofline fraction, the GPU count and the CPU reference time of the case.
"""

from __future__ import annotations

import csv
import importlib.util
import inspect
import io
import multiprocessing
import os
import shutil
import sys
import time
from collections import Counter, deque
from collections.abc import Callable, Iterator, Sequence
from concurrent.futures import FIRST_COMPLETED, BrokenExecutor, Executor, ProcessPoolExecutor, ThreadPoolExecutor, wait
from dataclasses import asdict, dataclass
from itertools import product
from pathlib import Path
from statistics import mean, median, pstdev
from typing import Any

import numpy as np

from . import roofline
from .candidate_filter import read_manifest, rejection_reason, select_diverse
from .kernel_spec import SEED, KernelSpec
from .paths import RunPaths

__all__ = ["run_cuda_bench", "run_baseline", "BenchStats", "BenchError", "publish_results", "result_columns"]


@dataclass(frozen=True)
class BenchStats:
    mean_ms: float | None
    median_ms: float | None
    min_ms: float | None
    max_ms: float | None
    std_dev_ms: float | None
    outputs: tuple[np.ndarray, ...] | None = None

    @classmethod
    def from_times(cls, times_ms: Sequence[float], outputs=None) -> BenchStats:
        if not times_ms:
            return cls(None, None, None, None, None, outputs)
        return cls(mean(times_ms), median(times_ms), min(times_ms), max(times_ms), pstdev(times_ms), outputs)


@dataclass(frozen=True)
class BenchError:
    message: str

    @classmethod
    def from_exception(cls, e: BaseException) -> BenchError:
        return cls(f"{type(e).__name__}: {e}")


BenchResult = BenchStats | BenchError


# ---- row store ------------------------------------------------------------------

def tile_cols(tile_args: Sequence[str]) -> list[str]:
    return [f"TILES_{a.upper().replace('TILES_IN_BLOCK_', '').replace('TILES_', '')}" for a in tile_args]


STATS_COLS = ["mean_ms", "median_ms", "min_ms", "max_ms", "std_dev_ms"]
KEY_PREFIX_COLS = ["lnc", "sharding", "hw_variant", "tile_variant"]
EXTRA_COLS = ["achieved", "unit", "roofline_frac", "n_gpus", "cpu_ref_ms"]


def result_columns(spec: KernelSpec) -> list[str]:
    return [*spec.dim_vars, *KEY_PREFIX_COLS, *tile_cols(spec.tile_args), *STATS_COLS, "correct", "max_abs_err",
            "error", "mode", *EXTRA_COLS]


def key_columns(spec: KernelSpec) -> list[str]:
    return [*KEY_PREFIX_COLS, *tile_cols(spec.tile_args)]


ResultKey = tuple[str, ...]


def read_result_keys(spec: KernelSpec, path: Path) -> set[ResultKey]:
    """Keys of every complete record; a torn last record is cut off first."""
    if not path.is_file() or path.stat().st_size == 0:
        return set()
    with path.open("rb+") as f:
        f.seek(-1, os.SEEK_END)
        if f.read(1) != b"\n":
            f.seek(0)
            f.truncate(f.read().rfind(b"\n") + 1)
    cols = result_columns(spec)
    idx = [cols.index(c) for c in key_columns(spec)]
    keys: set[ResultKey] = set()
    with path.open(newline="") as f:
        reader = csv.reader(f)
        header = next(reader, None)
        if header is None:
            return set()
        if header != cols:
            raise AssertionError(f"column drift on {path}: found {header} != expected {cols}; "
                                 f"delete {path.parent} to start fresh.")
        for lineno, rec in enumerate(reader, start=2):
            if len(rec) != len(cols):
                raise AssertionError(f"malformed record at {path}:{lineno}: {len(rec)} fields, expected {len(cols)}")
            key = tuple(rec[i] for i in idx)
            if key in keys:
                raise AssertionError(f"duplicate key {key} at {path}:{lineno}")
            keys.add(key)
    return keys


def append_result_row(path: Path, columns: Sequence[str], row: dict) -> None:
    """Append one terminal record durably: one physical line, then fsync."""
    path.parent.mkdir(parents=True, exist_ok=True)
    fresh = not path.exists() or path.stat().st_size == 0
    buf = io.StringIO()
    w = csv.writer(buf, lineterminator="\n")
    if fresh:
        w.writerow(columns)
    w.writerow([" ".join(str(row[c]).split()) if row.get(c) is not None else "" for c in columns])
    with path.open("a", newline="") as f:
        f.write(buf.getvalue())
        f.flush()
        os.fsync(f.fileno())


def publish_results(spec: KernelSpec, paths: RunPaths, expected: set[ResultKey]) -> None:
    if not expected:
        return
    have = read_result_keys(spec, paths.results)
    missing = sorted(expected - have)
    extra = sorted(have - expected)
    if missing or extra:
        raise AssertionError(f"{spec.name}: {paths.results} does not cover the run: {len(missing)} missing "
                             f"key(s) {missing[:5]}, {len(extra)} unexpected key(s) {extra[:5]}")
    tmp = paths.csv.with_name(paths.csv.name + ".publish.tmp")
    shutil.copyfile(paths.results, tmp)
    os.replace(tmp, paths.csv)
    print(f"\npublished {len(expected)} row(s) to {paths.csv}")


def clear_stale_artifacts(paths: RunPaths) -> None:
    """Axon reclaims per-key NEFF dirs here; CUDA variants leave none behind,
    so only a stale publish temp file can exist."""
    tmp = paths.csv.with_name(paths.csv.name + ".publish.tmp")
    tmp.unlink(missing_ok=True)


# ---- references -------------------------------------------------------------------

def compute_ref_outputs(spec: KernelSpec, inputs: Sequence) -> tuple[tuple[np.ndarray, ...] | None, float | None]:
    """`baseline_op` evaluated on float64 copies of the inputs, and its wall
    time in ms. Axon evaluates it on fp32 copies (src/axon/bench_runner.py:
    701); the same function in float64 is the oracle the checks here hold
    the kernels to: an fp32 evaluation carries its own rounding (a float32
    running sum over 32768 columns is ~2e-3 off at a 1e-3 case tolerance),
    which would mark a more accurate kernel wrong."""
    if spec.baseline_op is None:
        return None, None
    f64 = [np.asarray(a, dtype=np.float64) for a in inputs]
    t0 = time.perf_counter()
    with np.errstate(over="ignore"):  # exp(-x) of a large gate overflows to inf, as in fp32: silu -> 0
        out = spec.baseline_op(*f64)
    ms = (time.perf_counter() - t0) * 1e3
    arrs = out if isinstance(out, (tuple, list)) else (out,)
    return tuple(np.asarray(a, dtype=np.float64) for a in arrs), ms


def check_outputs(outputs, refs, rtol, atol) -> tuple[bool | None, float | None]:
    if refs is None or outputs is None:
        return None, None
    errs = [float(np.abs(np.asarray(o, np.float64) - r).max()) if r.size else 0.0 for o, r in zip(outputs, refs)]
    ok = all(np.allclose(np.asarray(o, np.float64), r, rtol=rtol, atol=atol) for o, r in zip(outputs, refs))
    return bool(ok), max(errs) if errs else 0.0


# ---- device worker ---------------------------------------------------------------

_WORKER_CACHE: dict[Any, Any] = {}


def load_variant(module_path: str, fn_name: str):
    key = "_axon_b200_variant_" + module_path.replace("/", "_").replace("\\", "_").replace(".", "_")
    mod = sys.modules.get(key)
    if mod is None:
        spec = importlib.util.spec_from_file_location(key, module_path)
        if spec is None or spec.loader is None:
            raise ImportError(f"could not load variant module from {module_path}")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[key] = mod
        spec.loader.exec_module(mod)
    return getattr(mod, fn_name)


def _device_inputs(spec_path: str, dims: dict, dtype: str | None):
    key = (spec_path, tuple(sorted(dims.items())), dtype)
    if key not in _WORKER_CACHE:
        _WORKER_CACHE.clear()
        from .catalogue import to_device
        from .specs import load_spec

        spec = load_spec(spec_path)
        kw = {"dtype": np.dtype(dtype)} if dtype else {}
        inputs = spec.make_inputs(**dims, **kw, rng=np.random.default_rng(SEED))
        _WORKER_CACHE[key] = (spec, [to_device(a, "cuda") for a in inputs])
    return _WORKER_CACHE[key]


def bench_one(args) -> BenchStats:
    """Time one tile key of one variant module on this process's GPU."""
    (module_path, fn_name, tile_values, tile_args, spec_path, dims, dtype, warmup, bench) = args
    import torch

    from . import ops

    spec, dev_inputs = _device_inputs(spec_path, dims, dtype)
    fn = load_variant(module_path, fn_name)
    params = [p for p in inspect.signature(fn).parameters if p not in set(tile_args)]
    names = spec.input_names()
    if sorted(params) != sorted(names):
        raise ValueError(f"variant params {params} do not match spec inputs {names}")
    by_name = dict(zip(names, dev_inputs))
    call_args = [by_name[p] for p in params]
    tiles = dict(zip(tile_args, tile_values))

    outs = fn(*call_args, **tiles)
    torch.cuda.synchronize()
    ops.gemm_status()
    outputs = tuple(o.detach().float().cpu().numpy() for o in outs)

    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(*call_args, **tiles)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g, stream=s):
        fn(*call_args, **tiles)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        g.replay()
    times = []
    for _ in range(bench):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    ops.gemm_status()
    del g, flush
    return BenchStats.from_times(times, outputs)


def _pin_device(index) -> None:
    os.environ["CUDA_VISIBLE_DEVICES"] = str(index)
    import faulthandler

    faulthandler.enable()  # a worker that crashes leaves its Python stack on stderr


def visible_gpu_ids() -> list[int]:
    raw = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    if raw:
        return [int(x) for x in raw.split(",") if x.strip().isdigit()]
    try:
        import torch

        return list(range(torch.cuda.device_count()))
    except Exception:
        return []


def make_device_pools(device_ids: Sequence[int]) -> list[Executor]:
    """One single-worker spawn pool per GPU, pinned before torch initialises CUDA."""
    if os.environ.get("AXON_B200_INPROCESS") == "1":
        return [ThreadPoolExecutor(max_workers=1)]
    ctx = multiprocessing.get_context("spawn")
    pools = []
    for d in device_ids:
        pool = ProcessPoolExecutor(max_workers=1, initializer=_pin_device, initargs=(d,), mp_context=ctx)
        pool._axon_device = d  # which GPU a replacement worker is pinned to
        pools.append(pool)
    return pools


def respawn_pool(pool: Executor) -> Executor:
    """A fresh single-worker pool on the dead pool's GPU."""
    return make_device_pools([getattr(pool, "_axon_device", 0)])[0]


def stream_bench(tasks: Sequence[tuple[tuple, tuple]], *, pools: Sequence[Executor],
                 bench_fn: Callable = bench_one,
                 respawn: Callable[[Executor], Executor] | None = None) -> Iterator[tuple[tuple, BenchResult]]:
    """Fan `(key, bench_args)` tasks out over the device pools; yield one
    terminal result per task as soon as it completes. A worker that dies
    (its pool breaks) costs only the key it was running: that key gets an
    error row and, with `respawn`, its device gets a fresh worker."""
    pools = list(pools)
    idle: deque[Executor] = deque(pools)
    todo = deque(tasks)
    running: dict[Any, tuple[tuple, Executor]] = {}
    try:
        while todo or running:
            while idle and todo:
                key, args = todo.popleft()
                pool = idle.popleft()
                try:
                    fut = pool.submit(bench_fn, args)
                except BrokenExecutor as e:
                    yield key, BenchError.from_exception(e)
                    if respawn is None:
                        continue  # this device is gone; the others carry on
                    pool = respawn(pool)
                    pools.append(pool)
                    idle.append(pool)
                    continue
                running[fut] = (key, pool)
            if not running:
                continue
            done, _ = wait(set(running), return_when=FIRST_COMPLETED)
            for fut in done:
                key, pool = running.pop(fut)
                try:
                    res: BenchResult = fut.result()
                except BrokenExecutor as e:  # the worker process died
                    res = BenchError(f"worker process died: {e}")
                    if respawn is not None:
                        pool.shutdown(wait=False, cancel_futures=True)
                        pool = respawn(pool)
                        pools.append(pool)
                except Exception as e:  # the worker raised
                    res = BenchError.from_exception(e)
                idle.append(pool)
                yield key, res
    finally:
        for pool in pools:
            pool.shutdown(wait=False, cancel_futures=True)


# ---- the per-module sweep ------------------------------------------------------------

def run_cuda_bench(spec: KernelSpec, dim_sizes: dict[str, int], *, hw_variant: int, tile_variant: int,
                   module_path: str, function_name: str, spec_path: str, warmup: int, bench: int,
                   paths: RunPaths, dtype: Any | None = None, rtol: float, atol: float, sharding: str = "cuda",
                   candidate_filter: bool = True, candidate_budget: int = 8, candidate_seed: int = SEED,
                   device_ids: Sequence[int] | None = None, pools: Sequence[Executor] | None = None,
                   bench_fn: Callable = bench_one) -> set[ResultKey]:
    """Bench every selected tile key of one variant module; returns its keys."""
    print(f"\n{'=' * 80}\nCUDA {spec.name.upper()} BENCHMARK (hw_variant={hw_variant}, "
          f"tile_variant={tile_variant}, sharding={sharding})\n{'=' * 80}")
    kw = {"dtype": dtype} if dtype else {}
    inputs = spec.make_inputs(**dim_sizes, **kw, rng=np.random.default_rng(SEED))
    dims_order = spec.dim_vars
    sizes = tuple(dim_sizes[d] for d in dims_order)
    keys = list(product(spec.tile_options, repeat=len(spec.tile_args)))
    if candidate_filter:
        cons = read_manifest(module_path)
        if cons:
            n0 = len(keys)
            legal = [k for k in keys if rejection_reason(spec.tile_args, k, cons) is None]
            keys = select_diverse(legal, budget=candidate_budget, seed=candidate_seed)
            print(f"\ncandidate filter: {n0} source -> {len(legal)} legal -> {len(keys)} selected "
                  f"(budget={candidate_budget or 'unlimited'})")
    tcols = tile_cols(spec.tile_args)
    cols = result_columns(spec)
    kidx = [cols.index(c) for c in key_columns(spec)]
    n_gpus = len(device_ids) if device_ids else 1
    itemsize = max(np.asarray(a).dtype.itemsize for a in inputs)
    kind, amount = roofline.work(spec.name, dim_sizes, itemsize) if spec.name in roofline.KNOWN else (None, None)

    def row(tv, *, stats=None, correct=None, err=None, error=None, cpu_ms=None) -> dict:
        timing = ({k: v for k, v in asdict(stats).items() if k != "outputs"} if stats is not None
                  else dict.fromkeys(STATS_COLS))
        extra = dict.fromkeys(EXTRA_COLS)
        if stats is not None and stats.median_ms and kind is not None:
            fr = roofline.fraction(kind, amount, stats.median_ms / 1e3)
            extra.update(achieved=round(fr["achieved"], 3), unit=fr["unit"], roofline_frac=round(fr["frac"], 4))
        extra.update(n_gpus=n_gpus, cpu_ref_ms=None if cpu_ms is None else round(cpu_ms, 3))
        return {**dict(zip(dims_order, sizes)), "lnc": 1, "sharding": sharding, "hw_variant": hw_variant,
                "tile_variant": tile_variant, **dict(zip(tcols, tv)), **timing, "correct": correct,
                "max_abs_err": err, "error": error, "mode": "device", **extra}

    def key_of(tv) -> ResultKey:
        r = row(tv)
        return tuple(str(r[cols[i]]) for i in kidx)

    expected = {key_of(tv) for tv in keys}
    paths.run_dir.mkdir(parents=True, exist_ok=True)
    done = read_result_keys(spec, paths.results)
    todo = [tv for tv in keys if key_of(tv) not in done]
    if len(todo) != len(keys):
        print(f"\nresuming: {len(keys) - len(todo)}/{len(keys)} key(s) already terminal")
    if not todo:
        return expected
    refs, cpu_ms = compute_ref_outputs(spec, inputs)
    if pools is None:
        ids = list(device_ids) if device_ids else (visible_gpu_ids()[:1] or [0])
        pools = make_device_pools(ids)
    dname = np.dtype(dtype).name if dtype else None
    tasks = [(tv, (module_path, function_name, tv, tuple(spec.tile_args), spec_path, dict(dim_sizes), dname,
                   warmup, bench)) for tv in todo]
    n_failed = n_wrong = 0
    errs: Counter[str] = Counter()
    respawn = respawn_pool if bench_fn is bench_one and os.environ.get("AXON_B200_INPROCESS") != "1" else None
    for tv, res in stream_bench(tasks, pools=pools, bench_fn=bench_fn, respawn=respawn):
        if isinstance(res, BenchError):
            append_result_row(paths.results, cols, row(tv, error=res.message, cpu_ms=cpu_ms))
            errs[res.message.split(":")[0]] += 1
            n_failed += 1
        else:
            ok, err = check_outputs(res.outputs, refs, rtol, atol)
            n_wrong += int(ok is False)
            append_result_row(paths.results, cols, row(tv, stats=res, correct=ok, err=err, cpu_ms=cpu_ms))
    if n_failed:
        print(f"\n[warn] {n_failed}/{len(todo)} key(s) for {spec.name} failed; see `error` in {paths.results}")
        for tag, c in errs.most_common():
            print(f"  {c:4d}  {tag}")
    if n_wrong:
        print(f"\n[warn] {n_wrong}/{len(todo)} runs for {spec.name} failed correctness (rtol={rtol}, atol={atol})")
    print(f"\n{spec.name} rows appended to {paths.results}")
    return expected


# ---- CPU reference timing (Axon's --mode baseline) ----------------------------------

def run_baseline(spec: KernelSpec, dim_sizes: dict[str, int], *, warmup: int, bench: int, paths: RunPaths,
                 dtype: Any | None = None) -> str:
    """Time the spec's reference on the host CPU (all cores): `torch_ref` on
    fp32 torch tensors, or `baseline_op` on fp32 numpy where there is none.
    This is the reference's own CPU path; Axon's `--mode baseline`
    (src/axon/bench_runner.py:828-889) timed baseline_op on a NeuronCore."""
    import torch

    if spec.baseline_op is None and spec.torch_ref is None:
        raise ValueError(f"kernel '{spec.name}' has no baseline_op set")
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    kw = {"dtype": dtype} if dtype else {}
    inputs = spec.make_inputs(**dim_sizes, **kw, rng=np.random.default_rng(SEED))
    f32 = [np.asarray(a, dtype=np.float32) for a in inputs]
    if spec.torch_ref is not None:
        targs = [torch.from_numpy(a.copy()) for a in f32]
        fn, which = (lambda: spec.torch_ref(*targs)), "torch_ref"
    else:
        fn, which = (lambda: spec.baseline_op(*f32)), "baseline_op"
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(bench):
        t0 = time.perf_counter()
        fn()
        times.append((time.perf_counter() - t0) * 1e3)
    st = BenchStats.from_times(times)
    rec = {**{k: v for k, v in asdict(st).items() if k != "outputs"}, **dim_sizes, "ref": which, "cores": threads}
    csv_path = paths.baseline_csv
    csv_path.parent.mkdir(parents=True, exist_ok=True)
    cols = list(rec)
    fresh = not csv_path.exists()
    with csv_path.open("a", newline="") as f:
        w = csv.DictWriter(f, fieldnames=cols)
        if fresh:
            w.writeheader()
        w.writerow(rec)
    print(f"\n{spec.name} CPU baseline ({which}, {threads} threads): median {st.median_ms:.3f} ms -> {csv_path}")
    return str(csv_path)
