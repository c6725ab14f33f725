"""`axon kernels/<name> --sizes ...` for the CUDA backend.

    python -m enzyme_b200 kernels/rmsnorm --sizes 1024 4096 --rtol 1e-2 --atol 1e-2 --out out/rmsnorm_h4096.csv

Same surface as Axon's CLI (src/axon/cli.py:825-1131) minus the synthesis
flags: the spec is loaded by path (exit 2 if it has no SPEC), `--sizes` binds
positionally to the spec's dim_vars (exit 2 on a count mismatch), `--rtol`
and `--atol` together mark a head-to-head case whose id is the `--out` stem
minus `<kernel>_` (exit 2 if the stem has another form), `--mode`
variants/baseline/both, `--phase` emit/bench/all, `--pick-by`, the candidate
filter and budget, `--warmup 20 --bench 100`. `--gpus N` benches on N local
GPUs in parallel (one pinned worker process per GPU); `--lnc 2` is accepted
as its alias. `--target` is accepted for compatibility; only sm_100a exists.
"""

from __future__ import annotations

import argparse
import inspect
import math
import sys
from pathlib import Path

import numpy as np

from . import catalogue
from .bench_runner import (ResultKey, clear_stale_artifacts, publish_results, run_baseline, run_cuda_bench,
                           visible_gpu_ids)
from .kernel_spec import KernelSpec
from .paths import RunPaths, run_paths
from .specs import SpecLoadError, load_spec, safe_name
from .winner import export_winner, pick_winner

DTYPE_CHOICES = ("bfloat16", "float16", "float32")
DEFAULT_RTOL = 2e-2
DEFAULT_ATOL = 2e-2


def _nonneg(v: str) -> int:
    x = int(v)
    if x < 0:
        raise argparse.ArgumentTypeError("must not be negative")
    return x


def _pos(v: str) -> int:
    x = int(v)
    if x <= 0:
        raise argparse.ArgumentTypeError("must be greater than zero")
    return x


def _pos_float(v: str) -> float:
    x = float(v)
    if not math.isfinite(x) or x <= 0:
        raise argparse.ArgumentTypeError("must be a finite value greater than zero")
    return x


def spec_default_dtype(spec: KernelSpec) -> str:
    p = inspect.signature(spec.make_inputs).parameters.get("dtype")
    if p is None or p.default is inspect.Parameter.empty:
        return "float32"
    return np.dtype(p.default).name


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="axon", description="Benchmark a kernel spec on the B200 CUDA backend.")
    ap.add_argument("kernel", help="path to a kernel-spec package dir or .py file with a top-level SPEC")
    ap.add_argument("--sizes", type=int, nargs="+", required=True, metavar="N",
                    help="dimension sizes bound positionally to the spec's dim_vars")
    ap.add_argument("--target", default="sm_100a", help="accepted for compatibility; only sm_100a is built")
    ap.add_argument("--dtype", choices=DTYPE_CHOICES, default=None, help="override make_inputs' dtype")
    ap.add_argument("--out", default=None, metavar="PATH", help="run stem (out/<stem>.csv, out/<stem>/)")
    ap.add_argument("--warmup", type=_nonneg, default=20)
    ap.add_argument("--bench", type=_pos, default=100)
    ap.add_argument("--mode", choices=("variants", "baseline", "both"), default="variants")
    ap.add_argument("--pick-by", choices=("median", "mean", "min"), default="median")
    ap.add_argument("--phase", choices=("emit", "bench", "all"), default="all")
    ap.add_argument("--gpus", type=_pos, default=1, help="local GPUs to bench on in parallel")
    ap.add_argument("--lnc", type=int, choices=(1, 2), default=None, help="alias of --gpus (Axon compatibility)")
    ap.add_argument("--candidate-filter", action=argparse.BooleanOptionalAction, default=True)
    ap.add_argument("--candidate-budget", type=_nonneg, default=8)
    ap.add_argument("--rtol", type=_pos_float, default=None)
    ap.add_argument("--atol", type=_pos_float, default=None)
    return ap


def _bench_modules(spec: KernelSpec, spec_path: str, dims: dict, paths: RunPaths, *, warmup, bench, dtype, rtol,
                   atol, candidate_filter, candidate_budget, device_ids) -> set[ResultKey]:
    fn = safe_name(spec.name)
    modules = sorted(paths.run_dir.glob(f"{fn}__v*_t*.py"))
    if not modules:
        print(f"--phase bench: no variant modules under {paths.run_dir}; run --phase emit first", file=sys.stderr)
        sys.exit(2)
    paths.csv.unlink(missing_ok=True)
    expected: set[ResultKey] = set()
    for mp in modules:
        tail = mp.stem.rsplit("__v", 1)[1]
        i_s, j_s = tail.split("_t", 1)
        expected |= run_cuda_bench(
            spec, dims, hw_variant=int(i_s), tile_variant=int(j_s.split("_")[0]), module_path=str(mp),
            function_name=fn, spec_path=spec_path, warmup=warmup, bench=bench, paths=paths, dtype=dtype,
            rtol=rtol, atol=atol, candidate_filter=candidate_filter, candidate_budget=candidate_budget,
            device_ids=device_ids)
    return expected


def run(args: argparse.Namespace) -> int:
    try:
        spec = load_spec(args.kernel)
    except SpecLoadError as e:
        print(str(e), file=sys.stderr)
        sys.exit(2)
    if len(args.sizes) != len(spec.dim_vars):
        print(f"{spec.name}: --sizes expects {len(spec.dim_vars)} values for dims {list(spec.dim_vars)} in "
              f"order, got {len(args.sizes)}", file=sys.stderr)
        sys.exit(2)
    dims = dict(zip(spec.dim_vars, args.sizes))
    paths = run_paths(spec, args.out)
    dtype = np.dtype(args.dtype) if args.dtype else None
    rtol = args.rtol if args.rtol is not None else DEFAULT_RTOL
    atol = args.atol if args.atol is not None else DEFAULT_ATOL
    gpus = args.lnc if args.lnc is not None else args.gpus
    spec_path = str(Path(args.kernel).expanduser().resolve())

    case_id = case_dtype = None
    if args.rtol is not None and args.atol is not None:
        prefix = f"{spec.name}_"
        if not paths.csv.stem.startswith(prefix):
            print(f"{spec.name}: head-to-head run needs an --out stem of the form '{spec.name}_<case_id>.csv', "
                  f"got {paths.csv.stem!r}", file=sys.stderr)
            sys.exit(2)
        case_id = paths.csv.stem[len(prefix):]
        case_dtype = args.dtype or spec_default_dtype(spec)

    if args.mode in ("variants", "both"):
        if spec.name not in catalogue.ALL_SPECS:
            print(f"{spec.name}: no CUDA variants in the catalogue (specs: {', '.join(catalogue.ALL_SPECS)})",
                  file=sys.stderr)
            return 2
        itemsize = np.dtype(dtype or spec_default_dtype(spec)).itemsize
        if args.phase in ("emit", "all"):
            for p in catalogue.emit_variant_modules(spec, dims, itemsize, paths):
                print(f"  +-- wrote {p}")
        if args.phase in ("bench", "all"):
            ids = visible_gpu_ids()[:gpus] or list(range(gpus))
            if len(ids) < gpus:
                print(f"--gpus {gpus}: only {len(ids)} GPU(s) visible", file=sys.stderr)
                return 2
            expected = _bench_modules(spec, spec_path, dims, paths, warmup=args.warmup, bench=args.bench,
                                      dtype=dtype, rtol=rtol, atol=atol, candidate_filter=args.candidate_filter,
                                      candidate_budget=args.candidate_budget, device_ids=ids)
            publish_results(spec, paths, expected)
            clear_stale_artifacts(paths)
            winner = pick_winner(paths.csv, spec, args.pick_by, rtol=rtol, atol=atol)
            if winner is None:
                print(f"{spec.name}: no timed variants in {paths.csv}", file=sys.stderr)
                return 1
            print(f"\nwinner: v{winner.hw_variant}_t{winner.tile_variant} tiles={winner.tile_values} "
                  f"median {winner.median_ms:.4f} ms")
            if case_id is not None:
                export_winner(spec, winner, case_id=case_id, kernel_path=spec_path, paths=paths, dtype=case_dtype,
                              rtol=rtol, atol=atol)
    if args.mode in ("baseline", "both"):
        if spec.baseline_op is None:
            print(f"kernel '{spec.name}' has no baseline_op set", file=sys.stderr)
            return 2
        paths.baseline_csv.unlink(missing_ok=True)
        run_baseline(spec, dims, warmup=max(1, min(args.warmup, 3)), bench=max(1, min(args.bench, 10)),
                     paths=paths, dtype=dtype)
    return 0


def main(argv: list[str] | None = None) -> None:
    sys.exit(run(build_parser().parse_args(argv)))


if __name__ == "__main__":
    main()
