"""Winner selection and head-to-head export (Axon src/axon/winner.py:47-166).

The winner is the fastest timed row that is not verified wrong: a
fast-but-wrong variant loses to a slower correct one; only when every timed
row is verified wrong does selection fail. An empty `correct` cell means
unverified, not wrong. The export copies the winning variant module to
`out/winners/<spec>_<case>.py` and writes the per-case harness beside it.
"""

from __future__ import annotations

import os

import shutil
from dataclasses import dataclass
from pathlib import Path
from typing import Literal

import pandas as pd

from .bench_runner import tile_cols
from .case_gen import generate_case_module
from .kernel_spec import KernelSpec
from .paths import RunPaths
from .specs import safe_name

PickBy = Literal["median", "mean", "min"]


@dataclass(frozen=True)
class WinnerRow:
    hw_variant: int
    tile_variant: int
    mean_ms: float | None
    median_ms: float | None
    min_ms: float | None
    sizes: tuple[int, ...]
    tile_values: tuple[int, ...]
    lnc: int = 1
    sharding: str = "cuda"


def _verified_wrong(v) -> bool:
    if pd.isna(v):
        return False
    if isinstance(v, str):
        return v.strip().lower() in ("false", "0")
    return not bool(v)


def _tag(row) -> str:
    return f"v{int(row['hw_variant'])}_t{int(row['tile_variant'])}"


def pick_winner(csv_path: Path, spec: KernelSpec, pick_by: PickBy, *, rtol: float, atol: float) -> WinnerRow | None:
    if not csv_path.is_file():
        return None
    df = pd.read_csv(csv_path)
    col = f"{pick_by}_ms"
    if col not in df.columns:
        return None
    timed = df[df[col].notna()].copy()
    if timed.empty:
        return None
    ranked = timed.sort_values(col, kind="stable")
    wrong = ranked["correct"].map(_verified_wrong).astype(bool)
    keep = ranked[~wrong]
    if keep.empty:
        worst = ranked.iloc[0]
        raise AssertionError(f"{spec.name} winner {_tag(worst)} failed on-device correctness: "
                             f"max_abs_err={worst['max_abs_err']} exceeds rtol={rtol} atol={atol}")
    row = keep.iloc[0]
    skipped = list(wrong).index(False)
    if skipped:
        print(f"[info] {spec.name} skipped {skipped} faster but incorrect variant(s); winner is {_tag(row)}")
    if pd.isna(row["correct"]):
        print(f"[warn] {spec.name} winner {_tag(row)} correctness unverified; shipping unchecked")
    return WinnerRow(
        hw_variant=int(row["hw_variant"]), tile_variant=int(row["tile_variant"]), mean_ms=float(row["mean_ms"]),
        median_ms=float(row["median_ms"]), min_ms=float(row["min_ms"]),
        sizes=tuple(int(row[c]) for c in spec.dim_vars),
        tile_values=tuple(int(row[c]) for c in tile_cols(spec.tile_args)),
        lnc=int(row["lnc"]) if "lnc" in row else 1,
        sharding=str(row["sharding"]) if "sharding" in row else "cuda")


def provenance(spec: KernelSpec, winner: WinnerRow, case_id: str) -> str:
    """A literal WINNER_PROVENANCE record appended to the exported winner: the
    device it was measured on, the source commit, the timings and the key
    (what Axon's specialised winners record in their docstrings)."""
    import subprocess

    device = "unknown"
    try:
        import torch

        if torch.cuda.is_available():
            device = torch.cuda.get_device_name(0)
    except Exception:
        pass
    try:
        commit = subprocess.run(["git", "rev-parse", "--short", "HEAD"], capture_output=True, text=True,
                                cwd=Path(__file__).resolve().parent, timeout=10).stdout.strip()
    except Exception:
        commit = ""
    # a checkout copied without its history (e.g. to a GPU host) names it here
    commit = commit or os.environ.get("AXON_SOURCE_COMMIT", "") or "unknown"
    rec = {"spec": spec.name, "case": case_id, "device": device, "commit": commit,
           "sizes": dict(zip(spec.dim_vars, winner.sizes)),
           "tiles": dict(zip(spec.tile_args, winner.tile_values)), "hw_variant": winner.hw_variant,
           "tile_variant": winner.tile_variant, "median_ms": winner.median_ms, "mean_ms": winner.mean_ms,
           "min_ms": winner.min_ms}
    return f"\n\nWINNER_PROVENANCE = {rec!r}\n"


def export_winner(spec: KernelSpec, winner: WinnerRow, *, case_id: str, kernel_path: Path | str, paths: RunPaths,
                  dtype: str, rtol: float, atol: float) -> None:
    entry = f"{spec.name}_{case_id}"
    print(f"\n=== export {entry} ===\n  winner: hw_variant={winner.hw_variant}, tile_variant={winner.tile_variant}, "
          f"median_ms={winner.median_ms}, mean_ms={winner.mean_ms}, min_ms={winner.min_ms}")
    fn = safe_name(spec.name)
    src = paths.variant_module(fn, winner.hw_variant, winner.tile_variant)
    if not src.is_file():
        raise FileNotFoundError(f"winning variant module not found at {src}; re-run the bench")
    dst = paths.winner_kernel(entry)
    dst.parent.mkdir(parents=True, exist_ok=True)
    shutil.copyfile(src, dst)
    with dst.open("a") as f:
        f.write(provenance(spec, winner, case_id))
    print(f"  wrote {dst}")
    shape = dict(zip(spec.dim_vars, winner.sizes))
    tiles = {a: int(v) for a, v in zip(spec.tile_args, winner.tile_values)}
    generate_case_module(spec, kernel_path, dtype, paths.winner_case(entry), name=entry, entry_point=fn,
                         shape_args={**shape, **tiles}, rtol=rtol, atol=atol)
    print(f"  wrote {paths.winner_case(entry)}")
