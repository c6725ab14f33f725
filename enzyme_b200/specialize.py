"""The `winners/` deliverable: one standalone module per head-to-head case,
with the winning tile key bound as constants.

    python -m enzyme_b200.specialize [STEM ...] [--all] [--force]

Axon's counterpart is tools/specialize_winner.py (README.md:233-280): the
bench leaves `out/<stem>.csv` (every benched key) and `out/<stem>/` (the
variant modules, whose entry points still take the TILES_IN_BLOCK_* knobs);
the deliverable is `winners/<stem>.py`, whose entry point takes only the
spec's tensor inputs. Two rules, as in the reference (:351-373):

* measured only: a case needs a benched row whose on-device check passed;
  the fastest such row wins, and the artifact records its median;
* best wins: an existing artifact is replaced only by a faster measurement
  (compared at the two decimals the artifact stores, so an equal re-run is
  kept as well); `--force` overwrites.

Each artifact records its provenance: the device it was measured on, the
source commit, the shape, the tile key and the run files (relative to the
directory the bench ran in).
"""

from __future__ import annotations

import argparse
import ast
import re
import subprocess
import sys
import time
from pathlib import Path

import pandas as pd

MEASURED_RE = re.compile(r"measured\s*:\s*([0-9]+(?:\.[0-9]+)?) us median")


class SpecializeError(RuntimeError):
    pass


class KeptExisting(RuntimeError):
    """The recorded artifact is at least as fast as this run: not rewritten."""


def recorded_measurement(path: Path) -> float | None:
    """The median (us) an existing artifact records, or None."""
    if not path.is_file():
        return None
    m = MEASURED_RE.search(path.read_text())
    return float(m.group(1)) if m else None


def decide_write(out_path: Path, new_us: float, force: bool) -> str | None:
    """None when the artifact should be written, else why it is kept."""
    if force or not out_path.is_file():
        return None
    old = recorded_measurement(out_path)
    if old is None:
        return None  # no measurement recorded: a measured artifact supersedes it
    new = round(new_us, 2)
    if new < old:
        return None
    return (f"kept existing {old:.2f} us; this run measured {new:.2f} us ({'tie' if new == old else 'slower'}). "
            f"Pass --force to overwrite.")


def device_id() -> str:
    try:
        import torch

        if torch.cuda.is_available():
            p = torch.cuda.get_device_properties(0)
            return (f"{p.name} (compute capability {p.major}.{p.minor}, {p.multi_processor_count} SMs, "
                    f"{p.total_memory // 2**30} GiB), torch CUDA {torch.version.cuda}")
    except Exception:
        pass
    return "unknown device"


def source_commit(repo: Path) -> str:
    """The source commit: git's HEAD, else AXON_SOURCE_COMMIT (a checkout
    copied without its history, e.g. to a GPU host), else "unknown"."""
    import os

    try:
        out = subprocess.run(["git", "rev-parse", "--short", "HEAD"], capture_output=True, text=True, cwd=repo,
                             timeout=10).stdout.strip()
    except Exception:
        out = ""
    return out or os.environ.get("AXON_SOURCE_COMMIT", "") or "unknown"


def _correct(v) -> bool:
    if isinstance(v, str):
        return v.strip().lower() in ("true", "1")
    return bool(v) if not pd.isna(v) else False


def winning_row(csv_path: Path) -> pd.Series:
    """The fastest row whose on-device check passed (measured only)."""
    if not csv_path.is_file():
        raise SpecializeError(f"{csv_path} not found (run the case first)")
    df = pd.read_csv(csv_path)
    ok = df[df["median_ms"].notna() & df["correct"].map(_correct)]
    if ok.empty:
        raise SpecializeError(f"{csv_path}: no benched row passed the correctness check")
    return ok.sort_values("median_ms", kind="stable").iloc[0]


def _entry(module: Path) -> tuple[str, list[str], list[str]]:
    """(function name, data params, tile params) of a variant module."""
    tree = ast.parse(module.read_text())
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and not node.name.startswith("_"):
            return node.name, [a.arg for a in node.args.args], [a.arg for a in node.args.kwonlyargs]
    raise SpecializeError(f"{module}: no entry point")


def _module_consts(module: Path) -> dict:
    out = {}
    for node in ast.parse(module.read_text()).body:
        if isinstance(node, ast.Assign) and len(node.targets) == 1 and isinstance(node.targets[0], ast.Name):
            if node.targets[0].id in ("SPEC_NAME", "HW_VARIANT"):
                out[node.targets[0].id] = ast.literal_eval(node.value)
    return out


def specialize(stem: str, *, out_root: Path, winners_dir: Path, repo: Path | None = None,
               force: bool = False) -> Path:
    """Write winners_dir/<stem>.py from out_root/<stem>.csv and its variant
    modules; raises KeptExisting when the recorded artifact is not slower."""
    csv_path = out_root / f"{stem}.csv"
    run_dir = out_root / stem
    row = winning_row(csv_path)
    hw, tv = int(row["hw_variant"]), int(row["tile_variant"])
    modules = sorted(run_dir.glob(f"*__v{hw}_t{tv}.py"))
    if not modules:
        raise SpecializeError(f"no variant module v{hw}_t{tv} under {run_dir}")
    module = modules[0]
    fn, data, tiles = _entry(module)
    consts = _module_consts(module)
    bindings = {}
    for t in tiles:
        col = "TILES_" + t.removeprefix("TILES_IN_BLOCK_").removeprefix("TILES_")
        if col not in row.index:
            raise SpecializeError(f"{module.name}: tile parameter {t} has no CSV column {col}")
        bindings[t] = int(row[col])
    dims = {c: int(row[c]) for c in row.index[:list(row.index).index("lnc")]}
    measured_us = float(row["median_ms"]) * 1000.0
    out_path = winners_dir / f"{stem}.py"
    skip = decide_write(out_path, measured_us, force)
    if skip:
        raise KeptExisting(skip)
    where = Path.cwd()
    rel = lambda p: str(p.resolve().relative_to(where)) if p.resolve().is_relative_to(where) else p.name  # noqa: E731
    prov = {"case": stem, "spec": consts.get("SPEC_NAME"), "hw_variant": hw, "tile_variant": tv,
            "tiles": bindings, "shape": dims, "median_us": round(measured_us, 2),
            "min_us": round(float(row["min_ms"]) * 1000.0, 2), "device": device_id(),
            "commit": source_commit(repo or Path(__file__).resolve().parents[1])}
    header = (
        f'"""Axon B200 winner for case {stem!r}, specialized to its tile configuration.\n\n'
        f"Generated by enzyme_b200.specialize. Do not edit by hand.\n\n"
        f"A standalone entry point: it takes only the spec's tensor inputs (device\n"
        f"tensors, in the spec's input order); the winning CUDA variant and tile key\n"
        f"are bound as constants, so the file cannot disagree with the run it came from.\n\n"
        f"Provenance\n"
        f"----------\n"
        f"    entry point   : {fn}\n"
        f"    shape         : {', '.join(f'{k}={v}' for k, v in dims.items())}\n"
        f"    variant       : hw_variant {hw}, tile_variant {tv}\n"
        f"    tile config   : {', '.join(f'{k}={v}' for k, v in bindings.items()) or 'n/a'}\n"
        f"    measured      : {measured_us:.2f} us median (on-device, correct; CUDA graph, L2 flushed)\n"
        f"    generated     : {time.strftime('%Y-%m-%d %H:%M:%S %Z')}\n"
        f"    commit        : {prov['commit']}\n"
        f"    measured on   : {prov['device']}\n\n"
        f"Run files (relative to the directory the bench ran in)\n"
        f"-------------------------------------------------------\n"
        f"    run CSV       : {rel(csv_path)}\n"
        f"    variant       : {rel(module)}\n"
        f'"""\n\n'
    )
    params = ", ".join(data)
    body = (
        "from enzyme_b200.catalogue import launch as _launch\n\n"
        f"SPEC_NAME = {consts.get('SPEC_NAME')!r}\n"
        f"HW_VARIANT = {hw}\n"
        f"TILES = {bindings!r}\n\n\n"
        f"def {fn}({params}):\n"
        f"    return _launch(SPEC_NAME, HW_VARIANT, TILES, ({params},))\n\n\n"
        f"WINNER_PROVENANCE = {prov!r}\n"
    )
    winners_dir.mkdir(parents=True, exist_ok=True)
    out_path.write_text(header + body)
    return out_path


def discover(out_root: Path) -> list[str]:
    """Head-to-head stems: those with an exported case harness."""
    return sorted(p.name[:-len("_case.py")] for p in (out_root / "winners").glob("*_case.py"))


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m enzyme_b200.specialize", description=__doc__.splitlines()[0])
    ap.add_argument("stems", nargs="*", help="case stems, e.g. rmsnorm_llama_config")
    ap.add_argument("--all", action="store_true", help="every head-to-head case under out/winners/")
    ap.add_argument("--out", default="out", help="the bench's output directory")
    ap.add_argument("--winners", default="winners", help="the deliverable directory")
    ap.add_argument("--force", action="store_true", help="overwrite even a faster recorded artifact")
    a = ap.parse_args(argv)
    out_root, winners = Path(a.out), Path(a.winners)
    stems = discover(out_root) if a.all else a.stems
    if not stems:
        ap.error("name case stems or pass --all")
    rc = 0
    for stem in stems:
        try:
            p = specialize(stem, out_root=out_root, winners_dir=winners, force=a.force)
            print(f"WROTE {p}")
        except KeptExisting as e:
            print(f"KEEP  {stem}: {e}")
        except SpecializeError as e:
            print(f"FAIL  {stem}: {e}", file=sys.stderr)
            rc = 1
    return rc


if __name__ == "__main__":
    sys.exit(main())
