"""Every per-run path, derived from the CSV path (the run "stem").

Same layout as Axon's `RunPaths` (src/axon/paths.py:20-92): `out/<stem>.csv`
is the published per-case CSV, `out/<stem>/` the run dir holding the durable
row store `results.csv` and the per-variant modules `<fn>__v<i>_t<j>.py`,
`out/baseline_<stem>.csv` the CPU-reference timings, and `out/winners/` the
head-to-head exports. There are no NEFF artifact dirs: the kernels are
compiled ahead of time into libaxon_b200.so.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

from .kernel_spec import KernelSpec


def out_dir() -> Path:
    return Path.cwd() / "out"


def fs_safe(tag: str) -> str:
    """Filesystem-safe form of a sharding tag (`shard=k:P+` -> `shard_k_Pplus`)."""
    return tag.replace("=", "_").replace(":", "_").replace("+", "plus").replace("#", "")


@dataclass(frozen=True, slots=True)
class RunPaths:
    csv: Path

    @property
    def run_dir(self) -> Path:
        return self.csv.with_suffix("")

    @property
    def results(self) -> Path:
        return self.run_dir / "results.csv"

    @property
    def baseline_dir(self) -> Path:
        return self.run_dir.parent / ("baseline_" + self.run_dir.name)

    @property
    def baseline_csv(self) -> Path:
        return self.baseline_dir.parent / (self.baseline_dir.name + ".csv")

    @property
    def winners_dir(self) -> Path:
        return self.csv.parent / "winners"

    def variant_module(self, fn_name: str, i: int, j: int) -> Path:
        return self.run_dir / f"{fn_name}__v{i}_t{j}.py"

    def sharded_variant_module(self, fn_name: str, i: int, j: int, plan_tag: str) -> Path:
        return self.run_dir / f"{fn_name}__v{i}_t{j}_{fs_safe(plan_tag)}.py"

    def winner_kernel(self, entry_name: str) -> Path:
        return self.winners_dir / f"{entry_name}.py"

    def winner_case(self, entry_name: str) -> Path:
        return self.winners_dir / f"{entry_name}_case.py"


def run_paths(spec: KernelSpec, out: str | None) -> RunPaths:
    """`--out out/x` and `--out out/x.csv` name the same run; a trailing slash
    names a container dir for the default `nki_<name>.csv`; omitted, the stem
    is `out/nki_<name>` (the default names are Axon's)."""
    default_name = f"nki_{spec.name}.csv"
    if out is None:
        csv = out_dir() / default_name
    elif out.endswith("/"):
        csv = Path(out) / default_name
    else:
        p = Path(out)
        csv = p if p.suffix == ".csv" else p.with_name(p.name + ".csv")
    return RunPaths(csv=csv.resolve())
