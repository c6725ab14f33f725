"""Build `libaxon_b200.so` in-tree for sm_100a (nvcc cross-compiles without a GPU).

    python -m enzyme_b200.build [--clean]
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent / "csrc"


def build(clean: bool = False, jobs: int | None = None) -> Path:
    jobs = jobs or max(1, min(8, os.cpu_count() or 1))
    if clean:
        subprocess.run(["make", "-C", str(CSRC), "clean"], check=True)
    subprocess.run(["make", "-C", str(CSRC), f"-j{jobs}"], check=True)
    from ._native import LIB_PATH

    if not LIB_PATH.is_file():
        raise RuntimeError(f"build finished but {LIB_PATH} is missing")
    return LIB_PATH


if __name__ == "__main__":
    print(build(clean="--clean" in sys.argv[1:]))
