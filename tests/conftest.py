"""Shared pytest setup: the `gpu` marker and spec/fixture helpers."""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"
KERNELS = ROOT / "kernels"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_spec(name: str):
    """Load kernels/<name>/ the way the CLI does (by path, as a package)."""
    from enzyme_b200.specs import load_spec as _load

    return _load(KERNELS / name)


def golden_cases():
    return sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load_golden(case: str):
    """(spec_name, dims dict, inputs (numpy, native dtypes), baseline outputs, record)."""
    import ml_dtypes

    d = np.load(GOLDEN / f"{case}.npz")
    spec_name = case.rsplit("_", 1)[0]
    dims = {str(k): int(v) for k, v in zip(d["dim_names"], d["dims"])}
    inputs = []
    for i, dt in enumerate(d["dtypes"]):
        a = d[f"in_{i}"]
        inputs.append(a.view(ml_dtypes.bfloat16) if str(dt) == "bfloat16" else a)
    outs = []
    i = 0
    while f"baseline_{i}" in d.files:
        outs.append(d[f"baseline_{i}"])
        i += 1
    return spec_name, dims, inputs, outs, d


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run with -m 'not gpu' on CPU hosts)")
    return torch.device("cuda:0")
