"""Generate the golden parity fixtures from the reference's own spec refs.

Run where the Axon reference tree is checked out, with `AXON_REF_ROOT`
naming its root (the script falls back to the build container's checkout):

    AXON_REF_ROOT=<reference checkout> python tests/golden/make_golden.py

For each case it imports the reference's `kernels/<name>/refs.py` by path
(those files need only numpy, torch and ml_dtypes), draws the seeded inputs
with the reference `make_inputs(..., rng=default_rng(42))`, and records

* the inputs, bf16 ones as their raw uint16 bit patterns (exact), with the
  dtype name,
* `baseline_op` on fp32 numpy inputs, as Axon's bench does
  (src/axon/bench_runner.py:562-573),
* the largest difference between that and `torch_ref` on fp32 torch inputs,
  as Axon's case harness calls it (src/axon/case_gen.py:190-201), where the
  spec has one (the two references agree to fp32 rounding).

The fixtures are committed; tests and the GPU box never read the reference.
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SEED = 42  # src/axon/kernel_spec.py:8

# (spec, case id, sizes in dim_vars order, dtype override or None)
CASES = [
    ("rmsnorm", "small", dict(m=64, n=512), None),
    ("rmsnorm", "ragged", dict(m=33, n=1000), None),
    ("layernorm", "small", dict(m=64, n=512), None),
    ("layernorm", "ragged", dict(m=17, n=777), None),
    ("softmax", "small", dict(m=64, n=512), None),
    ("softmax", "ragged", dict(m=5, n=1023), None),
    ("rope", "small", dict(half_d=128, free=128), None),
    ("rope", "ragged", dict(half_d=64, free=100), None),
    ("cumsum", "long", dict(m=4, n=6000), None),
    ("cumsum", "ragged", dict(m=8, n=1000), None),
    ("cumsum", "bf16", dict(m=16, n=1024), "bfloat16"),
    ("fused_adam", "bf16", dict(p=128, f=64), None),
    ("fused_adam", "fp32", dict(p=128, f=64), "float32"),
    ("matmul", "small", dict(m=128, n=256, k=64), None),
    ("matmul", "tiles", dict(m=160, n=320, k=96), None),
    ("silu_mlp", "small", dict(m=128, n=256, k=128, p=128), None),
    ("rmsnorm_matmul", "small", dict(m=128, n=192, k=384), None),
    ("qkv_cte", "small", dict(m=96, n=160, k=256), None),
    ("softmax_mm", "small", dict(m=64, n=96, k=192), None),
    ("attention_nkilib", "small", dict(s=128, d=64), None),
]


def _load_refs(root: Path, name: str):
    path = root / "kernels" / name / "refs.py"
    spec = importlib.util.spec_from_file_location(f"_golden_refs_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _tuple(out):
    if isinstance(out, (tuple, list)):
        return tuple(out)
    return (out,)


def main() -> int:
    import ml_dtypes  # noqa: F401  (registers bfloat16 with numpy)
    import torch

    raw = os.environ.get("AXON_REF_ROOT")
    if not raw:
        print("set AXON_REF_ROOT to the root of the reference (Axon) source tree", file=sys.stderr)
        return 2
    root = Path(raw)
    if not (root / "kernels").is_dir():
        print(f"reference tree not found at {root}", file=sys.stderr)
        return 2
    for name, case, dims, dtype in CASES:
        refs = _load_refs(root, name)
        kwargs = dict(dims)
        if dtype is not None:
            kwargs["dtype"] = np.dtype(dtype)
        inputs = refs.make_inputs(**kwargs, rng=np.random.default_rng(SEED))
        f32 = [np.asarray(a, dtype=np.float32) for a in inputs]
        record = {
            "dims": np.array([dims[k] for k in dims], dtype=np.int64),
            "dim_names": np.array(list(dims)),
            "dtypes": np.array([np.asarray(a).dtype.name for a in inputs]),
        }
        for i, a in enumerate(inputs):
            a = np.asarray(a)
            record[f"in_{i}"] = a.view(np.uint16) if a.dtype.name == "bfloat16" else a
        base = [np.asarray(o, dtype=np.float32) for o in _tuple(refs.baseline_op(*f32))]
        for i, o in enumerate(base):
            record[f"baseline_{i}"] = o
        if getattr(refs, "torch_ref", None) is not None:
            t_out = refs.torch_ref(*[torch.from_numpy(a.copy()) for a in f32])
            record["torch_vs_baseline"] = np.float64(max(
                float(np.abs(t.numpy().astype(np.float32) - b).max())
                for t, b in zip(_tuple(t_out), base, strict=True)
            ))
        dest = HERE / f"{name}_{case}.npz"
        np.savez_compressed(dest, **record)
        print(f"wrote {dest.name}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
