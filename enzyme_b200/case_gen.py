"""The per-case head-to-head harness module (`out/winners/<spec>_<case>_case.py`).

Contract kept from Axon's src/axon/case_gen.py:30-134 (the module nkilib's
TestAxonEmitted imports, agent_opt/test_axon_emitted.py:52-103): a `CASE`
dict (name, entry_point, kernel_rel, refs_rel, dtype, input_names,
shape_args, rtol, atol) plus `torch_ref`, `make_inputs` and
`output_tensors`. `torch_ref` coerces every input to fp32 torch before the
spec's reference and returns `output_<i>` in the case dtype. The spec's
`refs.py` is located by a path relative to the harness and loaded by path,
so the harness needs neither this package nor the kernel library to run the
reference side.
"""

from __future__ import annotations

import json
import os
from pathlib import Path

from .kernel_spec import SEED, KernelSpec


def generate_case_module(spec: KernelSpec, kernel_path: Path | str, dtype: str, dest: Path, *, name: str,
                         entry_point: str, shape_args: dict[str, int], rtol: float, atol: float) -> None:
    if spec.torch_ref is None or spec.baseline_op is None:
        raise ValueError(f"{spec.name}: head-to-head case needs both torch_ref and baseline_op")
    kabs = Path(kernel_path).resolve()
    if kabs.is_dir():
        refs = kabs / "refs.py"
        if not refs.is_file():
            raise ValueError(f"{spec.name}: kernel dir {kabs} has no refs.py")
        kabs = refs
    dest = Path(dest).resolve()
    krel = os.path.relpath(kabs, dest.parent)
    inputs = spec.input_names()
    for label, names in (("input", inputs), ("dim", list(spec.dim_vars)), ("tile", list(spec.tile_args))):
        bad = [n for n in names if not n.isidentifier()]
        if bad:
            raise ValueError(f"{spec.name}: {label} names are not valid identifiers: {bad}")
    case = {"name": name, "entry_point": entry_point, "kernel_rel": f"{name}.py", "refs_rel": krel,
            "dtype": dtype, "input_names": inputs, "shape_args": shape_args, "rtol": rtol, "atol": atol}
    tiles = list(spec.tile_args)
    dims = list(spec.dim_vars)
    del_tiles = f"    del {', '.join(tiles)}\n" if tiles else ""
    body = _TEMPLATE.format(
        kernel_name=spec.name, dtype=dtype, seed=SEED, refs_rel=krel, input_names=repr(inputs),
        case_literal=json.dumps(case, indent=4),
        ref_params=", ".join([*inputs, *tiles]), del_tiles=del_tiles,
        coerced=", ".join(f"_f32({n})" for n in inputs),
        mk_params=", ".join([*dims, *tiles]), dim_pass=", ".join(f"{d}={d}" for d in dims),
        tile_pass=", ".join(f'"{t}": int({t})' for t in tiles))
    dest.parent.mkdir(parents=True, exist_ok=True)
    dest.write_text(body)


_TEMPLATE = '''"""Head-to-head harness for {kernel_name!r} (dtype={dtype!r}); generated, do not edit."""

import importlib.util as _ilu
import os as _os

import ml_dtypes  # noqa: F401  (registers bfloat16 with numpy)
import numpy as np
import torch

_SEED = {seed}
_DTYPE = "{dtype}"
_REFS_PATH = _os.path.normpath(_os.path.join(_os.path.dirname(_os.path.abspath(__file__)), {refs_rel!r}))
_INPUT_NAMES = {input_names}

CASE = {case_literal}

_torch_dt = getattr(torch, _DTYPE)
_np_dt = np.dtype(_DTYPE)


def _f32(a):
    """fp32 torch tensor (numpy bfloat16 is widened on the numpy side first)."""
    if isinstance(a, torch.Tensor):
        return a.to(torch.float32)
    return torch.from_numpy(np.asarray(a).astype(np.float32))


def _load_refs():
    s = _ilu.spec_from_file_location("_axon_b200_case_refs_{kernel_name}", _REFS_PATH)
    m = _ilu.module_from_spec(s)
    s.loader.exec_module(m)
    return getattr(m, "SPEC", m)


_SPEC = _load_refs()


def torch_ref({ref_params}):  # noqa: N803
{del_tiles}    out = _SPEC.torch_ref({coerced})
    if not isinstance(out, tuple):
        out = (out,)
    return {{f"output_{{i}}": t.to(_torch_dt) for i, t in enumerate(out)}}


def make_inputs({mk_params}):  # noqa: N803
    data = _SPEC.make_inputs({dim_pass}, dtype=_np_dt, rng=np.random.default_rng(_SEED))
    out = dict(zip(_INPUT_NAMES, data))
    out.update({{{tile_pass}}})
    return out


def output_tensors(kernel_input):
    ref = _SPEC.baseline_op(*[kernel_input[n] for n in _INPUT_NAMES])
    if not isinstance(ref, tuple):
        ref = (ref,)
    return {{f"output_{{i}}": np.zeros(np.asarray(a).shape, dtype=_np_dt) for i, a in enumerate(ref)}}
'''
