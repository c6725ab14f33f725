"""Algorithmic work per spec (each input read once, each output written once;
GEMM FLOPs 2*m*n*k) and the roofline denominators.

The peaks are the driver-measured ones in MEASURED_PEAKS.json at the repository
root (a STREAM-style copy and a cuBLAS bf16 GEMM on this pool's B200s); when
that file is absent the earlier pool measurement (6650 GB/s, 1590 TFLOP/s) is
used and reported as "fallback".
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            d = json.loads(p.read_text())
            return {**FALLBACK, **{k: float(d[k]) for k in FALLBACK if k in d}, "source": "measured"}
        except (ValueError, KeyError):
            pass
    return {**FALLBACK, "source": "fallback"}


def nbytes(shape, itemsize: int) -> int:
    return int(np.prod(shape)) * itemsize


KNOWN = frozenset({"rmsnorm", "layernorm", "softmax", "cumsum", "cumsum_nucleus_sorted", "rmsnorm_llama", "rope",
                   "rope_gqa", "fused_adam", "fused_adam_cfg", "matmul", "rmsnorm_matmul", "silu_mlp",
                   "silu_mlp_swiglu"})


def work(spec: str, dims: dict, itemsize: int = 2) -> tuple[str, float]:
    """('hbm', bytes) or ('tensor', flops) for one launch of a spec at dims."""
    d = dims
    if spec in ("rmsnorm", "layernorm", "softmax", "cumsum", "cumsum_nucleus_sorted"):
        return "hbm", 2 * d["m"] * d["n"] * itemsize
    if spec == "rmsnorm_llama":
        return "hbm", 2 * d["m"] * d["n"] * itemsize + d["n"] * itemsize
    if spec == "rope":
        return "hbm", 6 * d["half_d"] * d["free"] * itemsize
    if spec == "rope_gqa":
        qk = d["s"] * (d["hq"] + d["hkv"]) * 2 * d["half_d"] * itemsize
        return "hbm", 2 * qk + 2 * d["s"] * d["half_d"] * 4
    if spec == "fused_adam":
        return "hbm", 7 * d["p"] * d["f"] * itemsize + 3 * d["p"] * itemsize
    if spec == "fused_adam_cfg":
        return "hbm", 26 * d["p"] * d["f"] + 3 * 4 * d["p"]
    if spec in ("matmul", "rmsnorm_matmul", "softmax_mm"):
        return "tensor", 2.0 * d["m"] * d["n"] * d["k"]
    if spec == "qkv_cte":
        # three [m, k] inputs read, w read, y written: HBM-bound at the
        # reference's shapes (n = 512: 2n/6 ~ 170 FLOP per byte, below B200's
        # ridge of ~250)
        return "hbm", (3 * d["m"] * d["k"] + d["k"] * d["n"] + d["m"] * d["n"]) * itemsize
    if spec == "attention_nkilib":
        return "tensor", 4.0 * d["s"] * d["s"] * d["d"]
    if spec in ("silu_mlp", "silu_mlp_swiglu"):
        return "tensor", 2.0 * d["m"] * d["k"] * d["n"] * 2 + 2.0 * d["m"] * d["n"] * d["p"]
    raise KeyError(spec)


def fraction(kind: str, amount: float, seconds: float, sustained: bool = False) -> dict:
    """Achieved rate over the measured peak. `sustained` selects, for a
    tensor-bound kernel timed inside a long loop (where the 1 kW power cap
    holds the clock near 1.3 GHz), the sustained GEMM peak; the burst
    fraction is reported beside it."""
    pk = peaks()
    if kind == "hbm":
        achieved = amount / seconds / 1e9
        return {"bound": kind, "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "peak_source": pk["source"]}
    achieved = amount / seconds / 1e12
    peak = pk["bf16_tflops_sustained"] if sustained else pk["bf16_tflops"]
    return {"bound": kind, "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": pk["source"], "peak_kind": "sustained" if sustained else "burst",
            "frac_of_burst": achieved / pk["bf16_tflops"]}
