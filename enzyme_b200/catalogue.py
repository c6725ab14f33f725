"""The static variant catalogue: which CUDA kernel variants implement each spec,
how a spec's TILES_IN_BLOCK_* values map onto `axon_tune_t`, and the variant
modules the bench runner loads.

This replaces Axon's synthesis + emission stage (src/axon/cli.py:697-755
writes `out/<stem>/<fn>__v<i>_t<j>.py` from e-graph extraction): here the
hardware variants are hand-written kernels, so "emission" writes one small
Python module per (hw_variant, tile_variant) whose entry point -- named by
Axon's identifier rule, with the spec's input names as data parameters and
the tile args as keyword-only parameters -- launches the kernel through the
C ABI. Each module embeds the `__axon_tile_constraints__` manifest of its
variant.

Tile knob meaning (the CUDA counterpart of TILES_IN_BLOCK_*):
  row ops, rope, Adam   TILES_IN_BLOCK_N = v -> 32*v threads per row / CTA
                        (row_bulk_warp: v warps per CTA, one row each);
                        TILES_IN_BLOCK_M must be 1 (rows per CTA are derived).
  cumsum                TILES_IN_BLOCK_N = v -> 1024*v elements per scan tile
                        (cluster_dsmem: v CTAs per row; row_stream and
                        balanced_ranges: v = 1).
  GEMM specs            (matmul, rmsnorm_matmul, qkv_cte, softmax_mm)
                        TILES_IN_BLOCK_M must be 1 (128-row tcgen05 tiles per CTA),
                        TILES_IN_BLOCK_N = v -> BLOCK_N = 64*v,
                        TILES_IN_BLOCK_K = v -> min(v, deepest that fits)
                        shared-memory pipeline stages. hw_variant 0 = one CTA
                        per tile, 1 = CTA pairs (cta_group::2, 256-row tiles).
  attention_nkilib      N -> BLOCK_N = 64*v of the exp(q @ k_t) GEMM, K -> its
                        stages; M and P must be 1 (the second GEMM picks its tile).
  silu_mlp              N -> gate/up BLOCK_N = 128*v (64*v output columns),
                        K -> stages, P -> down-projection BLOCK_N = 64*v
                        (recorded; the down GEMM picks its own tile today).
                        hw_variant 0/1/2 stores the activation as 1/2/3 bf16
                        terms, 3 as f16, 4 as f16 with both GEMMs in one
                        kernel (see axon_silu_mlp).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .candidate_filter import TileConstraint, manifest_literal
from .specs import safe_name

ROW_SPECS = ("rmsnorm", "rmsnorm_llama", "layernorm", "softmax")
ROPE_SPECS = ("rope", "rope_gqa")
SCAN_SPECS = ("cumsum", "cumsum_nucleus_sorted")
ADAM_SPECS = ("fused_adam", "fused_adam_cfg")
# GEMM-backed specs: a row pass (or the first GEMM's epilogue) and a
# row-scaled tcgen05 GEMM; their tile knobs are the GEMM's
GEMM_SPECS = ("matmul", "rmsnorm_matmul", "softmax_mm")
QKV_SPECS = ("qkv_cte",)
ATTN_SPECS = ("attention_nkilib",)
MLP_SPECS = ("silu_mlp", "silu_mlp_swiglu")
ALL_SPECS = ROW_SPECS + ROPE_SPECS + SCAN_SPECS + ADAM_SPECS + GEMM_SPECS + QKV_SPECS + ATTN_SPECS + MLP_SPECS

ADAM_BETAS = {"fused_adam": (0.9, 0.999), "fused_adam_cfg": (0.9, 0.95)}


@dataclass(frozen=True)
class Variant:
    hw_variant: int
    name: str


def variants(spec_name: str) -> list[Variant]:
    if spec_name in ROW_SPECS:
        return [Variant(0, "row_resident"), Variant(1, "row_streaming"), Variant(2, "row_bulk_warp")]
    if spec_name == "rope":
        return [Variant(0, "flat_vec16")]
    if spec_name == "rope_gqa":
        return [Variant(0, "token_blocked"), Variant(1, "flat_vec16")]
    if spec_name in SCAN_SPECS:
        return [Variant(0, "decoupled_lookback"), Variant(1, "cluster_dsmem"), Variant(2, "row_stream"),
                Variant(3, "balanced_ranges")]
    if spec_name in ADAM_SPECS:
        return [Variant(0, "grid_stride_vec")]
    if spec_name in GEMM_SPECS:
        # hw_variant i runs axon_gemm variant i + 1 (0 is the library's auto pick)
        return [Variant(0, "tcgen05_ws_persistent"), Variant(1, "tcgen05_cta_pair")]
    if spec_name in ATTN_SPECS:
        # 0: one kernel, scores in TMEM / shared memory (head dim 64, 128);
        # 1: exp GEMM with row sums + row-scaled GEMM (its column tile is the knob)
        return [Variant(0, "tcgen05_fused_attention"), Variant(1, "tcgen05_exp_rowsum")]
    if spec_name in QKV_SPECS:
        # 0: residual sum formed while staging the GEMM operand (one kernel);
        # 1 / 2: a row pass writing h, then the one-CTA / CTA-pair GEMM
        return [Variant(0, "tcgen05_resid3_fused"), Variant(1, "rowpass_tcgen05"), Variant(2, "rowpass_tcgen05_pair")]
    if spec_name in MLP_SPECS:
        return [Variant(0, "tcgen05_act_1term"), Variant(1, "tcgen05_act_2term"), Variant(2, "tcgen05_act_3term"),
                Variant(3, "tcgen05_act_f16"), Variant(4, "tcgen05_act_f16_fused")]
    raise KeyError(f"no CUDA variants for spec '{spec_name}'")


def gemm_max_stages(pair: bool, block_n: int) -> int:
    """Deepest shared-memory ring axon_gemm accepts: 227 KB less barriers over
    one stage (a 128 x 64 A slab plus the B columns the CTA stages), at most 8."""
    b_cols = block_n // 2 if pair else block_n
    return min(8, (232448 - 1280) // (128 * 64 * 2 + b_cols * 64 * 2))


def _one(arg: str) -> TileConstraint:
    return TileConstraint(arg, extent=1, tile_size=1, require_divisible=True)


def constraints(spec_name: str, hw_variant: int, dims: dict, itemsize: int,
                tile_args: Sequence[str]) -> list[TileConstraint]:
    """The feasibility manifest of one variant at concrete dims."""
    out: list[TileConstraint] = []
    args = list(tile_args)
    if spec_name in ROW_SPECS and hw_variant == 2:
        # N = warps per CTA, one row per warp staged in shared memory; rows of
        # a multiple of 16 bytes up to 32 KB (plus the weight, for rmsnorm)
        row_bytes = dims["n"] * itemsize
        fixed = row_bytes if spec_name.startswith("rmsnorm") else 0
        ok = row_bytes % 16 == 0 and row_bytes <= 32768
        allowed = tuple(v for v in (1, 2, 4, 8, 16, 32) if ok and 512 + fixed + v * row_bytes <= 232448)
        out.append(TileConstraint(args[1], extent=32, tile_size=1, require_divisible=False, allowed=allowed or (0,)))
        out.append(_one(args[0]))
    elif spec_name in ROW_SPECS:
        n = dims["n"]
        e = 16 // itemsize
        max_v = (512 if itemsize == 2 else 1024) // 32
        if hw_variant == 0:
            allowed = tuple(v for v in (1, 2, 4, 8, 16, 32) if v <= max_v and 32 * v * e * 8 >= n)
        else:
            allowed = tuple(v for v in (4, 8, 16, 32) if v <= 32)
        out.append(TileConstraint(args[1], extent=max(n, 32 * e * max_v), tile_size=32 * e,
                                  require_divisible=False, allowed=allowed))
        out.append(_one(args[0]))
    elif spec_name == "rope_gqa" and hw_variant == 0:
        # the token-blocked kernel sizes its CTA from the head count; N = tokens per CTA
        out.append(TileConstraint(args[1], extent=8, tile_size=1, require_divisible=True, allowed=(1, 2, 4, 8)))
        out.append(_one(args[0]))
    elif spec_name in ROPE_SPECS or spec_name in ADAM_SPECS:
        out.append(TileConstraint(args[1], extent=256, tile_size=32, require_divisible=True, allowed=(1, 2, 4, 8)))
        out.append(_one(args[0]))
    elif spec_name in SCAN_SPECS and hw_variant in (2, 3):
        # one CTA per row (2) or per SM (3), no tile knob: N must be 1
        out.append(_one(args[1]))
        out.append(_one(args[0]))
    elif spec_name in SCAN_SPECS and hw_variant == 1:
        # N = CTAs per row cluster; each CTA stages its slice of the row (a
        # multiple of 8 elements) in at most 200 KB of shared memory
        n = dims["n"]
        allowed = tuple(v for v in (1, 2, 4, 8) if (-(-n // v) + 7) // 8 * 8 * itemsize <= 200 * 1024)
        out.append(TileConstraint(args[1], extent=8, tile_size=1, require_divisible=True, allowed=allowed or (0,)))
        out.append(_one(args[0]))
    elif spec_name in SCAN_SPECS:
        out.append(TileConstraint(args[1], extent=16384, tile_size=1024, require_divisible=True,
                                  allowed=(2, 4, 8, 16)))
        out.append(_one(args[0]))
    elif spec_name in GEMM_SPECS:
        out.append(_one(args[0]))
        out.append(TileConstraint(args[1], extent=256, tile_size=64, require_divisible=True,
                                  allowed=(1, 2, 4) if hw_variant == 0 else (2, 4)))
        out.append(TileConstraint(args[2], extent=8, tile_size=1, require_divisible=True, allowed=(2, 4, 8)))
    elif spec_name in QKV_SPECS:
        out.append(_one(args[0]))
        out.append(TileConstraint(args[1], extent=256, tile_size=64, require_divisible=True,
                                  allowed=(2, 4) if hw_variant != 1 else (1, 2, 4)))
        out.append(TileConstraint(args[2], extent=8, tile_size=1, require_divisible=True, allowed=(2, 4)))
    elif spec_name in ATTN_SPECS and hw_variant == 0:
        for a in args:  # the fused kernel's tiles are fixed (128 queries x 128 keys)
            out.append(_one(a))
    elif spec_name in ATTN_SPECS:
        # N -> column tile of the exp GEMM (64 * v); K -> stages; M, P fixed
        out.append(_one(args[0]))
        out.append(TileConstraint(args[1], extent=256, tile_size=64, require_divisible=True, allowed=(1, 2, 4)))
        out.append(TileConstraint(args[2], extent=8, tile_size=1, require_divisible=True, allowed=(2, 4)))
        out.append(_one(args[3]))
    elif spec_name in MLP_SPECS:
        out.append(_one(args[0]))
        out.append(TileConstraint(args[1], extent=256, tile_size=128, require_divisible=True, allowed=(1, 2)))
        out.append(TileConstraint(args[2], extent=8, tile_size=1, require_divisible=True, allowed=(2, 4)))
        out.append(TileConstraint(args[3], extent=256, tile_size=64, require_divisible=True, allowed=(1, 2, 4)))
    return out


def tune_for(spec_name: str, hw_variant: int, tiles: dict[str, int]) -> dict | list[dict]:
    """axon_tune_t fields for one tile key (two dicts for the two MLP GEMMs)."""
    t = {k.replace("TILES_IN_BLOCK_", ""): int(x) for k, x in tiles.items()}
    if spec_name in ROW_SPECS:
        return {"variant": hw_variant, "threads": 32 * t["N"]}
    if spec_name == "rope_gqa" and hw_variant == 0:
        return {"variant": 0, "rows_per_cta": t["N"]}
    if spec_name in ROPE_SPECS or spec_name in ADAM_SPECS:
        return {"variant": hw_variant, "threads": 32 * t["N"]}
    if spec_name in SCAN_SPECS:
        if hw_variant in (2, 3):
            return {"variant": hw_variant}
        return {"variant": hw_variant, "split": t["N"] if hw_variant == 1 else 1024 * t["N"]}
    if spec_name in GEMM_SPECS:
        bn = 64 * t["N"]
        return {"variant": hw_variant + 1, "block_n": bn, "stages": min(t["K"], gemm_max_stages(hw_variant == 1, bn))}
    if spec_name in ATTN_SPECS:
        if hw_variant == 0:
            return {"variant": 0}
        bn = 64 * t["N"]
        return {"variant": 1, "block_n": bn, "stages": min(t["K"], gemm_max_stages(False, bn))}
    if spec_name in QKV_SPECS:
        bn = 64 * t["N"]
        if hw_variant == 0:  # stages of x, r1, r2 and the B slab
            return {"variant": 0, "block_n": bn, "stages": min(t["K"], (232448 - 3584) // (3 * 16384 + bn * 128))}
        return {"variant": hw_variant, "block_n": bn,
                "stages": min(t["K"], gemm_max_stages(hw_variant == 2, bn))}
    if spec_name in MLP_SPECS:
        if hw_variant == 4:  # both GEMMs in one kernel (256-column tiles; N and P are recorded only)
            return {"variant": 3, "stages": t["K"], "precision": 4, "down_block_n": 64 * t["P"]}
        precision = 4 if hw_variant == 3 else hw_variant + 1
        return {"block_n": 128 * t["N"], "stages": t["K"], "precision": precision, "down_block_n": 64 * t["P"]}
    raise KeyError(spec_name)


# ---- launching -----------------------------------------------------------------


def to_device(a, device):
    """numpy (incl. ml_dtypes bfloat16) -> torch tensor on `device`."""
    import torch

    a = np.asarray(a)
    if a.dtype.name == "bfloat16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def launch(spec_name: str, hw_variant: int, tiles: dict[str, int], inputs: Sequence, *, out=None):
    """Run one spec on device tensors (positional, in input_specs order) with
    the kernel variant and tile key given; returns the output tensors."""
    from . import _native as N
    from . import ops

    tune = tune_for(spec_name, hw_variant, tiles)
    t = list(inputs)
    if spec_name == "rmsnorm":
        return (ops.rmsnorm(t[0], tune=tune, out=out and out[0]),)
    if spec_name == "rmsnorm_llama":
        n = t[0].shape[1]
        return (ops.rmsnorm(t[0], t[1], scale=1.0 / n, eps=1e-6, tune=tune, out=out and out[0]),)
    if spec_name == "layernorm":
        return (ops.layernorm(t[0], eps=1e-6, tune=tune, out=out and out[0]),)
    if spec_name == "softmax":
        return (ops.softmax(t[0], tune=tune, out=out and out[0]),)
    if spec_name == "rope":
        oe, oo = (out if out else (None, None))
        return ops.rope_split(*t, out_even=oe, out_odd=oo, tune=tune)
    if spec_name == "rope_gqa":
        qo, ko = (out if out else (None, None))
        return ops.rope_rotate_half(*t, q_out=qo, k_out=ko, tune=tune)
    if spec_name in SCAN_SPECS:
        return (ops.cumsum(t[0], tune=tune, out=out and out[0]),)
    if spec_name in ADAM_SPECS:
        b1, b2 = ADAM_BETAS[spec_name]
        return ops.adam(*t[:4], step_size=t[4], inv_bc2_sqrt=t[5], wd=t[6], beta1=b1, beta2=b2, eps=1e-8,
                        out=out, tune=tune)
    if spec_name == "matmul":
        return (ops.gemm(t[0], t[1], tune=tune, out=out and out[0]),)
    if spec_name == "rmsnorm_matmul":
        return (ops.rmsnorm_matmul(t[0], t[1], tune=tune, out=out and out[0]),)
    if spec_name == "qkv_cte":
        return (ops.qkv_cte(*t, tune=tune, out=out and out[0]),)
    if spec_name == "softmax_mm":
        return (ops.softmax_mm(*t, tune=tune, out=out and out[0]),)
    if spec_name in ATTN_SPECS:
        return (ops.attention(*t, tune=tune, out=out and out[0]),)
    if spec_name in MLP_SPECS:
        tune = dict(tune)
        tune.pop("down_block_n")
        return (ops.silu_mlp(*t, out=out and out[0], tune=tune),)
    raise KeyError(spec_name)


# ---- variant modules -------------------------------------------------------------

_MODULE = '''"""Axon B200 variant module: spec {spec!r}, hw_variant {hw} ({vname}), tile_variant {tv}.

Generated by enzyme_b200.catalogue; the bench runner loads it by path and calls
`{fn}` with device tensors bound by name and the tile key as keywords.
"""

from enzyme_b200.catalogue import launch as _launch

{manifest_name} = {manifest}

SPEC_NAME = {spec!r}
HW_VARIANT = {hw}


def {fn}({params}, *, {tile_params}):
    return _launch(SPEC_NAME, HW_VARIANT, {tile_dict}, ({params},))
'''


def emit_variant_modules(spec, dims: dict, itemsize: int, paths) -> list[Path]:
    """Write one module per hw variant (tile_variant 0) into the run dir."""
    from .candidate_filter import MANIFEST_NAME

    fn = safe_name(spec.name)
    params = ", ".join(spec.input_names())
    tile_params = ", ".join(spec.tile_args)
    tile_dict = "{" + ", ".join(f"{a!r}: {a}" for a in spec.tile_args) + "}"
    written = []
    paths.run_dir.mkdir(parents=True, exist_ok=True)
    for var in variants(spec.name):
        cons = constraints(spec.name, var.hw_variant, dims, itemsize, spec.tile_args)
        text = _MODULE.format(spec=spec.name, hw=var.hw_variant, vname=var.name, tv=0, fn=fn, params=params,
                              tile_params=tile_params, tile_dict=tile_dict, manifest_name=MANIFEST_NAME,
                              manifest=manifest_literal(cons))
        p = paths.variant_module(fn, var.hw_variant, 0)
        p.write_text(text)
        written.append(p)
    return written
