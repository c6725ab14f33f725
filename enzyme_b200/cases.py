"""Named benchmark cases and the command each runs.

Axon keeps its cases in eval/sizes.json and generates one make target per
case (eval/gen_size_targets.py:25-86), each running
`axon kernels/<kernel> --sizes ... [--dtype D] [--rtol R --atol A] [--lnc 2]
--out out/<kernel>_<case>.csv`; a case with rtol/atol is a head-to-head case
(winner + harness exported). This module holds the cases of the specs this
backend implements -- the reference's own cases for them and one case per
BASELINE config -- and builds the same command for the CUDA backend:

    python -m enzyme_b200.cases list
    python -m enzyme_b200.cases run rmsnorm_h4096 [extra CLI flags]

`--lnc 2` cases map to `--gpus 2`. After a head-to-head case the winner is
specialized into `winners/<kernel>_<case>.py` (enzyme_b200.specialize: a
faster measurement replaces it, a slower or equal one keeps it).
"""

from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

# kernel -> case id -> {sizes (dim_vars order), dtype?, lnc?, rtol?, atol?}
CASES: dict[str, dict[str, dict]] = {
    "cumsum": {
        "fast_small": {"sizes": [1024, 1024], "rtol": 1e-3, "atol": 1e-3},
        "fast_small_bf16": {"sizes": [1024, 1024], "dtype": "bfloat16", "rtol": 1e-2, "atol": 1e-2},
        "nucleus": {"sizes": [128, 32768], "rtol": 1e-3, "atol": 1e-3},
        "fast_large": {"sizes": [4096, 4096], "rtol": 1e-3, "atol": 1e-3},
        "llama3_vocab": {"sizes": [128, 128256], "rtol": 1e-3, "atol": 1e-3},
        "qwen_vocab": {"sizes": [128, 151936], "rtol": 1e-3, "atol": 1e-3},
    },
    "rmsnorm": {
        "h1024": {"sizes": [1024, 1024], "rtol": 1e-2, "atol": 1e-2},
        "h4096": {"sizes": [1024, 4096], "rtol": 1e-2, "atol": 1e-2},
        "h8192": {"sizes": [128, 8192], "rtol": 1e-2, "atol": 1e-2},
        "h8192_l2": {"sizes": [128, 8192], "lnc": 2, "rtol": 1e-2, "atol": 1e-2},
    },
    "layernorm": {
        "llama70b": {"sizes": [128, 8192], "rtol": 2e-2, "atol": 2e-2},
        "qwen32b": {"sizes": [128, 5120], "rtol": 2e-2, "atol": 2e-2},
        "roofline": {"sizes": [2048, 8192]},
    },
    "rope": {
        "llama3_8b": {"sizes": [128, 4096], "rtol": 7.8125e-3, "atol": 2e-2},
        "gqa_long": {"sizes": [128, 32768], "rtol": 7.8125e-3, "atol": 2e-2},
    },
    "fused_adam": {
        "opt_1m": {"sizes": [128, 8192], "rtol": 1e-2, "atol": 1e-2},
        "opt_1m_fp32": {"sizes": [128, 8192], "dtype": "float32", "rtol": 1e-4, "atol": 1e-4},
    },
    "matmul": {
        "sq1k": {"sizes": [1024, 1024, 1024]},
        "ck_16k_l2": {"sizes": [1024, 1024, 16384], "dtype": "float32", "lnc": 2, "rtol": 1e-3, "atol": 1e-3},
        "pm_16k_l2": {"sizes": [16384, 1024, 1024], "lnc": 2, "rtol": 2e-2, "atol": 2e-2},
        "roofline": {"sizes": [4096, 4096, 4096]},
    },
    "rmsnorm_matmul": {
        "sq1k": {"sizes": [1024, 1024, 1024]},
        "h8192": {"sizes": [1024, 8192, 8192]},
    },
    "silu_mlp": {"sq1k": {"sizes": [1024, 1024, 1024, 1024]}},
    "softmax": {"sq1k": {"sizes": [1024, 1024]}, "roofline": {"sizes": [4096, 32768]}},
    # the GEMM-backed neighbours of the hot path (eval/sizes.json:47-74, :96)
    "qkv_cte": {
        "llama405b_1k": {"sizes": [1024, 512, 16384], "rtol": 5e-2, "atol": 1.5e-1},
        "llama405b_8k": {"sizes": [8192, 512, 16384], "rtol": 5e-2, "atol": 1.5e-1},
        "llama70b": {"sizes": [16384, 512, 8192], "rtol": 5e-2, "atol": 1.5e-1},
        "llama70b_l2": {"sizes": [16384, 512, 8192], "lnc": 2, "rtol": 5e-2, "atol": 1.5e-1},
        "mistral123b": {"sizes": [16384, 640, 12288], "rtol": 5e-2, "atol": 1.5e-1},
        "vision_l4": {"sizes": [578, 264, 1408], "rtol": 5e-2, "atol": 1.5e-1},
        # fp32 operands: no fp32 tensor-core GEMM here, the rows record AXON_E_UNSUPPORTED
        "llama405b_1k_fp32": {"sizes": [1024, 512, 16384], "dtype": "float32", "rtol": 1e-3, "atol": 1e-3},
        "vision_l4_fp32": {"sizes": [578, 264, 1408], "dtype": "float32", "rtol": 1e-3, "atol": 1e-3},
    },
    "softmax_mm": {"sq1k": {"sizes": [1024, 1024, 1024]}},
    "attention_nkilib": {
        "d128": {"sizes": [1024, 128], "rtol": 5e-2, "atol": 5e-2},
        "s2k_d128": {"sizes": [2048, 128], "rtol": 5e-2, "atol": 5e-2},
        "s4k_d128": {"sizes": [4096, 128], "rtol": 5e-2, "atol": 5e-2},
        "s8k_d128": {"sizes": [8192, 128], "rtol": 5e-2, "atol": 5e-2},
    },
    # the BASELINE configs (sibling specs)
    "rmsnorm_llama": {"config": {"sizes": [2048, 4096], "rtol": 1e-2, "atol": 1e-2}},
    "rope_gqa": {"config": {"sizes": [4096, 32, 8, 64], "rtol": 1e-2, "atol": 1e-2}},
    "cumsum_nucleus_sorted": {"config": {"sizes": [256, 128256], "rtol": 1e-5, "atol": 1e-7}},
    "silu_mlp_swiglu": {"config": {"sizes": [4096, 14336, 4096, 4096], "rtol": 1e-2, "atol": 1e-2}},
    "fused_adam_cfg": {"config": {"sizes": [15625, 64000], "rtol": 1e-5, "atol": 1e-9}},
}


def all_cases() -> list[str]:
    return [f"{k}_{c}" for k, cs in CASES.items() for c in cs]


def resolve(case: str) -> tuple[str, str, dict]:
    """Split `<kernel>_<case>` (kernel names contain underscores: longest
    kernel prefix wins)."""
    for k in sorted(CASES, key=len, reverse=True):
        if case.startswith(k + "_") and case[len(k) + 1:] in CASES[k]:
            return k, case[len(k) + 1:], CASES[k][case[len(k) + 1:]]
    raise KeyError(f"unknown case {case!r}; see `python -m enzyme_b200.cases list`")


def argv(case: str, out_dir: str = "out") -> list[str]:
    """The CLI arguments of one case (what the reference's make target runs)."""
    kernel, cid, c = resolve(case)
    args = [str(ROOT / "kernels" / kernel), "--sizes", *map(str, c["sizes"])]
    if "dtype" in c:
        args += ["--dtype", c["dtype"]]
    if "rtol" in c and "atol" in c:
        args += ["--rtol", repr(c["rtol"]), "--atol", repr(c["atol"])]
    if c.get("lnc", 1) > 1:
        args += ["--gpus", str(c["lnc"])]
    args += ["--out", f"{out_dir}/{kernel}_{cid}.csv"]
    return args


def main(argv_in: list[str] | None = None) -> int:
    a = list(sys.argv[1:] if argv_in is None else argv_in)
    if not a or a[0] not in ("list", "run", "argv"):
        print(__doc__)
        return 2
    if a[0] == "list":
        for c in all_cases():
            print(c)
        return 0
    if len(a) < 2:
        print("usage: python -m enzyme_b200.cases run <kernel>_<case> [extra CLI flags]", file=sys.stderr)
        return 2
    cmd = argv(a[1]) + a[2:]
    if a[0] == "argv":
        print(" ".join(cmd))
        return 0
    from .cli import build_parser, run

    rc = run(build_parser().parse_args(cmd))
    kernel, cid, c = resolve(a[1])
    if rc == 0 and "rtol" in c and "atol" in c:
        # a head-to-head case updates its deliverable, best measurement wins
        # (what the reference's Makefile does after the bench)
        from .specialize import KeptExisting, SpecializeError, specialize

        try:
            print(f"WROTE {specialize(f'{kernel}_{cid}', out_root=Path('out'), winners_dir=Path('winners'))}")
        except KeptExisting as e:
            print(f"KEEP  {kernel}_{cid}: {e}")
        except SpecializeError as e:
            print(f"no winner for {kernel}_{cid}: {e}", file=sys.stderr)
            return 1
    return rc


if __name__ == "__main__":
    sys.exit(main())
