"""ctypes binding of `libaxon_b200.so`, the C ABI declared in include/axon_b200.h.

The shared library is built in-tree (`python -m enzyme_b200.build`) into
`enzyme_b200/lib/`. There is no fallback: if the library is missing or does
not export a symbol the header declares, `lib()` raises.
"""

from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "lib" / "libaxon_b200.so"
HEADER_PATH = PKG_DIR.parent / "include" / "axon_b200.h"

AXON_OK = 0
AXON_E_SHAPE = -1
AXON_E_ALIGN = -2
AXON_E_LAUNCH = -3
AXON_E_TIMEOUT = -4
AXON_E_UNSUPPORTED = -5
AXON_E_ARG = -6
AXON_E_CUDA = -7

AXON_F32 = 0
AXON_BF16 = 1
AXON_F16 = 2

AXON_EPI_NONE = 0
AXON_EPI_ROWSCALE = 1
AXON_EPI_SILU_GATE = 2
AXON_EPI_EXP = 3

AXON_IPC_HANDLE_BYTES = 64

_CODE_NAMES = {
    AXON_E_SHAPE: "AXON_E_SHAPE",
    AXON_E_ALIGN: "AXON_E_ALIGN",
    AXON_E_LAUNCH: "AXON_E_LAUNCH",
    AXON_E_TIMEOUT: "AXON_E_TIMEOUT",
    AXON_E_UNSUPPORTED: "AXON_E_UNSUPPORTED",
    AXON_E_ARG: "AXON_E_ARG",
    AXON_E_CUDA: "AXON_E_CUDA",
}


class AxonError(RuntimeError):
    """A negative status from the C ABI, with axon_last_error()'s message."""

    def __init__(self, code: int, message: str):
        self.code = code
        self.message = message
        super().__init__(f"{_CODE_NAMES.get(code, code)}: {message}")

    def __reduce__(self):
        # rebuilt from (code, message): a bench worker process sends it back
        # to the CLI, which records it in the key's error row
        return (type(self), (self.code, self.message))


class Tune(ctypes.Structure):
    """`axon_tune_t`: variant id and tile knobs; zero means the op's default."""

    _fields_ = [
        ("variant", ctypes.c_int32),
        ("threads", ctypes.c_int32),
        ("rows_per_cta", ctypes.c_int32),
        ("block_m", ctypes.c_int32),
        ("block_n", ctypes.c_int32),
        ("block_k", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("split", ctypes.c_int32),
        ("precision", ctypes.c_int32),
        ("max_ctas", ctypes.c_int32),
    ]

    @classmethod
    def of(cls, tune: dict | None) -> Tune | None:
        if not tune:
            return None
        t = cls()
        for k, v in tune.items():
            setattr(t, k, int(v))
        return t


class AdamHParams(ctypes.Structure):
    """`axon_adam_hparams_t`."""

    _fields_ = [
        ("beta1", ctypes.c_float),
        ("beta2", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("step_size", ctypes.c_float),
        ("inv_bc2_sqrt", ctypes.c_float),
        ("wd", ctypes.c_float),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F = ctypes.c_float
_TUNE = ctypes.POINTER(Tune)

# name -> (restype, argtypes); mirrors include/axon_b200.h
SIGNATURES: dict[str, tuple] = {
    "axon_version": (ctypes.c_char_p, []),
    "axon_last_error": (ctypes.c_char_p, []),
    "axon_variants": (_I64, [ctypes.c_char_p, ctypes.c_char_p, _I64]),
    "axon_rmsnorm": (_I32, [_P, _P, _P, _I64, _I64, _I64, _I64, _I32, _I32, _F, _F, _TUNE, _P]),
    "axon_layernorm": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _I32, _F, _TUNE, _P]),
    "axon_softmax": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _I32, _TUNE, _P]),
    "axon_rope_split": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _TUNE, _P]),
    "axon_rope_rotate_half": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _TUNE, _P]),
    "axon_cumsum_workspace_bytes": (_I64, [_I64, _I64, _TUNE]),
    "axon_cumsum": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _I32, _I32, _P, _I64, _TUNE, _P]),
    "axon_cumsum_status": (_I32, [_P, _P]),
    "axon_cumsum_noalloc": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _I32, _I32, _TUNE, _P]),
    "axon_adam": (
        _I32,
        [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I32, _I32, _P, _P, _P, _I32,
         ctypes.POINTER(AdamHParams), _TUNE, _P],
    ),
    "axon_gemm": (_I32, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _I32, _I32, _TUNE, _P]),
    "axon_gemm_status": (_I32, [_P]),
    "axon_cast": (_I32, [_P, _P, _I64, _I32, _I32, _P]),
    "axon_selftest_bounded_wait": (_I32, [_I64, _P, _P, _P]),
    "axon_row_rsqrt": (_I32, [_P, _P, _I64, _I64, _I64, _I32, _F, _F, _P]),
    "axon_row_status": (_I32, [_P]),
    "axon_rmsnorm_matmul": (_I32, [_P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _TUNE, _P]),
    "axon_gemm_exp": (_I32, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _I32, _TUNE, _P]),
    "axon_gemm_resid3_workspace_bytes": (_I64, [_I64, _I64, _I64, _TUNE]),
    "axon_gemm_resid3": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _I32, _F, _TUNE, _P]),
    "axon_qkv_cte_workspace_bytes": (_I64, [_I64, _I64, _I64, _TUNE]),
    "axon_qkv_cte": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _I32, _TUNE, _P]),
    "axon_softmax_mm_workspace_bytes": (_I64, [_I64, _I64]),
    "axon_softmax_mm": (_I32, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I32, _I32, _TUNE, _P]),
    "axon_attention_workspace_bytes": (_I64, [_I64, _I64, _TUNE]),
    "axon_attention_fused_workspace_bytes": (_I64, [_I64, _I64, _TUNE]),
    "axon_attention_fused": (_I32, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _TUNE, _P]),
    "axon_attention": (_I32, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _TUNE, _P]),
    "axon_silu_mlp_workspace_bytes": (_I64, [_I64, _I64, _I64, _I32, _TUNE]),
    "axon_ipc_handle": (_I32, [_P, _P, ctypes.POINTER(_I64)]),
    "axon_ipc_open": (_I32, [_P, _I64, ctypes.POINTER(_P)]),
    "axon_ipc_close": (_I32, [_P, _I64]),
    "axon_tp_down_partial": (_I32, [_P, _P, _P, _I32, _I32, _I64, _I64, _I64, _I64, _I32, _TUNE, _P]),
    "axon_tp_mlp_workspace_bytes": (_I64, [_I64, _I64]),
    "axon_tp_mlp_partial": (
        _I32, [_P, _P, _P, _P, _P, _I64, _P, _I32, _I32, _I64, _I64, _I64, _I64, _I64, _TUNE, _P]
    ),
    "axon_tp_step_done_per_epoch": (_I64, [_I32, _I64, _I64]),
    "axon_tp_mlp_step": (
        _I32, [_P, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _TUNE, _P]
    ),
    "axon_tp_mlp_step_multicast": (
        _I32, [_P, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _TUNE, _P]
    ),
    "axon_tp_wait_count": (_I32, [_P, _I32, _P]),
    "axon_tp_signal": (_I32, [_P, _I32, _I32, _I32, _P]),
    "axon_tp_wait": (_I32, [_P, _I32, _I32, _P]),
    "axon_tp_reduce_gather": (_I32, [_P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _I32, _I32, _P]),
    "axon_tp_reduce_local": (_I32, [_P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _I32, _I32, _P]),
    "axon_tp_reduce_multicast": (_I32, [_P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I64, _I64, _I32, _I32, _P]),
    "axon_tp_push_rows": (_I32, [_P, _P, _I64, _I32, _I32, _P]),
    "axon_tp_status": (_I32, [_P]),
    "axon_silu_mlp": (
        _I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I32, _I32, _TUNE, _P]
    ),
}

_LIB: ctypes.CDLL | None = None


def header_symbols() -> list[str]:
    """Every function the C header declares (the ABI contract)."""
    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"^AXON_API\s+[\w\s\*]+?\b(axon_\w+)\s*\(", text, re.M)))


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it is missing (no CPU fallback)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = Path(os.environ.get("AXON_B200_LIB", LIB_PATH))
    if not path.is_file():
        raise RuntimeError(
            f"libaxon_b200.so not found at {path}; build it with "
            "`python -m enzyme_b200.build` (the CUDA path has no fallback)"
        )
    handle = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = handle
    return handle


def last_error() -> str:
    return lib().axon_last_error().decode()


def check(rc: int) -> None:
    if rc != AXON_OK:
        raise AxonError(int(rc), last_error())


def variants(op: str) -> str:
    n = lib().axon_variants(op.encode(), None, 0)
    if n < 0:
        check(int(n))
    buf = ctypes.create_string_buffer(int(n) + 1)
    lib().axon_variants(op.encode(), buf, n + 1)
    return buf.value.decode()


def version() -> str:
    return lib().axon_version().decode()
