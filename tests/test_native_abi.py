"""The C-ABI library loads and exports every symbol include/axon_b200.h
declares; argument validation runs on the host (no GPU needed)."""

from __future__ import annotations

import ctypes
import json

import pytest

from enzyme_b200 import _native as N


def test_library_exports_every_header_symbol():
    lib = N.lib()
    declared = N.header_symbols()
    assert len(declared) >= 18
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(declared) == set(N.SIGNATURES), "ctypes signature table out of sync with the header"


def test_version_and_variants():
    assert N.version().startswith("axon_b200")
    for op in ("rmsnorm", "layernorm", "softmax", "rope", "cumsum", "adam", "gemm"):
        d = json.loads(N.variants(op))
        assert d["op"] == op and d["variants"]
    with pytest.raises(N.AxonError) as e:
        N.variants("nope")
    assert e.value.code == N.AXON_E_UNSUPPORTED


def test_variants_truncates_to_buffer():
    lib = N.lib()
    need = lib.axon_variants(b"gemm", None, 0)
    buf = ctypes.create_string_buffer(8)
    assert lib.axon_variants(b"gemm", buf, 8) == need
    assert len(buf.value) == 7


def test_null_pointers_are_rejected_before_any_launch():
    lib = N.lib()
    rc = lib.axon_rmsnorm(None, None, None, 4, 4, 4, 4, N.AXON_BF16, 0, 1.0, 0.0, None, None)
    assert rc == N.AXON_E_ARG
    assert "NULL" in N.last_error()
    rc = lib.axon_gemm(None, None, None, None, None, 8, 8, 8, 8, 8, 8, N.AXON_BF16, N.AXON_BF16, 0, None, None)
    assert rc == N.AXON_E_ARG


def test_gemm_shape_rules_checked_on_host():
    lib = N.lib()
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: validation fails first
    rc = lib.axon_gemm(fake, fake, None, fake, None, 8, 8, 12, 12, 8, 8, N.AXON_BF16, N.AXON_BF16, 0, None, None)
    assert rc == N.AXON_E_SHAPE and "multiples of 8" in N.last_error()
    rc = lib.axon_gemm(fake, fake, None, fake, None, 8, 8, 8, 8, 8, 8, N.AXON_F32, N.AXON_BF16, 0, None, None)
    assert rc == N.AXON_E_UNSUPPORTED
    t = N.Tune(block_n=96)
    rc = lib.axon_gemm(fake, fake, None, fake, None, 8, 8, 8, 8, 8, 8, N.AXON_BF16, N.AXON_BF16, 0,
                       ctypes.byref(t), None)
    assert rc == N.AXON_E_ARG


def test_cumsum_workspace_query_is_host_only():
    lib = N.lib()
    nbytes = lib.axon_cumsum_workspace_bytes(256, 128256, None)
    tiles = 256 * -(-128256 // 8192)
    assert nbytes == 32 + 32 * tiles
    assert lib.axon_cumsum_workspace_bytes(-1, 4, None) == N.AXON_E_SHAPE
    rc = lib.axon_cumsum(ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 4, 4, 4, N.AXON_F32, N.AXON_F32, None, 0,
                         None, None)
    assert rc == N.AXON_E_ARG and "workspace" in N.last_error()


def test_error_is_thread_local():
    import threading

    lib = N.lib()
    lib.axon_rmsnorm(None, None, None, 1, 1, 1, 1, 0, 0, 1.0, 0.0, None, None)
    seen = []
    t = threading.Thread(target=lambda: seen.append(N.last_error()))
    t.start()
    t.join()
    assert seen == [""]
    assert "NULL" in N.last_error()
