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


def test_row_variants_and_host_checks():
    """Row ops list variants 0-3; an unknown variant and a CTA size that is not
    whole warps are refused on the host, before any CUDA call."""
    lib = N.lib()
    for op in ("rmsnorm", "layernorm", "softmax"):
        d = json.loads(N.variants(op))
        assert [v["id"] for v in d["variants"]] == [0, 1, 2, 3]
        assert d["variants"][3]["name"] == "row_bulk_cta"
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: validation fails first
    for tune, text in ((N.Tune(variant=4), "unknown variant"), (N.Tune(variant=3, threads=100), "multiple of 32")):
        rc = lib.axon_softmax(fake, fake, 4, 64, 64, 64, N.AXON_F32, ctypes.byref(tune), None)
        assert rc == N.AXON_E_ARG and text in N.last_error()


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


def test_split_plans_without_a_gpu():
    """Workspace queries of the one-kernel qkv_cte and attention paths (on a
    host without a GPU the SM count reads as B200's 148): no k split once the
    row blocks fill the GPU, splits (fp32 partials + row sums) when they
    do not, and explicit splits honoured."""
    lib = N.lib()
    t = N.Tune.of
    assert lib.axon_gemm_resid3_workspace_bytes(16384, 512, 8192, None) == 0
    # 8 row blocks of 1024 rows: 18 k splits of 15 k-blocks (16384 / 64 = 256 k-blocks)
    want = -(-(18 * 1024 * 512 * 4) // 256) * 256 + 18 * 1024 * 4
    assert lib.axon_gemm_resid3_workspace_bytes(1024, 512, 16384, None) == want
    assert lib.axon_gemm_resid3_workspace_bytes(1024, 512, 16384, t({"split": 1})) == 0
    assert lib.axon_gemm_resid3_workspace_bytes(1024, 512, 16384, t({"block_n": 100})) < 0  # rejected width
    # attention: 64 query blocks at s = 8192 -> 2 key splits; 128 or more -> none
    want = -(-(2 * 8192 * 128 * 4) // 256) * 256 + 2 * 8192 * 4
    assert lib.axon_attention_fused_workspace_bytes(8192, 128, None) == want
    assert lib.axon_attention_fused_workspace_bytes(32768, 128, None) == 0
    assert lib.axon_attention_workspace_bytes(8192, 128, None) == want
    # the two-GEMM form stages the [s, s] scores
    assert lib.axon_attention_workspace_bytes(8192, 128, t({"variant": 1})) >= 8192 * 8192 * 2
    assert lib.axon_attention_workspace_bytes(1024, 512, None) >= 1024 * 1024 * 2  # d = 512: two-GEMM form
    # qkv_cte: the one-kernel default vs the row-pass variants (h + row scales)
    assert lib.axon_qkv_cte_workspace_bytes(16384, 512, 8192, None) == 0
    assert lib.axon_qkv_cte_workspace_bytes(578, 264, 1408, t({"variant": 1})) >= 578 * 1408 * 2 + 578 * 4
