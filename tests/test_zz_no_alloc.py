"""The allocation-free cumsum entry point, called through the C ABI.

`axon_cumsum_noalloc` is for callers that must not allocate device memory
(a plugin whose host framework owns every allocation, or a path where
cudaMalloc's device-wide synchronisation is not allowed). It uses a fixed
static device array as its look-back scratch instead of a caller workspace.
These tests check it against the workspace entry point `axon_cumsum` on the
same inputs, twice in a row (the static scratch keeps the previous call's
contents, so the second call proves it is cleared), that the device status
word read by `axon_cumsum_status(NULL, ...)` reports no look-back wait that
gave up after each call, and that shapes beyond the static capacity are
refused on the host. This file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from enzyme_b200 import _native as N

pytestmark = pytest.mark.gpu

CAPACITY = 1 << 20


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _code(t):
    return {torch.float32: N.AXON_F32, torch.bfloat16: N.AXON_BF16}[t.dtype]


def _cumsum_with_workspace(x, y, tune):
    lib = N.lib()
    m, n = x.shape
    need = lib.axon_cumsum_workspace_bytes(m, n, tune)
    ws = torch.empty(need, dtype=torch.uint8, device=x.device)
    rc = lib.axon_cumsum(x.data_ptr(), y.data_ptr(), m, n, x.stride(0), y.stride(0), _code(x), _code(y),
                         ws.data_ptr(), need, tune, _stream())
    assert rc == N.AXON_OK, N.last_error()
    assert lib.axon_cumsum_status(ws.data_ptr(), _stream()) == N.AXON_OK


def _cumsum_noalloc(x, y, tune):
    m, n = x.shape
    return N.lib().axon_cumsum_noalloc(x.data_ptr(), y.data_ptr(), m, n, x.stride(0), y.stride(0), _code(x),
                                       _code(y), tune, _stream())


def _assert_no_timeout():
    """The look-back kernel records a wait that gave up in the library's
    device status word; reading it synchronises the stream and clears it."""
    rc = N.lib().axon_cumsum_status(None, _stream())
    assert rc == N.AXON_OK, N.last_error()


@pytest.mark.parametrize("split", [0, 2048])
def test_noalloc_matches_workspace_entry_point_twice(split, cuda_device):
    torch.cuda.set_device(cuda_device)
    gen = torch.Generator(device=cuda_device).manual_seed(42)
    x = torch.softmax(2.0 * torch.randn(96, 50000, device=cuda_device, generator=gen), dim=1)
    x = torch.sort(x, dim=1, descending=True).values.contiguous()
    tune = ctypes.byref(N.Tune(split=split)) if split else None
    want = torch.empty_like(x)
    _cumsum_with_workspace(x, want, tune)
    for _ in range(2):
        got = torch.full_like(x, float("nan"))
        rc = _cumsum_noalloc(x, got, tune)
        assert rc == N.AXON_OK, N.last_error()
        _assert_no_timeout()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=1e-7)


def test_noalloc_bf16_in_fp32_out(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(7)
    x = torch.randn(8, 30000, device=cuda_device, generator=gen).to(torch.bfloat16)
    want = torch.empty(x.shape, dtype=torch.float32, device=cuda_device)
    _cumsum_with_workspace(x, want, None)
    got = torch.empty_like(want)
    assert _cumsum_noalloc(x, got, None) == N.AXON_OK, N.last_error()
    _assert_no_timeout()
    np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=1e-5, atol=1e-5)


def test_noalloc_refuses_shapes_beyond_the_static_scratch(cuda_device):
    x = torch.zeros(4, 8, device=cuda_device)
    # 40000 rows x 2 tiles of 8192 needs 2.56 MB of descriptors: refused on the
    # host before anything is launched (the tiny tensors are never touched)
    rc = N.lib().axon_cumsum_noalloc(x.data_ptr(), x.data_ptr(), 40000, 16384, 16384, 16384, N.AXON_F32,
                                     N.AXON_F32, None, _stream())
    assert rc == N.AXON_E_SHAPE
    assert "static" in N.last_error() and str(CAPACITY) in N.last_error()
