"""Torch-facing wrappers over the C ABI (one function per entry point).

Tensors must live on a CUDA device; PyTorch provides memory and the current
stream, the kernels are `libaxon_b200.so`'s. Every call checks the returned
status and raises `AxonError` on failure. Nothing here computes on the CPU.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N
from ._native import AdamHParams, Tune, check

_DT = {torch.float32: N.AXON_F32, torch.bfloat16: N.AXON_BF16, torch.float16: N.AXON_F16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise N.AxonError(N.AXON_E_UNSUPPORTED, f"dtype {t.dtype} not supported") from None


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise N.AxonError(N.AXON_E_ARG, "tensor is not on a CUDA device (no CPU path)")


def _rows(x: torch.Tensor) -> tuple[int, int, int]:
    """(m, n, ld) of a 2-D tensor whose last dim is contiguous."""
    if x.dim() != 2 or x.stride(1) != 1:
        raise N.AxonError(N.AXON_E_SHAPE, "expected a 2-D tensor with a contiguous last dim")
    return x.shape[0], x.shape[1], x.stride(0)


def _tune(tune: dict | None):
    t = Tune.of(tune)
    return ctypes.byref(t) if t is not None else None


def rmsnorm(x, w=None, *, scale=None, eps=0.0, out=None, tune=None):
    """y = x * rsqrt(scale*sum(x^2) + eps) [* w]; scale defaults to 1 (sum form)."""
    _require_cuda(x, w)
    m, n, ldx = _rows(x)
    y = out if out is not None else torch.empty_like(x)
    _, _, ldy = _rows(y)
    wd = dtype_code(w) if w is not None else 0
    check(N.lib().axon_rmsnorm(_ptr(x), _ptr(w), _ptr(y), m, n, ldx, ldy, dtype_code(x), wd,
                               1.0 if scale is None else float(scale), float(eps), _tune(tune), _stream(x)))
    return y


def layernorm(x, *, eps=1e-6, out=None, tune=None):
    _require_cuda(x)
    m, n, ldx = _rows(x)
    y = out if out is not None else torch.empty_like(x)
    _, _, ldy = _rows(y)
    check(N.lib().axon_layernorm(_ptr(x), _ptr(y), m, n, ldx, ldy, dtype_code(x), float(eps), _tune(tune),
                                 _stream(x)))
    return y


def softmax(x, *, out=None, tune=None):
    _require_cuda(x)
    m, n, ldx = _rows(x)
    y = out if out is not None else torch.empty_like(x)
    _, _, ldy = _rows(y)
    check(N.lib().axon_softmax(_ptr(x), _ptr(y), m, n, ldx, ldy, dtype_code(x), _tune(tune), _stream(x)))
    return y


def rope_split(x_even, x_odd, cos, sin, *, out_even=None, out_odd=None, tune=None):
    _require_cuda(x_even, x_odd, cos, sin)
    for t in (x_even, x_odd, cos, sin):
        if not t.is_contiguous() or t.shape != x_even.shape or t.dtype != x_even.dtype:
            raise N.AxonError(N.AXON_E_SHAPE, "rope_split: inputs must be contiguous, same shape and dtype")
    oe = out_even if out_even is not None else torch.empty_like(x_even)
    oo = out_odd if out_odd is not None else torch.empty_like(x_odd)
    half_d, free = x_even.shape
    check(N.lib().axon_rope_split(_ptr(x_even), _ptr(x_odd), _ptr(cos), _ptr(sin), _ptr(oe), _ptr(oo), half_d,
                                  free, dtype_code(x_even), _tune(tune), _stream(x_even)))
    return oe, oo


def rope_rotate_half(q, k, cos, sin, *, q_out=None, k_out=None, tune=None):
    """q [s, hq, d] (or [s, hq, 2, d/2]), k likewise, fp32 tables [s, d/2]."""
    _require_cuda(q, k, cos, sin)
    if not q.is_contiguous() or (k is not None and not k.is_contiguous()):
        raise N.AxonError(N.AXON_E_SHAPE, "rope_rotate_half: q/k must be contiguous")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32:
        raise N.AxonError(N.AXON_E_UNSUPPORTED, "rope_rotate_half: cos/sin tables must be fp32")
    seq, hq = q.shape[0], q.shape[1]
    d = q[0, 0].numel()
    hkv = k.shape[1] if k is not None else 0
    qo = q_out if q_out is not None else torch.empty_like(q)
    ko = k_out if k_out is not None else (torch.empty_like(k) if k is not None else None)
    check(N.lib().axon_rope_rotate_half(_ptr(q), _ptr(k), _ptr(cos), _ptr(sin), _ptr(qo), _ptr(ko), seq, hq, hkv,
                                        d, dtype_code(q), _tune(tune), _stream(q)))
    return qo, ko


def cumsum_workspace_bytes(m: int, n: int, tune=None) -> int:
    nbytes = N.lib().axon_cumsum_workspace_bytes(m, n, _tune(tune))
    if nbytes < 0:
        check(int(nbytes))
    return int(nbytes)


# Zero-filled cumsum workspaces kept per (device, stream): the scans leave a
# workspace zero-filled (variant 0 clears it itself, variant 3's slots are
# cleared by their readers), so one buffer serves every call on a stream.
_CUMSUM_WS: dict[tuple[int, int], torch.Tensor] = {}


def _cumsum_workspace(x, need: int) -> torch.Tensor:
    key = (x.device.index or 0, _stream(x))
    ws = _CUMSUM_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, dtype=torch.uint8, device=x.device)
        _CUMSUM_WS[key] = ws
    return ws


def cumsum(x, *, out=None, out_dtype=None, workspace=None, tune=None):
    """Inclusive scan along the last axis. Without a `workspace` (uint8
    tensor of cumsum_workspace_bytes, zero-filled before its first use) a
    zero-filled one kept for this device and stream is used."""
    _require_cuda(x)
    m, n, ldx = _rows(x)
    y = out if out is not None else torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    _, _, ldy = _rows(y)
    need = cumsum_workspace_bytes(m, n, tune)
    if workspace is None and need > 0:
        workspace = _cumsum_workspace(x, need)
    wsb = workspace.numel() if workspace is not None else 0
    check(N.lib().axon_cumsum(_ptr(x), _ptr(y), m, n, ldx, ldy, dtype_code(x), dtype_code(y), _ptr(workspace), wsb,
                              _tune(tune), _stream(x)))
    return y


def cumsum_status(workspace=None) -> None:
    """Raise AxonError(AXON_E_TIMEOUT) if a bounded wait gave up (the status
    word of `workspace`, if given, and the device word). A wait that gave up
    can leave a carry slot set, so the kept workspaces are then dropped and
    a caller's own workspace must be zero-filled again."""
    try:
        if workspace is not None:
            check(N.lib().axon_cumsum_status(_ptr(workspace), _stream(workspace)))
        else:
            check(N.lib().axon_cumsum_status(None, torch.cuda.current_stream().cuda_stream))
    except N.AxonError:
        _CUMSUM_WS.clear()
        raise


def adam(param, grad, exp_avg, exp_avg_sq, *, step_size=None, inv_bc2_sqrt=None, wd=None, beta1=0.9,
         beta2=0.999, eps=1e-8, out=None, tune=None):
    """L2-regularised Adam. step_size / inv_bc2_sqrt / wd are floats or
    per-row tensors [rows] / [rows, 1]. out = (param_out, m_out, v_out) or None
    for new tensors; pass the inputs themselves to update in place."""
    _require_cuda(param, grad, exp_avg, exp_avg_sq)
    for t in (param, grad, exp_avg, exp_avg_sq):
        if not t.is_contiguous() or t.shape != param.shape:
            raise N.AxonError(N.AXON_E_SHAPE, "adam: tensors must be contiguous and the same shape")
    if param.dtype != exp_avg.dtype or param.dtype != exp_avg_sq.dtype:
        raise N.AxonError(N.AXON_E_UNSUPPORTED, "adam: param/exp_avg/exp_avg_sq must share a dtype")
    rows = param.shape[0] if param.dim() >= 2 else 1
    cols = param.numel() // max(rows, 1) if param.numel() else 0
    if out is None:
        out = (torch.empty_like(param), torch.empty_like(exp_avg), torch.empty_like(exp_avg_sq))
    hp = AdamHParams(beta1, beta2, eps, 0.0, 1.0, 0.0)
    row_ptrs, row_dt = [], N.AXON_F32
    for name, v in (("step_size", step_size), ("inv_bc2_sqrt", inv_bc2_sqrt), ("wd", wd)):
        if isinstance(v, torch.Tensor):
            _require_cuda(v)
            if v.numel() != rows or not v.is_contiguous():
                raise N.AxonError(N.AXON_E_SHAPE, f"adam: per-row {name} must have {rows} elements")
            row_ptrs.append(_ptr(v))
            row_dt = dtype_code(v)
        else:
            setattr(hp, name, 0.0 if v is None else float(v))
            if name == "inv_bc2_sqrt" and v is None:
                hp.inv_bc2_sqrt = 1.0
            row_ptrs.append(None)
    check(N.lib().axon_adam(_ptr(param), _ptr(grad), _ptr(exp_avg), _ptr(exp_avg_sq), _ptr(out[0]), _ptr(out[1]),
                            _ptr(out[2]), rows, cols, dtype_code(param), dtype_code(grad), row_ptrs[0], row_ptrs[1],
                            row_ptrs[2], row_dt, ctypes.byref(hp), _tune(tune), _stream(param)))
    return out


def gemm(a, b, *, b2=None, row_scale=None, epilogue=N.AXON_EPI_NONE, out=None, out_dtype=None, tune=None):
    """C = epilogue(A @ B) on tcgen05; A [m, k], B (and B2) [k, n]."""
    _require_cuda(a, b, b2, row_scale)
    m, k, lda = _rows(a)
    kb, n, ldb = _rows(b)
    if kb != k:
        raise N.AxonError(N.AXON_E_SHAPE, f"gemm: inner dims differ ({k} vs {kb})")
    if b2 is not None and (b2.shape != b.shape or b2.stride() != b.stride()):
        raise N.AxonError(N.AXON_E_SHAPE, "gemm: b2 must match b's shape and strides")
    c = out if out is not None else torch.empty((m, n), dtype=out_dtype or a.dtype, device=a.device)
    _, _, ldc = _rows(c)
    check(N.lib().axon_gemm(_ptr(a), _ptr(b), _ptr(b2), _ptr(c), _ptr(row_scale), m, n, k, lda, ldb, ldc,
                            dtype_code(a), dtype_code(c), epilogue, _tune(tune), _stream(a)))
    return c


def cast(src, dtype, *, out=None):
    """Elementwise dtype conversion on the device (contiguous tensors)."""
    _require_cuda(src, out)
    if not src.is_contiguous():
        raise N.AxonError(N.AXON_E_SHAPE, "cast: source must be contiguous")
    dst = out if out is not None else torch.empty(src.shape, dtype=dtype, device=src.device)
    if dst.numel() != src.numel() or not dst.is_contiguous():
        raise N.AxonError(N.AXON_E_SHAPE, "cast: destination must be contiguous with as many elements")
    check(N.lib().axon_cast(_ptr(src), _ptr(dst), src.numel(), dtype_code(src), dtype_code(dst), _stream(src)))
    return dst


def row_status(device=None) -> None:
    check(N.lib().axon_row_status(torch.cuda.current_stream(device).cuda_stream))


def gemm_status(device=None) -> None:
    check(N.lib().axon_gemm_status(torch.cuda.current_stream(device).cuda_stream))


def row_rsqrt(x, *, scale=1.0, eps=0.0, out=None):
    _require_cuda(x)
    m, n, ldx = _rows(x)
    r = out if out is not None else torch.empty(m, dtype=torch.float32, device=x.device)
    check(N.lib().axon_row_rsqrt(_ptr(x), _ptr(r), m, n, ldx, dtype_code(x), float(scale), float(eps), _stream(x)))
    return r


def rmsnorm_matmul(x, w, *, out=None, out_dtype=None, workspace=None, tune=None):
    _require_cuda(x, w)
    m, k = x.shape
    n = w.shape[1]
    if not x.is_contiguous() or not w.is_contiguous():
        raise N.AxonError(N.AXON_E_SHAPE, "rmsnorm_matmul: x and w must be contiguous")
    y = out if out is not None else torch.empty((m, n), dtype=out_dtype or x.dtype, device=x.device)
    ws = workspace if workspace is not None else torch.empty(m, dtype=torch.float32, device=x.device)
    check(N.lib().axon_rmsnorm_matmul(_ptr(x), _ptr(w), _ptr(y), _ptr(ws), m, n, k, dtype_code(x), dtype_code(y),
                                      _tune(tune), _stream(x)))
    return y


def _workspace(nbytes: int, device, workspace=None) -> torch.Tensor:
    if workspace is not None:
        if workspace.numel() < nbytes:
            raise N.AxonError(N.AXON_E_ARG, f"workspace of {nbytes} bytes needed")
        return workspace
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _check_ws_bytes(nbytes: int) -> int:
    if nbytes < 0:
        check(int(nbytes))
    return int(nbytes)


def gemm_exp(a, b, *, row_part=None, out=None, out_dtype=None, tune=None):
    """C = exp(A @ B); with `row_part` (fp32 [tiles, m], tiles = ceil(n /
    block_n)) also each row's sum of the stored values per column tile."""
    _require_cuda(a, b, row_part)
    m, k, lda = _rows(a)
    kb, n, ldb = _rows(b)
    if kb != k:
        raise N.AxonError(N.AXON_E_SHAPE, f"gemm_exp: inner dims differ ({k} vs {kb})")
    c = out if out is not None else torch.empty((m, n), dtype=out_dtype or a.dtype, device=a.device)
    _, _, ldc = _rows(c)
    part_ld = row_part.stride(0) if row_part is not None else 0
    check(N.lib().axon_gemm_exp(_ptr(a), _ptr(b), _ptr(c), _ptr(row_part), part_ld, m, n, k, lda, ldb, ldc,
                                dtype_code(a), dtype_code(c), _tune(tune), _stream(a)))
    return c


def qkv_cte(x, mlp_prev, attention_prev, w, *, out=None, out_dtype=None, workspace=None, tune=None):
    """(h / sqrt(mean(h^2) + 1e-6)) @ w with h = x + mlp_prev + attention_prev:
    one kernel by default (tune variant 0); variants 1 / 2 run a row pass and
    the one-CTA / CTA-pair GEMM."""
    _require_cuda(x, mlp_prev, attention_prev, w)
    for t in (x, mlp_prev, attention_prev, w):
        if not t.is_contiguous():
            raise N.AxonError(N.AXON_E_SHAPE, "qkv_cte: tensors must be contiguous")
    m, k = x.shape
    n = w.shape[1]
    if mlp_prev.shape != x.shape or attention_prev.shape != x.shape or w.shape[0] != k:
        raise N.AxonError(N.AXON_E_SHAPE, "qkv_cte: x, mlp_prev, attention_prev [m, k] and w [k, n]")
    y = out if out is not None else torch.empty((m, n), dtype=out_dtype or x.dtype, device=x.device)
    ws = workspace
    nbytes = _check_ws_bytes(N.lib().axon_qkv_cte_workspace_bytes(m, n, k, _tune(tune)))
    if nbytes > 0:  # k-split partials (variant 0) or the staged h (variants 1, 2)
        ws = _workspace(nbytes, x.device, workspace)
    check(N.lib().axon_qkv_cte(_ptr(x), _ptr(mlp_prev), _ptr(attention_prev), _ptr(w), _ptr(y), _ptr(ws),
                               ws.numel() if ws is not None else 0, m, n, k, dtype_code(x), dtype_code(y),
                               _tune(tune), _stream(x)))
    return y


def softmax_mm(x, w, *, out=None, out_dtype=None, workspace=None, tune=None):
    """(exp(x) / sum(exp(x))) @ w, the bare exponential of the spec."""
    _require_cuda(x, w)
    if not x.is_contiguous() or not w.is_contiguous():
        raise N.AxonError(N.AXON_E_SHAPE, "softmax_mm: x and w must be contiguous")
    m, k = x.shape
    if w.shape[0] != k:
        raise N.AxonError(N.AXON_E_SHAPE, "softmax_mm: x [m, k] and w [k, n]")
    n = w.shape[1]
    y = out if out is not None else torch.empty((m, n), dtype=out_dtype or x.dtype, device=x.device)
    nbytes = _check_ws_bytes(N.lib().axon_softmax_mm_workspace_bytes(m, k))
    ws = _workspace(nbytes, x.device, workspace)
    check(N.lib().axon_softmax_mm(_ptr(x), _ptr(w), _ptr(y), _ptr(ws), ws.numel(), m, n, k, dtype_code(x),
                                  dtype_code(y), _tune(tune), _stream(x)))
    return y


def attention(q, k_t, v, *, out=None, out_dtype=None, workspace=None, tune=None):
    """softmax(q @ k_t) @ v (bare exponential), q [s, d], k_t [d, s], v [s, d]:
    one kernel by default for head dim 64 / 128 (tune variant 0), the
    exp-GEMM + row-scaled GEMM form as variant 1."""
    _require_cuda(q, k_t, v)
    for t in (q, k_t, v):
        if not t.is_contiguous():
            raise N.AxonError(N.AXON_E_SHAPE, "attention: tensors must be contiguous")
    s, d = q.shape
    if k_t.shape != (d, s) or v.shape != (s, d):
        raise N.AxonError(N.AXON_E_SHAPE, "attention: q [s, d], k_t [d, s], v [s, d]")
    y = out if out is not None else torch.empty((s, d), dtype=out_dtype or q.dtype, device=q.device)
    nbytes = _check_ws_bytes(N.lib().axon_attention_workspace_bytes(s, d, _tune(tune)))
    ws = _workspace(nbytes, q.device, workspace) if nbytes > 0 else workspace
    check(N.lib().axon_attention(_ptr(q), _ptr(k_t), _ptr(v), _ptr(y), _ptr(ws), ws.numel() if ws is not None else 0,
                                 s, d, dtype_code(q), dtype_code(y), _tune(tune), _stream(q)))
    return y


def silu_mlp_workspace_bytes(m: int, n: int, p: int, dtype_code_: int, tune=None) -> int:
    nbytes = int(N.lib().axon_silu_mlp_workspace_bytes(m, n, p, dtype_code_, _tune(tune)))
    if nbytes < 0:
        check(nbytes)
    return nbytes


def silu_mlp(x, w1, w2, w3, *, out=None, out_dtype=None, workspace=None, tune=None):
    """(silu(x @ w1) * (x @ w2)) @ w3. tune['precision'] picks how the
    activation is stored: 1 (default) x's dtype, 2/3 split terms, 4 f16."""
    _require_cuda(x, w1, w2, w3)
    for t in (x, w1, w2, w3):
        if not t.is_contiguous():
            raise N.AxonError(N.AXON_E_SHAPE, "silu_mlp: operands must be contiguous")
    m, k = x.shape
    n = w1.shape[1]
    p = w3.shape[1]
    y = out if out is not None else torch.empty((m, p), dtype=out_dtype or x.dtype, device=x.device)
    need = silu_mlp_workspace_bytes(m, n, p, dtype_code(x), tune)
    ws = workspace if workspace is not None else torch.empty(need, dtype=torch.uint8, device=x.device)
    check(N.lib().axon_silu_mlp(_ptr(x), _ptr(w1), _ptr(w2), _ptr(w3), _ptr(y), _ptr(ws), ws.numel() * ws.element_size(),
                                m, n, k, p, dtype_code(x), dtype_code(y), _tune(tune), _stream(x)))
    return y
