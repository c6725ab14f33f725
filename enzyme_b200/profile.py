"""Single-launch cases for Nsight Compute captures of the library's kernels.

    python -m enzyme_b200.profile CASE [--launches N]

Each case builds seeded inputs on cuda:0, sized so that every launch streams
from HBM (inputs past the 126 MB L2 where the kernel streams) while the
device holds a few GB at most, then runs the case's call N times (default 2:
one warm launch and one to capture, e.g. `ncu -k regex:<kernel> -s 1 -c 1`).
The capture commands and the figures taken from them are in profiles/*.md.
The kernel each case launches is listed in CASES; `--list` prints them.
"""

from __future__ import annotations

import argparse
import math
import sys

import torch


def _randn(*shape, dtype=torch.bfloat16, scale=1.0, gen=None):
    return (scale * torch.randn(*shape, device="cuda", generator=gen)).to(dtype)


def case_adam(gen):
    """adam_vec: 64 Mi fp32 parameters, bf16 grads (0.9 GB streamed)."""
    from . import ops

    n = 64 << 20
    p, g = _randn(n, dtype=torch.float32, scale=0.02, gen=gen), _randn(n, scale=1e-3, gen=gen)
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    ss, ib = 3e-4 / (1 - 0.9 ** 10), 1 / math.sqrt(1 - 0.95 ** 10)
    return lambda: ops.adam(p, g, m, v, step_size=ss, inv_bc2_sqrt=ib, wd=0.1, beta1=0.9, beta2=0.95,
                            out=(p, m, v))


def case_cast(gen):
    """cast_vec: bf16 -> f16 of a [28672, 4096] matrix (two W_down shards)."""
    from . import ops

    w = _randn(28672, 4096, scale=0.02, gen=gen)
    out = torch.empty(w.shape, dtype=torch.float16, device="cuda")
    return lambda: ops.cast(w, torch.float16, out=out)


def _cumsum_rows(gen):
    logits = 2.0 * torch.randn(256, 128256, device="cuda", generator=gen)
    return torch.sort(torch.softmax(logits, dim=1), dim=1, descending=True).values.contiguous()


def case_cumsum_lookback(gen):
    """cumsum_lookback: the nucleus config (256 x 128256 fp32) by the
    decoupled look-back scan (variant 0, 16384-element tiles)."""
    from . import ops

    x = _cumsum_rows(gen)
    y = torch.empty_like(x)
    tune = {"variant": 0, "split": 16384}
    ws = torch.zeros(ops.cumsum_workspace_bytes(256, 128256, tune), dtype=torch.uint8, device="cuda")
    return lambda: ops.cumsum(x, out=y, workspace=ws, tune=tune)


def case_cumsum_balanced(gen):
    """cumsum_balanced: the nucleus config by balanced chunk ranges (variant 3)."""
    from . import ops

    x = _cumsum_rows(gen)
    y = torch.empty_like(x)
    tune = {"variant": 3}
    ws = torch.zeros(ops.cumsum_workspace_bytes(256, 128256, tune), dtype=torch.uint8, device="cuda")
    return lambda: ops.cumsum(x, out=y, workspace=ws, tune=tune)


def case_rope_split(gen):
    """rope_split_vec: the rope spec's layout, four [64, 2 Mi] bf16 inputs."""
    from . import ops

    shape = (64, 2 << 20)
    xe, xo, c, s = (_randn(*shape, gen=gen) for _ in range(4))
    oe, oo = torch.empty_like(xe), torch.empty_like(xo)
    return lambda: ops.rope_split(xe, xo, c, s, out_even=oe, out_odd=oo)


def case_softmax_mm(gen):
    """row_prologue_kernel (the exp row pass) and the row-scaled GEMM of
    softmax_mm at m = n = k = 4096."""
    from . import ops

    x, w = _randn(4096, 4096, gen=gen), _randn(4096, 4096, gen=gen)
    y = torch.empty(4096, 4096, dtype=torch.bfloat16, device="cuda")
    return lambda: ops.softmax_mm(x, w, out=y)


def case_qkv_split(gen):
    """gemm_resid3 with a k split and its resid3_reduce_kernel: qkv_cte at
    m 1024, n 512, k 8192 (eight row tiles, so k is split 18 ways)."""
    from . import ops

    ins = [_randn(1024, 8192, gen=gen) for _ in range(3)]
    w = _randn(8192, 512, scale=1 / 8192 ** 0.5, gen=gen)
    y = torch.empty(1024, 512, dtype=torch.bfloat16, device="cuda")
    return lambda: ops.qkv_cte(*ins, w, out=y)


def case_attention(gen):
    """attn_fused and attn_reduce_kernel: attention_nkilib s 8192, d 128."""
    from . import ops

    q = torch.rand(8192, 128, device="cuda", generator=gen).bfloat16()
    kt = torch.rand(128, 8192, device="cuda", generator=gen).bfloat16()
    v = torch.rand(8192, 128, device="cuda", generator=gen).bfloat16()
    y = torch.empty(8192, 128, dtype=torch.bfloat16, device="cuda")
    return lambda: ops.attention(q, kt, v, out=y)


def case_attention_two_gemm(gen):
    """recip_sum_kernel and the exp-epilogue GEMM: attention variant 1 at
    s 8192, d 128."""
    from . import ops

    q = torch.rand(8192, 128, device="cuda", generator=gen).bfloat16()
    kt = torch.rand(128, 8192, device="cuda", generator=gen).bfloat16()
    v = torch.rand(8192, 128, device="cuda", generator=gen).bfloat16()
    y = torch.empty(8192, 128, dtype=torch.bfloat16, device="cuda")
    return lambda: ops.attention(q, kt, v, out=y, tune={"variant": 1})


def case_rmsnorm_matmul(gen):
    """row_bulk_kernel (rsqrt of the row sums of squares) and the row-scaled
    tcgen05 GEMM of rmsnorm_matmul at m 1024, n 8192, k 8192."""
    from . import ops

    x, w = _randn(1024, 8192, gen=gen), _randn(8192, 8192, gen=gen)
    y = torch.empty(1024, 8192, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(4 * 1024, dtype=torch.uint8, device="cuda")
    return lambda: ops.rmsnorm_matmul(x, w, out=y, workspace=ws)


def case_softmax_long(gen):
    """row_streaming_kernel: softmax of 1024 fp32 rows of 65536 (256 KB:
    past the bulk kernel's 32 KB rows and one CTA's registers)."""
    from . import ops

    x = torch.randn(1024, 65536, device="cuda", generator=gen)
    y = torch.empty_like(x)
    return lambda: ops.softmax(x, out=y)


def case_softmax_cta(gen):
    """row_cta_bulk_kernel: softmax of 2048 fp32 rows of 32768 (128 KB rows
    staged in shared memory in 16 KB chunks; 512 MB streamed)."""
    from . import ops

    x = torch.randn(2048, 32768, device="cuda", generator=gen)
    y = torch.empty_like(x)
    return lambda: ops.softmax(x, out=y)


def _tp_shard(gen, inter):
    h = 4096
    x = _randn(4096, h, gen=gen)
    return x, _randn(h, inter, scale=0.02, gen=gen), _randn(h, inter, scale=0.02, gen=gen), \
        _randn(inter, h, scale=0.02, gen=gen)


def case_tp_slabs(gen):
    """The tensor-parallel step's separate launches on one rank (world 1, the
    4-rank shard: inter 3584): the SiLU-gate GEMM, the down GEMM whose
    epilogue writes f16 partial rows to the owner's inbox
    (gemm_tcgen05_pair<..., 7, ...>), tp_signal_kernel, tp_reduce_push_kernel
    and tp_wait_kernel. With one rank the inbox and the output are local:
    the kernels' instruction mix and DRAM traffic, not NVLink's."""
    from .tp import FusedTPSwiGLU

    x, w1, w2, w3 = _tp_shard(gen, 3584)
    f = FusedTPSwiGLU(w1, w2, w3, m=4096, slabs=2)
    return lambda: f.forward(x)


def case_tp_step(gen):
    """swiglu_fused_pair<__half, 2>: the whole tensor-parallel step in one
    kernel on one rank (world 1, inter 3584): GEMM tiles beside the
    reduction warps."""
    from .tp import FusedTPSwiGLU

    x, w1, w2, w3 = _tp_shard(gen, 3584)
    f = FusedTPSwiGLU(w1, w2, w3, m=4096, whole_step=True)
    return lambda: f.forward(x)


CASES = {
    "adam": (case_adam, "adam_vec"),
    "cast": (case_cast, "cast_vec"),
    "cumsum_lookback": (case_cumsum_lookback, "cumsum_lookback"),
    "cumsum_balanced": (case_cumsum_balanced, "cumsum_balanced"),
    "rope_split": (case_rope_split, "rope_split_vec"),
    "softmax_mm": (case_softmax_mm, "row_prologue_kernel"),
    "qkv_split": (case_qkv_split, "resid3_reduce_kernel"),
    "attention": (case_attention, "attn_reduce_kernel"),
    "attention_two_gemm": (case_attention_two_gemm, "recip_sum_kernel"),
    "rmsnorm_matmul": (case_rmsnorm_matmul, "gemm_tcgen05"),
    "softmax_long": (case_softmax_long, "row_streaming_kernel"),
    "softmax_cta": (case_softmax_cta, "row_cta_bulk_kernel"),
    "tp_slabs": (case_tp_slabs, "tp_reduce_push_kernel"),
    "tp_step": (case_tp_step, "swiglu_fused_pair"),
}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("case", nargs="?", choices=sorted(CASES))
    ap.add_argument("--launches", type=int, default=2)
    ap.add_argument("--list", action="store_true")
    args = ap.parse_args(argv)
    if args.list or args.case is None:
        for name, (fn, kernel) in CASES.items():
            print(f"{name:20s} {kernel:24s} {fn.__doc__.splitlines()[0]}")
        return 0
    from . import ops

    torch.cuda.set_device(0)
    gen = torch.Generator(device="cuda").manual_seed(42)
    run = CASES[args.case][0](gen)
    torch.cuda.synchronize()
    for _ in range(args.launches):
        run()
    torch.cuda.synchronize()
    ops.gemm_status()
    ops.row_status()
    print(f"profile case {args.case}: {args.launches} launches ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
