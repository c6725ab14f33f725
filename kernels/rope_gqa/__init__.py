"""Spec package `rope_gqa`: the BASELINE rope config (Llama-3-8B GQA shape).

q [s, hq, 128] and k [s, hkv, 128] bf16 in rotate-half layout; fp32 cos/sin
tables [s, 64] for positions 0..s-1 and theta 500000. The head dim is written
as (2, half_d) so that `x1 = x[..., 0, :]` and `x2 = x[..., 1, :]` are the two
halves of the same contiguous [s, h, 128] memory; every symbolic label is then
a dim var, as KernelSpec requires. Outputs: (q_rot, k_rot).

The pointwise math is the reference spec's (Axon kernels/rope/kernel.py:34-35):
`out1 = x1*cos - x2*sin`, `out2 = x2*cos + x1*sin`.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_rope_gqa
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="rope_gqa",
    axon_kernel=kernel_rope_gqa,
    dim_vars=("s", "hq", "hkv", "half_d"),
    input_specs=(
        ("q", ("s", "hq", 2, "half_d")),
        ("k", ("s", "hkv", 2, "half_d")),
        ("cos", ("s", "half_d")),
        ("sin", ("s", "half_d")),
    ),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"),
)
