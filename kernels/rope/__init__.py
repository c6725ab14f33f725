"""Spec package `rope`: pointwise rotary embedding on pre-split halves.

Same contract as Axon's kernels/rope/__init__.py:15-33: four (half_d, free)
inputs, two outputs. The Llama-3 GQA config (q/k in rotate-half layout with
fp32 tables) is the sibling `rope_gqa`.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_rope
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="rope",
    axon_kernel=kernel_rope,
    dim_vars=("half_d", "free"),
    input_specs=(
        ("x_even", ("half_d", "free")),
        ("x_odd", ("half_d", "free")),
        ("cos", ("half_d", "free")),
        ("sin", ("half_d", "free")),
    ),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"),
)
