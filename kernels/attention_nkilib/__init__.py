"""Spec package `attention_nkilib`: `softmax(q @ k_t) @ v` with q, the
pre-transposed k_t and v as inputs (a bare exponential, no row max).

Same contract as Axon's kernels/attention_nkilib/__init__.py:22-43 (dims s, d;
four canonical tile args).
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_attention_nkilib
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="attention_nkilib",
    axon_kernel=kernel_attention_nkilib,
    dim_vars=("s", "d"),
    input_specs=(
        ("q", ("s", "d")),
        ("k_t", ("d", "s")),
        ("v", ("s", "d")),
    ),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N", "TILES_IN_BLOCK_K", "TILES_IN_BLOCK_P"),
    tile_options=(1, 2, 4, 8, 16),
)
