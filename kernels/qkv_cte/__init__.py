"""Spec package `qkv_cte`: residual add, mean-RMS norm, fused QKV projection.

Same contract as Axon's kernels/qkv_cte/__init__.py:23-37 (dims m, n, k;
x, mlp_prev, attention_prev [m, k], w [k, n]).
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_qkv_cte
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="qkv_cte",
    axon_kernel=kernel_qkv_cte,
    dim_vars=("m", "n", "k"),
    input_specs=(
        ("x", ("m", "k")),
        ("mlp_prev", ("m", "k")),
        ("attention_prev", ("m", "k")),
        ("w", ("k", "n")),
    ),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N", "TILES_IN_BLOCK_K"),
)
