"""Spec package `layernorm`: bare LayerNorm over the last axis, no affine.

Same contract as Axon's kernels/layernorm/__init__.py:16-25.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_layernorm
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="layernorm",
    axon_kernel=kernel_layernorm,
    dim_vars=("m", "n"),
    input_specs=(("x", ("m", "n")),),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"),
)
