"""Spec package `cumsum`: inclusive prefix sum along the last axis.

Same contract as Axon's kernels/cumsum/__init__.py:15-24. The nucleus-sampling
config (sorted softmax rows) is the sibling `cumsum_nucleus_sorted`.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_cumsum
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="cumsum",
    axon_kernel=kernel_cumsum,
    dim_vars=("m", "n"),
    input_specs=(("x", ("m", "n")),),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"),
)
