"""Spec package `softmax`: row softmax `exp(x) / sum(exp(x))`.

Same contract as Axon's kernels/softmax/__init__.py:15-22. Like the
reference it has no `torch_ref`; `baseline_op` is the oracle.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_softmax
from .refs import baseline_op, make_inputs

SPEC = KernelSpec(
    name="softmax",
    axon_kernel=kernel_softmax,
    dim_vars=("m", "n"),
    input_specs=(("x", ("m", "n")),),
    baseline_op=baseline_op,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"),
)
