"""Spec package `rmsnorm`: sum-based RMS normalisation, `x / sqrt(sum(x^2))`.

Same contract as Axon's kernels/rmsnorm/__init__.py:15-24 (dims (m, n), one
input `x`, no eps, no weight). The BASELINE config form with a mean, an eps
and a weight lives in the sibling package `rmsnorm_llama`.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_rmsnorm
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="rmsnorm",
    axon_kernel=kernel_rmsnorm,
    dim_vars=("m", "n"),
    input_specs=(("x", ("m", "n")),),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"),
)
