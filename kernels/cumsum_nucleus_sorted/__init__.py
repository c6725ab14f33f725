"""Spec package `cumsum_nucleus_sorted`: the BASELINE cumsum config.

Rows are softmax(N(0, 2) logits) sorted descending (the nucleus-sampling
CDF), 256 x 128256 fp32; inclusive prefix sum along the vocab axis, checked
at rel 1e-5 against float64. Same math as Axon kernels/cumsum/kernel.py:12-13.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_cumsum_sorted
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="cumsum_nucleus_sorted",
    axon_kernel=kernel_cumsum_sorted,
    dim_vars=("m", "n"),
    input_specs=(("x", ("m", "n")),),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"),
)
