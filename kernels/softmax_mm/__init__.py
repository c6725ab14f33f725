"""Spec package `softmax_mm`: `softmax(x) @ w` with a bare exponential.

Same contract as Axon's kernels/softmax_mm/__init__.py:15-27; no
`torch_ref`, so `baseline_op` is the oracle.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_softmax_matmul
from .refs import baseline_op, make_inputs

SPEC = KernelSpec(
    name="softmax_mm",
    axon_kernel=kernel_softmax_matmul,
    dim_vars=("m", "n", "k"),
    input_specs=(("x", ("m", "k")), ("w", ("k", "n"))),
    baseline_op=baseline_op,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N", "TILES_IN_BLOCK_K"),
    tile_options=(1, 2, 4, 8, 16),
)
