"""Spec package `matmul`: `x @ w` with x (m, k) and w (k, n).

Same contract as Axon's kernels/matmul/__init__.py:15-27.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_matmul
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="matmul",
    axon_kernel=kernel_matmul,
    dim_vars=("m", "n", "k"),
    input_specs=(("x", ("m", "k")), ("w", ("k", "n"))),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N", "TILES_IN_BLOCK_K"),
)
