"""Spec package `rmsnorm_matmul`: `(x / sqrt(sum(x^2))) @ w`.

Same contract as Axon's kernels/rmsnorm_matmul/__init__.py:15-26; no
`torch_ref`, so `baseline_op` is the oracle.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_rmsnorm_matmul
from .refs import baseline_op, make_inputs

SPEC = KernelSpec(
    name="rmsnorm_matmul",
    axon_kernel=kernel_rmsnorm_matmul,
    dim_vars=("m", "n", "k"),
    input_specs=(("x", ("m", "k")), ("w", ("k", "n"))),
    baseline_op=baseline_op,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N", "TILES_IN_BLOCK_K"),
)
