"""Spec package `rmsnorm_llama`: the BASELINE rmsnorm config,
`x * rsqrt(mean(x^2) + 1e-6) * w`, computed in fp32.

A sibling of `rmsnorm` with the same KernelSpec contract; it exists because
the reference spec (Axon kernels/rmsnorm/kernel.py:13-20) fixes the sum form
with no eps and no weight, while the north-star config asks for Llama's form
(x [2048, 4096] bf16 ~ N(0, 1), weight [4096] bf16 ~ N(1, 0.1), eps 1e-6).
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_rmsnorm_llama
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="rmsnorm_llama",
    axon_kernel=kernel_rmsnorm_llama,
    dim_vars=("m", "n"),
    input_specs=(("x", ("m", "n")), ("w", ("n",))),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"),
)
