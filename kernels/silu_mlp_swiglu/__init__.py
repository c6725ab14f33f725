"""Spec package `silu_mlp_swiglu`: the BASELINE SwiGLU config.

Same math and dims as `silu_mlp` (Axon kernels/silu_mlp/kernel.py:7-14;
x (m, k), w1 = W_gate and w2 = W_up (k, n), w3 = W_down (n, p)), with weights
drawn from N(0, 0.02) as the config asks (m=4096, hidden 4096, inter 14336).
It adds an fp32 `torch_ref`.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_swiglu
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="silu_mlp_swiglu",
    axon_kernel=kernel_swiglu,
    dim_vars=("m", "n", "k", "p"),
    input_specs=(
        ("x", ("m", "k")),
        ("w1", ("k", "n")),
        ("w2", ("k", "n")),
        ("w3", ("n", "p")),
    ),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=(
        "TILES_IN_BLOCK_M",
        "TILES_IN_BLOCK_N",
        "TILES_IN_BLOCK_K",
        "TILES_IN_BLOCK_P",
    ),
)
