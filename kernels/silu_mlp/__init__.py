"""Spec package `silu_mlp`: `(silu(x @ w1) * (x @ w2)) @ w3`.

Same contract as Axon's kernels/silu_mlp/__init__.py:16-34 (dims m, n, k, p:
x (m, k), w1/w2 (k, n), w3 (n, p)); like the reference it has no
`torch_ref`. The BASELINE SwiGLU config (weights ~ N(0, 0.02)) is the
sibling `silu_mlp_swiglu`.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_silu_mlp_full
from .refs import baseline_op, make_inputs

SPEC = KernelSpec(
    name="silu_mlp",
    axon_kernel=kernel_silu_mlp_full,
    dim_vars=("m", "n", "k", "p"),
    input_specs=(
        ("x", ("m", "k")),
        ("w1", ("k", "n")),
        ("w2", ("k", "n")),
        ("w3", ("n", "p")),
    ),
    baseline_op=baseline_op,
    make_inputs=make_inputs,
    tile_args=(
        "TILES_IN_BLOCK_M",
        "TILES_IN_BLOCK_N",
        "TILES_IN_BLOCK_K",
        "TILES_IN_BLOCK_P",
    ),
)
