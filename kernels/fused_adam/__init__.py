"""Spec package `fused_adam`: L2-regularised Adam (no AMSGrad), three outputs.

Same contract as Axon's kernels/fused_adam/__init__.py:27-48: four (p, f)
tensors and three (p, 1) per-row scalars (step_size, inv_bc2_sqrt, wd).
The BASELINE config (fp32 state, bf16 grads, betas (0.9, 0.95)) is the
sibling `fused_adam_cfg`.
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_fused_adam
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="fused_adam",
    axon_kernel=kernel_fused_adam,
    dim_vars=("p", "f"),
    input_specs=(
        ("param", ("p", "f")),
        ("grad", ("p", "f")),
        ("exp_avg", ("p", "f")),
        ("exp_avg_sq", ("p", "f")),
        ("step_size", ("p", 1)),
        ("inv_bc2_sqrt", ("p", 1)),
        ("wd", ("p", 1)),
    ),
    baseline_op=baseline_op,
    torch_ref=torch_ref,
    make_inputs=make_inputs,
    tile_args=("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"),
)
