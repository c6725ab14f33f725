"""Spec package `fused_adam_cfg`: the BASELINE Adam config.

fp32 params ~ N(0, 0.02), bf16 grads ~ N(0, 1e-3), fp32 exp_avg/exp_avg_sq
starting at zero, lr 3e-4, betas (0.9, 0.95), eps 1e-8, wd 0.1 at step 10.
The update rule is the reference spec's L2-regularised Adam (Axon
kernels/fused_adam/kernel.py:36-45) with beta2 = 0.95 instead of the spec's
fixed 0.999; the per-row scalars carry step_size = lr / (1 - beta1**step) and
inv_bc2_sqrt = 1 / sqrt(1 - beta2**step).
"""

from enzyme_b200.kernel_spec import KernelSpec

from .kernel import kernel_adam_cfg
from .refs import baseline_op, make_inputs, torch_ref

SPEC = KernelSpec(
    name="fused_adam_cfg",
    axon_kernel=kernel_adam_cfg,
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
