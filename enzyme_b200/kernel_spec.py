"""The kernel-spec contract every `kernels/<name>/` package fills in.

Same fields, order and validation as Axon's `KernelSpec`
(src/axon/kernel_spec.py:11-43): a spec names its ordered `dim_vars` (the
`--sizes` positions and CSV dim columns), its symbolic `input_specs`, a seeded
`make_inputs(*, <dims>, dtype, rng)`, its tile knob names, and the CPU
references (`baseline_op` numpy, `torch_ref` torch) the bench checks against.
`SEED` is the shared input seed (src/axon/kernel_spec.py:8).

`baseline_compiler_args` is kept for signature compatibility with Axon specs;
the CUDA backend compiles ahead of time and never reads it.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any

SEED = 42


@dataclass(frozen=True, slots=True)
class KernelSpec:
    name: str
    axon_kernel: Callable[..., Any]
    dim_vars: tuple[str, ...]
    input_specs: Sequence[tuple[str, tuple[str | int, ...]]]
    make_inputs: Callable[..., tuple[Any, ...]]
    tile_args: Sequence[str]
    baseline_op: Callable[..., Any] | None = None
    torch_ref: Callable[..., Any] | None = None
    baseline_compiler_args: str = "--model-type=transformer"
    tile_options: Sequence[int] = (1, 2, 4, 8, 16, 32)

    def __post_init__(self) -> None:
        if len(set(self.dim_vars)) != len(self.dim_vars):
            raise ValueError(
                f"kernel '{self.name}': dim_vars has duplicate names: {self.dim_vars}"
            )
        used = {
            label
            for _, shape in self.input_specs
            for label in shape
            if isinstance(label, str)
        }
        if set(self.dim_vars) != used:
            raise ValueError(
                f"kernel '{self.name}': dim_vars {set(self.dim_vars)} does not "
                f"match input_specs labels {used}"
            )

    def input_names(self) -> list[str]:
        return [name for name, _ in self.input_specs]

    def concrete_shapes(self, dim_sizes: dict[str, int]) -> list[tuple[int, ...]]:
        """Bind each input's symbolic shape to the given dim sizes."""
        return [
            tuple(dim_sizes[d] if isinstance(d, str) else int(d) for d in shape)
            for _, shape in self.input_specs
        ]
