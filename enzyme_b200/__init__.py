"""Axon B200 backend: hand-written sm_100a CUDA kernels behind a C ABI, driven
by Axon's kernel-spec API, CLI and per-variant CSV bench contract.

* `enzyme_b200.kernel_spec` -- the `KernelSpec` contract of the spec packages.
* `enzyme_b200.ops`         -- torch-facing wrappers over `libaxon_b200.so`.
* `enzyme_b200.cli`         -- the `axon kernels/<name> --sizes ...` command.
"""

from .kernel_spec import SEED, KernelSpec

__all__ = ["SEED", "KernelSpec"]
__version__ = "0.1.0"
