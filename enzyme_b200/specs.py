"""Spec loading: import a `kernels/<name>/` package (or a single-file spec) by
path and return its `SPEC`, as Axon's `_load_spec` does (src/axon/cli.py:100-135).

Reference spec packages import `axon.kernel_spec` and `axon`; `install_axon_alias`
maps those module names onto this package so an unmodified Axon spec package
loads here too.
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

from .kernel_spec import KernelSpec


def safe_name(node_id: str) -> str:
    """Axon's identifier rule for module and function names (src/axon/codegen/ops.py:57-62)."""
    result = node_id.replace("-", "_").replace(".", "_").replace("/", "_").lstrip("_")
    if not result or result[0].isdigit():
        result = "v" + result
    return result


def install_axon_alias() -> None:
    """Make `import axon`, `from axon import AxonArray` and
    `from axon.kernel_spec import KernelSpec` resolve to this package."""
    if "axon.kernel_spec" in sys.modules:
        return
    from . import ir, kernel_spec

    mod = types.ModuleType("axon")
    mod.AxonArray = ir.AxonArray
    mod.kernel_spec = kernel_spec
    mod.__path__ = []  # a package, so `axon.kernel_spec` imports resolve
    sys.modules.setdefault("axon", mod)
    sys.modules.setdefault("axon.kernel_spec", kernel_spec)


class SpecLoadError(ValueError):
    pass


def load_spec(path: str | Path) -> KernelSpec:
    """Load `SPEC` from a spec package directory or a single .py file."""
    p = Path(path).expanduser().resolve()
    install_axon_alias()
    if p.is_dir():
        init = p / "__init__.py"
        if not init.is_file():
            raise SpecLoadError(f"kernel-spec dir has no __init__.py: {p}")
        module_name = f"_axon_kernel_spec_{safe_name(p.name)}"
        target, search = init, [str(p)]
    elif p.is_file():
        module_name = f"_axon_kernel_spec_{safe_name(p.stem)}"
        target, search = p, None
    else:
        raise SpecLoadError(f"kernel-spec file not found: {p}")
    spec = importlib.util.spec_from_file_location(module_name, target, submodule_search_locations=search)
    if spec is None or spec.loader is None:
        raise SpecLoadError(f"could not load kernel-spec from {p}")
    module = importlib.util.module_from_spec(spec)
    sys.modules[module_name] = module
    spec.loader.exec_module(module)
    obj = getattr(module, "SPEC", None)
    if not isinstance(obj, KernelSpec) and type(obj).__name__ != "KernelSpec":
        raise SpecLoadError(f"{p} does not define a top-level `SPEC: KernelSpec`")
    return obj
