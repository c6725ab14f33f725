"""Spec packages: every hot-path spec loads with the KernelSpec contract."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import KERNELS, load_spec
from enzyme_b200.kernel_spec import SEED, KernelSpec
from enzyme_b200.specs import SpecLoadError, install_axon_alias, safe_name
from enzyme_b200.specs import load_spec as load_path

SPECS = sorted(p.name for p in KERNELS.iterdir() if (p / "__init__.py").is_file())
REFERENCE_SPECS = {"rmsnorm", "layernorm", "rope", "softmax", "cumsum", "fused_adam", "matmul", "silu_mlp",
                   "rmsnorm_matmul"}
CONFIG_SPECS = {"rmsnorm_llama", "rope_gqa", "cumsum_nucleus_sorted", "silu_mlp_swiglu", "fused_adam_cfg"}


def test_all_specs_present():
    assert REFERENCE_SPECS | CONFIG_SPECS <= set(SPECS)


@pytest.mark.parametrize("name", SPECS)
def test_spec_loads_and_validates(name):
    spec = load_spec(name)
    assert isinstance(spec, KernelSpec)
    assert spec.name == name
    assert spec.baseline_op is not None
    labels = {d for _, shape in spec.input_specs for d in shape if isinstance(d, str)}
    assert labels == set(spec.dim_vars)


@pytest.mark.parametrize("name", SPECS)
def test_make_inputs_shapes(name):
    spec = load_spec(name)
    dims = {d: 16 if d not in ("half_d",) else 8 for d in spec.dim_vars}
    ins = spec.make_inputs(**dims, rng=np.random.default_rng(SEED))
    assert [tuple(np.asarray(a).shape) for a in ins] == spec.concrete_shapes(dims)


def test_kernel_spec_rejects_label_mismatch():
    with pytest.raises(ValueError, match="does not match"):
        KernelSpec(name="bad", axon_kernel=lambda x: x, dim_vars=("m",), input_specs=(("x", ("m", "n")),),
                   make_inputs=lambda **_: (), tile_args=())
    with pytest.raises(ValueError, match="duplicate"):
        KernelSpec(name="bad", axon_kernel=lambda x: x, dim_vars=("m", "m"), input_specs=(("x", ("m",)),),
                   make_inputs=lambda **_: (), tile_args=())


def test_safe_name_rule():
    assert safe_name("rmsnorm") == "rmsnorm"
    assert safe_name("a-b.c/d") == "a_b_c_d"
    assert safe_name("_9x") == "v9x"


def test_load_errors(tmp_path):
    with pytest.raises(SpecLoadError):
        load_path(tmp_path / "missing")
    (tmp_path / "nospec").mkdir()
    with pytest.raises(SpecLoadError):
        load_path(tmp_path / "nospec")


def test_reference_style_spec_package_loads(tmp_path):
    """An unmodified Axon-style package (imports `axon`) loads via the alias."""
    pkg = tmp_path / "double"
    pkg.mkdir()
    (pkg / "__init__.py").write_text(
        "from axon.kernel_spec import KernelSpec\n"
        "from axon import AxonArray\n"
        "import numpy as np\n"
        "def k(x: AxonArray):\n    return x * 2.0\n"
        "def make_inputs(*, m, n, dtype=np.float32, rng):\n"
        "    return (rng.standard_normal((m, n)).astype(dtype),)\n"
        "SPEC = KernelSpec(name='double', axon_kernel=k, dim_vars=('m','n'), input_specs=(('x',('m','n')),),\n"
        "                  make_inputs=make_inputs, tile_args=('TILES_IN_BLOCK_M',), baseline_op=lambda x: 2*x)\n"
    )
    install_axon_alias()
    spec = load_path(pkg)
    assert spec.name == "double"


def test_cluster_scan_keys_fit_shared_memory():
    """cumsum variant 1 stages a row slice of a multiple of 8 elements per CTA
    in at most 200 KB: the nucleus rows (128256 fp32) need 4 or 8 CTAs."""
    from enzyme_b200 import catalogue

    cons = catalogue.constraints("cumsum_nucleus_sorted", 1, {"m": 256, "n": 128256}, 4,
                                 ("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"))
    assert cons[0].allowed == (4, 8)
    cons = catalogue.constraints("cumsum", 1, {"m": 8, "n": 1000}, 4, ("TILES_IN_BLOCK_M", "TILES_IN_BLOCK_N"))
    assert cons[0].allowed == (1, 2, 4, 8)


def test_profile_cases_list_without_a_gpu(capsys):
    from enzyme_b200 import profile

    assert profile.main(["--list"]) == 0
    out = capsys.readouterr().out
    for name in profile.CASES:
        assert name in out
