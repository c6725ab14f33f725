"""Pin the CPU oracle and the spec packages to the reference's own outputs.

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py
from the reference's `kernels/<name>/refs.py` (seeded `make_inputs`,
`baseline_op` on fp32 inputs, `torch_ref`). These tests need no GPU.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_cases, load_golden, load_spec
from enzyme_b200 import ir
from enzyme_b200.kernel_spec import SEED
from oracle import f64

CASES = golden_cases()

# baseline_op ran in fp32; the oracle is float64: agreement is fp32 rounding.
ORACLE_TOL = {"rtol": 2e-4, "atol": 2e-5}


def _scale(outs):
    return max(1.0, max(float(np.abs(o).max()) for o in outs))


def test_fixtures_present():
    assert len(CASES) >= 17


@pytest.mark.parametrize("case", CASES)
def test_make_inputs_reproduces_reference_draws(case):
    spec_name, dims, inputs, _, _ = load_golden(case)
    spec = load_spec(spec_name)
    dtype = np.asarray(inputs[0]).dtype
    ours = spec.make_inputs(**dims, dtype=dtype, rng=np.random.default_rng(SEED))
    assert len(ours) == len(inputs)
    for a, b in zip(ours, inputs):
        a, b = np.asarray(a), np.asarray(b)
        assert a.dtype == b.dtype and a.shape == b.shape
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), "seeded inputs differ bit-wise"


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_baseline(case):
    spec_name, _, inputs, outs, _ = load_golden(case)
    got = f64.evaluate(spec_name, *inputs)
    assert len(got) == len(outs)
    s = _scale(outs)
    for g, o in zip(got, outs):
        np.testing.assert_allclose(g, o.astype(np.float64), rtol=ORACLE_TOL["rtol"], atol=ORACLE_TOL["atol"] * s)


@pytest.mark.parametrize("case", CASES)
def test_spec_refs_match_reference(case):
    spec_name, _, inputs, outs, rec = load_golden(case)
    spec = load_spec(spec_name)
    f32 = [np.asarray(a, dtype=np.float32) for a in inputs]
    base = spec.baseline_op(*f32)
    base = base if isinstance(base, tuple) else (base,)
    s = _scale(outs)
    for b, o in zip(base, outs):
        np.testing.assert_allclose(np.asarray(b, np.float32), o, rtol=1e-5, atol=1e-6 * s)
    if spec.torch_ref is not None:
        t = spec.torch_ref(*[torch.from_numpy(a.copy()) for a in f32])
        t = t if isinstance(t, tuple) else (t,)
        for a, o in zip(t, outs):
            np.testing.assert_allclose(a.numpy(), o, rtol=1e-4, atol=1e-5 * s)
        assert float(rec["torch_vs_baseline"]) <= 1e-3 * s


@pytest.mark.parametrize("case", CASES)
def test_axon_kernel_math_matches_reference(case):
    spec_name, _, inputs, outs, _ = load_golden(case)
    spec = load_spec(spec_name)
    got = ir.evaluate(spec.axon_kernel, *inputs)
    s = _scale(outs)
    for g, o in zip(got, outs):
        np.testing.assert_allclose(g, o.astype(np.float64), rtol=ORACLE_TOL["rtol"], atol=ORACLE_TOL["atol"] * s)


def test_rope_gqa_oracle_agrees_with_reference_rope():
    """The BASELINE rope layout reuses the reference's pointwise rotation: the
    rotate-half oracle on [s, h, 2, half] data equals the reference rope's
    baseline outputs when the halves are laid out as (half_d, free)."""
    _, dims, (xe, xo, c, s), outs, _ = load_golden("rope_small")
    half, free = xe.shape
    x = np.stack([xe.T, xo.T], axis=1).astype(np.float64)[:, None]  # [free, 1, 2, half]
    # rotate-half wants one table row per position; give each position its own
    # row of the reference's per-element tables by using 1 head.
    got = np.empty((free, 1, 2, half))
    for t in range(free):
        got[t] = f64.rope_rotate_half(x[t:t + 1], c.T[t:t + 1], s.T[t:t + 1])[0]
    np.testing.assert_allclose(got[:, 0, 0, :].T, outs[0], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got[:, 0, 1, :].T, outs[1], rtol=1e-5, atol=1e-5)


def test_config_siblings_reduce_to_reference_math():
    """The BASELINE siblings reuse the reference formulas: with the reference
    spec's parameters they reproduce its golden outputs."""
    _, _, (x,), outs, _ = load_golden("rmsnorm_small")
    # sum form == mean form with scale n and no eps
    n = x.shape[1]
    got = f64.rmsnorm_mean(x, None, 0.0) / np.sqrt(n)
    np.testing.assert_allclose(got, outs[0], rtol=1e-5, atol=1e-7)
    _, _, ins, outs, _ = load_golden("fused_adam_fp32")
    got = f64.ORACLES["fused_adam_cfg"]  # betas (0.9, 0.95)
    ref = f64.adam(*ins)  # spec betas (0.9, 0.999)
    for r, o in zip(ref, outs):
        np.testing.assert_allclose(r, o, rtol=2e-4, atol=2e-6)
    assert callable(got)
