"""CPU oracle for the Axon B200 backend -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the math of every spec on the hot path so
tests can check the CUDA kernels. Only `tests/`, `__graft_entry__.smoke()`
and the CPU-baseline leg of `bench.py` may import it, and only as the
checker or the timed CPU baseline; the product path (`enzyme_b200`) never
calls it and has no CPU fallback.

* `f64`    -- float64 numpy restatements, each citing the Axon reference
              file:line it follows. This is the parity oracle.
* `cpu_torch` -- fp32 torch forms of the specs' `torch_ref`s (the
              reference's CPU path), timed as the CPU baseline.

Parity pin: `tests/golden/make_golden.py` imports the reference's own
`kernels/<name>/refs.py` (where the reference tree is present) and stores
its seeded inputs and `baseline_op`/`torch_ref` outputs as fixtures;
`tests/test_oracle_golden.py` checks `f64` against them.
"""
