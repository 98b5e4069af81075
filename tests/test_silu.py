"""The SiLU * up prologue's oracle, pinned on the CPU.

The reference decoder computes the down projection's input as
``g1 = siluf(g1) * g2`` with ``siluf(x) = x / (1.0f + std::exp(-x))``
(``kernel/qwen35_decoder.cpp:129, 408``): its bits depend on the host C
library's ``expf``.  ``oracle/expf_ref.c`` restates that exponential (the
published table-driven double-precision method) and the tests here pin it:

* against ``tests/golden/golden_silu.npz``, made by the reference's own
  ``siluf`` (``oracle/ref_norm_probe.cpp`` compiles ``qwen35_decoder.cpp`` where
  it lies), bit for bit;
* against the live reference build, where it exists;
* against this host's ``expf`` over every one of the 2^32 float inputs (the
  fused form: zero differences; the unfused form differs on exactly two).
"""
import os

import numpy as np
import pytest

from cases import silu_cases, silu_digest
from conftest import bits_equal

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def golden_silu():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden_silu.npz"))


@pytest.mark.parametrize("name", sorted(silu_cases()))
def test_oracle_silu_matches_reference_goldens(name, golden_silu, oracle):
    g, u = silu_cases()[name]
    assert bytes(golden_silu[f"{name}/digest"]).hex() == silu_digest(g, u), "inputs changed"
    assert bits_equal(oracle.silu_mul(g, u), golden_silu[f"{name}/y"])


def test_oracle_silu_matches_live_reference(oracle):
    from oracle.oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref not built")
    ref = Reference()
    rng = np.random.default_rng(5)
    g = (rng.standard_normal(200_000) * rng.choice([0.1, 1.0, 10.0, 40.0], 200_000)).astype(np.float32)
    u = rng.standard_normal(200_000).astype(np.float32)
    assert bits_equal(oracle.silu_mul(g, u), ref.silu_mul(g, u))


def test_restated_expf_matches_the_host_library_on_every_float(oracle):
    """All 2^32 inputs: the fused evaluation equals the C library's expf on
    every one (NaN results compare equal to NaN).  A few seconds per core."""
    bad, first = oracle.expf_check(0, 0xFFFFFFFF, fused=True)
    assert bad == 0, f"{bad} mismatches, first at bit pattern {first:#010x}"


def test_unfused_evaluation_differs_where_documented(oracle):
    """Without the fused multiply-adds the method differs from the library on
    two inputs near float rounding midpoints (by one ulp) -- why the GPU
    evaluates it with explicit fused operations."""
    for x in (32.564632415771484, -63.09946060180664):
        u = int(np.array([x], np.float32).view(np.uint32)[0])
        assert oracle.expf_check(u, u, fused=False)[0] == 1
        assert oracle.expf_check(u, u, fused=True)[0] == 0
