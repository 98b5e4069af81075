"""The oracle is pinned before it is trusted (CPU only).

Checks the C restatement (oracle/ql_oracle.c) and the NumPy restatement
against the golden vectors that the compiled reference produced
(tests/golden/make_golden.py), and -- where oracle/_ref was built -- against
the reference library itself on fresh random inputs.
"""
import numpy as np
import pytest

from conftest import bits_equal
from oracle.oracle import Reference, np_block_sums, np_quantize_i16

from cases import all_cases, input_digest

CASES = sorted(all_cases())


@pytest.mark.parametrize("name", CASES)
def test_inputs_regenerate_exactly(name, cases, golden):
    case = cases[name]()
    stored = bytes(golden[f"{name}/digest"]).hex()
    assert input_digest(case) == stored, "input recipe or RNG stream drifted; regenerate the goldens"


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_goldens(name, cases, golden, oracle):
    case = cases[name]()
    for i, (hp, a) in enumerate(case["acts"]):
        c = oracle.matmul(case["qweight"], case["scales"], case["qzeros"], case["N"], case["K"],
                          case["bits"], a, hi_prec=hp)
        assert bits_equal(c, golden[f"{name}/C{i}"]), f"{name} set {i} (hi_prec={hp})"


@pytest.mark.parametrize("name", [n for n in CASES if not n.startswith("width")])
def test_oracle_integer_stages_match_goldens(name, cases, golden, oracle):
    case = cases[name]()
    checked = 0
    for i, (hp, a) in enumerate(case["acts"]):
        key = f"{name}/cs{i}"
        if key not in golden.files:
            continue
        hi, lo, asc = oracle.quantize_i16(a)
        assert np.array_equal(hi, golden[f"{name}/hi{i}"])
        assert np.array_equal(lo, golden[f"{name}/lo{i}"])
        assert bits_equal(asc, golden[f"{name}/as{i}"])
        cs = oracle.block_sums(case["qweight"], case["qzeros"], case["N"], case["K"], case["bits"], hi, lo)
        assert np.array_equal(cs, golden[key])
        # the NumPy restatement agrees on the integer stages too
        nhi, nlo, nas = np_quantize_i16(a)
        assert np.array_equal(nhi, hi) and np.array_equal(nlo, lo) and bits_equal(nas, asc)
        ncs = np_block_sums(case["qweight"], case["qzeros"], case["N"], case["K"], case["bits"], nhi, nlo)
        assert np.array_equal(ncs, cs)
        # and the FP32 chain over the golden INT32 accumulators reproduces the output
        c = oracle.rescale(golden[key], asc, case["scales"], case["N"], case["K"])
        assert bits_equal(c, golden[f"{name}/C{i}"])
        checked += 1
    assert checked or name.startswith("rtn_b8") or name.startswith("rtn_b4_m1")


@pytest.mark.skipif(not Reference.available(), reason="oracle/_ref not built (no reference checkout)")
@pytest.mark.parametrize("seed", range(6))
def test_oracle_matches_live_reference(seed, oracle):
    rng = np.random.default_rng(1000 + seed)
    N = 16 * int(rng.integers(1, 6))
    K = 32 * int(rng.integers(1, 40))
    bits = int(rng.choice([4, 8]))
    M = int(rng.integers(1, 20))
    qw = rng.integers(0, 256, (N, K // 32, 4 * bits), dtype=np.uint8)
    sc = rng.uniform(1e-4, 0.05, (N, K // 32)).astype(np.float16 if seed % 2 else np.float32)
    qz = rng.integers(0, 256, (N, (K // 32 + 1) // 2), dtype=np.uint8) if (bits == 4 and seed % 3) else None
    a = rng.standard_normal((M, K)).astype(np.float32) * np.float32(rng.uniform(0.01, 100))
    ref = Reference()
    h = ref.prepack(qw, sc, qz, K, N, bits)
    try:
        for hp in (True, False):
            expect = ref.matmul(h, a, N, hi_prec=hp, threads=2)
            got = oracle.matmul(qw, sc, qz, N, K, bits, a, hi_prec=hp)
            assert bits_equal(got, expect)
    finally:
        ref.free(h)
