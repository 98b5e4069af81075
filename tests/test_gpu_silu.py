"""GPU parity of the fused SiLU * up prologue (the down projection's input).

``ql_quantize_act_silu_mul_dev`` writes silu(gate) * up as it quantizes it;
those products must equal the reference's own ``siluf(g) * u``
(``kernel/qwen35_decoder.cpp:129, 408``; the golden fixture) bit for bit,
including the inputs near rounding midpoints of the C library's expf, the
overflow/underflow edges, infinities and NaN.  ``ql_matmul_silu_mul_dev``
must equal the oracle's matmul on those products (decode kernels and the
tensor-core GEMM, both activation modes, gate and up side by side in one
buffer as a concatenated gate|up output leaves them).
"""
import os

import numpy as np
import pytest

import qlc
from cases import silu_cases
from conftest import bits_equal

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(autouse=True)
def _mode_reset():
    yield
    qlc.set_hi_prec(False)
    assert qlc.device_error() == 0


@pytest.mark.parametrize("name", sorted(silu_cases()))
@pytest.mark.parametrize("hp", [True, False])
def test_silu_products_match_reference_goldens(name, hp):
    golden = np.load(os.path.join(ROOT, "tests", "golden", "golden_silu.npz"))
    g, u = silu_cases()[name]
    _, out = qlc.silu_quantize_dev(g, u, hp)
    assert bits_equal(out, golden[f"{name}/y"])


def test_silu_products_in_the_gemm_layout(oracle):
    """More than 64 rows quantize into the GEMM's records; the products are
    the same, with gate and up side by side (ld = 2K)."""
    rng = np.random.default_rng(3)
    M, K = 130, 512
    g = (rng.normal(size=(M, K)) * 6.0).astype(np.float32)
    u = rng.normal(size=(M, K)).astype(np.float32)
    _, out = qlc.silu_quantize_dev(g, u, True, ld=2 * K)
    assert bits_equal(out, oracle.silu_mul(g, u))


@pytest.mark.parametrize("hp", [True, False])
def test_matmul_silu_matches_oracle(hp, oracle):
    from breeze_engine_b200.quant import quantize_matmul_nbits
    rng = np.random.default_rng(11)
    K, N = 1024, 8192 + 16          # N >= 8192: the INT4 dp4a kernel at one and two rows
    w = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    qw, sc, qz = quantize_matmul_nbits(w, bits=4, symmetric=False)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    qlc.set_hi_prec(hp)
    try:
        for M in (1, 2, 5, 64, 130):
            g = (rng.normal(size=(M, K)) * 3.0).astype(np.float32)
            u = rng.normal(size=(M, K)).astype(np.float32)
            got = qlc.matmul_silu_dev(h, g, u, N, ld_pad=4 * (M % 3))
            expect = oracle.matmul(qw, sc, qz, N, K, 4, oracle.silu_mul(g, u), hi_prec=hp)
            assert bits_equal(got, expect), M
    finally:
        qlc.free(h)


def test_backend_silu_mul_matmul_on_a_concatenated_output(oracle):
    """backend.silu_mul_matmul on the two halves of one [M, 2K] gate|up tensor."""
    import torch
    from breeze_engine_b200 import backend
    from breeze_engine_b200.quant import quantize_matmul_nbits
    rng = np.random.default_rng(12)
    K, N, M = 512, 256, 3
    w = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    qw, sc, qz = quantize_matmul_nbits(w, bits=4)
    h = backend.prepack(qw, sc, qz, K, N, bits=4)
    backend.set_hi_prec(True)
    try:
        gu = torch.from_numpy((rng.normal(size=(M, 2 * K)) * 4.0).astype(np.float32)).cuda()
        got = backend.silu_mul_matmul(h, gu[:, :K], gu[:, K:], N)
        torch.cuda.synchronize()
        g, u = gu[:, :K].cpu().numpy(), gu[:, K:].cpu().numpy()
        assert bits_equal(got.cpu().numpy(), oracle.matmul(qw, sc, qz, N, K, 4, oracle.silu_mul(g, u)))
    finally:
        backend.free(h)
