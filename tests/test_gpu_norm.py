"""GPU parity of the fused RMSNorm prologue and of concatenated weights.

The reference decoder runs rmsnorm into a scratch row and then i4_matmul on it
(kernel/qwen35_decoder.cpp:133-141 and 405-407).  The library's
ql_quantize_act_rmsnorm_dev / ql_matmul_rmsnorm_dev fold the normalisation
into the activation quantizer; the bar is bit-exact against the reference's
own normalised rows (golden_norm.npz) and against i4_matmul on them.  The
tie rows force the row-factor kernel off its certified parallel sum onto the
reference's serial loop.  ql_weight_concat stacks gate and up along N; its
outputs must equal the separate weights' bit for bit.
"""
import ctypes
import os

import numpy as np
import pytest

import qlc
from breeze_engine_b200 import _lib as L
from cases import fixture_weights, norm_cases, outlier_activations, tie_rows
from conftest import ROOT, bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _mode_reset():
    yield
    qlc.set_hi_prec(False)
    assert qlc.device_error() == 0


@pytest.fixture(scope="module")
def golden_norm():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden_norm.npz"))


def _norm_w(K, seed=41):
    return (1.0 + 0.1 * np.random.default_rng(seed).normal(size=K)).astype(np.float32)


@pytest.mark.parametrize("hp", [True, False])
@pytest.mark.parametrize("name", list(norm_cases()))
def test_hn_matches_reference_golden(name, hp, golden_norm):
    x, w, eps = norm_cases()[name]
    _, hn = qlc.rmsnorm_quantize_dev(x, w, eps, hp)
    assert bits_equal(hn, golden_norm[f"{name}/hn"])


@pytest.mark.parametrize("reps", [3, 7])          # 72 and 168 rows: the GEMM layout
def test_tie_rows_in_the_gemm_layout(reps, oracle):
    x = np.tile(tie_rows(), (reps, 1))
    w = np.ones(x.shape[1], np.float32)
    _, hn = qlc.rmsnorm_quantize_dev(x, w, 0.0, True)
    assert bits_equal(hn, oracle.rmsnorm(x, w, 0.0))


@pytest.mark.parametrize("hp", [True, False])
@pytest.mark.parametrize("bits,zp,half", [(4, False, True), (4, True, True), (8, False, False)])
@pytest.mark.parametrize("M", [1, 3, 64, 65, 200])
def test_fused_matmul_equals_matmul_of_reference_rows(M, bits, zp, half, hp, oracle):
    N, K = 96, 5120
    qw, sc, qz = fixture_weights(N, K, bits, np.float16 if half else np.float32, zp)
    x = outlier_activations(M, K, 43 + M)
    w = _norm_w(K)
    hn = oracle.rmsnorm(x, w, 1e-6)
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    try:
        qlc.set_hi_prec(hp)
        fused = qlc.matmul_rmsnorm_dev(h, x, w, 1e-6, N)
        want = oracle.matmul(qw, sc, qz, N, K, bits, hn, hi_prec=hp)
        assert bits_equal(fused, want)
        assert bits_equal(qlc.matmul_dev(h, hn, N), want)
    finally:
        qlc.free(h)


@pytest.mark.parametrize("name", ["edge_k96", "ties", "zero_eps0_k32"])
def test_fused_matmul_edge_rows(name, golden_norm, oracle):
    """NaN, inf, zero and subnormal rows, eps = 0, and the serial-order rows,
    through the whole fused call (against the oracle on the reference's rows)."""
    x, w, eps = norm_cases()[name]
    K = x.shape[1]
    N = 32
    qw, sc, qz = fixture_weights(N, K, 4, np.float16, True)
    hn = golden_norm[f"{name}/hn"]
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    try:
        qlc.set_hi_prec(True)
        assert bits_equal(qlc.matmul_rmsnorm_dev(h, x, w, eps, N), oracle.matmul(qw, sc, qz, N, K, 4, hn))
    finally:
        qlc.free(h)


@pytest.mark.parametrize("hp", [True, False])
@pytest.mark.parametrize("M", [1, 9, 130])
def test_gate_up_concat_on_one_normalised_input(M, hp, oracle):
    """The MLP front of the reference decoder (rmsnorm, then gate and up on the
    same rows, kernel/qwen35_decoder.cpp:405-407) as one quantize and one
    launch over the concatenated weight."""
    K, Ng, Nu = 2048, 80, 48
    gq, gs, gz = fixture_weights(Ng, K, 4, np.float16, False)
    uq, us, uz = fixture_weights(Nu, K, 4, np.float16, False)
    x = outlier_activations(M, K, 47)
    w = _norm_w(K, 48)
    hn = oracle.rmsnorm(x, w, 1e-6)
    hg = qlc.prepack(gq, gs, gz, Ng, K, 4)
    hu = qlc.prepack(uq, us, uz, Nu, K, 4)
    hc = qlc.concat([hg, hu])
    try:
        N = ctypes.c_int()
        assert qlc.lib().ql_weight_info(ctypes.c_void_p(hc), ctypes.byref(N), None, None, None, None) == 0
        assert N.value == Ng + Nu
        ws, _ = qlc.rmsnorm_quantize_dev(x, w, 1e-6, hp, want_hn=False)
        both = qlc.matmul_quantized_dev(hc, ws, M, hp, Ng + Nu)
        qlc.set_hi_prec(hp)
        assert bits_equal(both[:, :Ng], qlc.matmul_dev(hg, hn, Ng))
        assert bits_equal(both[:, Ng:], qlc.matmul_dev(hu, hn, Nu))
        assert bits_equal(both[:, :Ng], qlc.matmul_quantized_dev(hg, ws, M, hp, Ng))
    finally:
        for h in (hc, hg, hu):
            qlc.free(h)


def test_concat_rejects_mismatched_weights():
    a = qlc.prepack(*fixture_weights(32, 64, 4, np.float16, False), 32, 64, 4)
    b = qlc.prepack(*fixture_weights(32, 96, 4, np.float16, False), 32, 96, 4)      # K differs
    c = qlc.prepack(*fixture_weights(32, 64, 4, np.float16, True), 32, 64, 4)       # zero points
    d = qlc.prepack(*fixture_weights(32, 64, 8, np.float16, False), 32, 64, 8)      # bits
    e = qlc.prepack(*fixture_weights(32, 64, 4, np.float32, False), 32, 64, 4)      # scale type
    try:
        for other in (b, c, d, e):
            arr = (ctypes.c_void_p * 2)(a, other)
            out = ctypes.c_void_p()
            assert qlc.lib().ql_weight_concat(arr, 2, ctypes.byref(out)) == L.QL_EINVAL
            assert not out.value
    finally:
        for h in (a, b, c, d, e):
            qlc.free(h)


def test_backend_rmsnorm_matmul_and_concat(oracle):
    """The Python host API over the same entry points (torch CUDA tensors)."""
    import torch
    from breeze_engine_b200 import backend
    K, N = 1024, 64
    qw, sc, qz = fixture_weights(N, K, 4, np.float16, True)
    x = outlier_activations(5, K, 51)
    w = _norm_w(K, 52)
    h = backend.prepack(qw, sc, qz, K, N, 4)
    hc = backend.concat_packed([h, h])
    try:
        backend.set_hi_prec(True)
        got = backend.rmsnorm_matmul(h, torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), 1e-6, N)
        want = oracle.matmul(qw, sc, qz, N, K, 4, oracle.rmsnorm(x, w, 1e-6))
        assert bits_equal(got.cpu().numpy(), want)
        both = backend.matmul(hc, oracle.rmsnorm(x, w, 1e-6), 2 * N)
        assert bits_equal(both[:, :N], want) and bits_equal(both[:, N:], want)
        with pytest.raises(TypeError):
            backend.rmsnorm_matmul(h, x, w, 1e-6, N)
    finally:
        backend.set_hi_prec(False)
        backend.free(hc)
        backend.free(h)
