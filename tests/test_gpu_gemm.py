"""GPU parity of the prefill GEMM (M > 64 tokens, tcgen05) against the oracle.

Token counts above 64 route through the tensor-core GEMM (ql_gemm.cu) and its
own activation records (ql_quant.cu).  The shapes here hit its tails: token
tiles of 128 with a ragged last tile, weight tiles of 8 row groups with a
ragged last tile, and block counts that leave a partial stage of 4 blocks.
The bar is the same as for the decode kernel: FP32 outputs and INT32 block
sums bit-identical to the reference algorithm.  INT4 weights with fp16 scales
have four GEMMs (tcgen05 kind::f16 on pre-dequantized FP16 operands, kind::f16
unpacking per tile on CTA pairs or single CTAs, and kind::i8); every test runs
under each selector.
"""
import ctypes

import numpy as np
import pytest

import qlc
from cases import edge_activations, outlier_activations
from conftest import bits_equal

pytestmark = pytest.mark.gpu


_KINDS = {"auto": 0, "i8": 1, "f16_pair": 2, "f16_stream": 3}


@pytest.fixture(autouse=True, params=list(_KINDS))
def prefill_kernel(request):
    """Every test runs under each prefill kernel: the automatic choice (for
    INT4 weights with fp16 scales the FP16-operand GEMM on weights dequantized
    per call, given the full workspace; else kind::i8), the kind::i8 GEMM
    forced, and the kind::f16 GEMM that unpacks weights per tile on CTA pairs
    and on single CTAs (ql_set_prefill_kernel 0 / 1 / 2 / 3)."""
    lib = qlc.lib()
    assert lib.ql_set_prefill_kernel(_KINDS[request.param]) == 0
    yield request.param
    lib.ql_set_prefill_kernel(0)
    qlc.set_hi_prec(False)
    assert qlc.device_error() == 0


def _weights(N, K, bits, zp, half, seed):
    rng = np.random.default_rng(seed)
    qw = rng.integers(0, 256, (N, K // 32, 4 * bits), dtype=np.uint8)
    sc = rng.uniform(1e-4, 0.03, (N, K // 32)).astype(np.float16 if half else np.float32)
    qz = rng.integers(0, 256, (N, (K // 32 + 1) // 2), dtype=np.uint8) if (zp and bits == 4) else None
    return qw, sc, qz


FORMATS = [(4, False, True), (4, True, True), (4, True, False), (4, False, False),
           (8, False, True), (8, False, False)]


@pytest.mark.parametrize("bits,zp,half", FORMATS)
@pytest.mark.parametrize("hp", [True, False])
def test_gemm_formats_and_tails(bits, zp, half, hp, oracle):
    """N = 272 (tiles of 8, 8 and 1 row groups), K = 224 (a stage of 4 blocks
    then one of 3), token counts around the 128-token tile."""
    N, K = 272, 224
    qw, sc, qz = _weights(N, K, bits, zp, half, 11 + bits)
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    qlc.set_hi_prec(hp)
    try:
        for M in (65, 127, 128, 129, 300):
            a = outlier_activations(M, K, M)
            expect = oracle.matmul(qw, sc, qz, N, K, bits, a, hi_prec=hp)
            assert bits_equal(qlc.matmul_dev(h, a, N), expect), f"M={M}"
    finally:
        qlc.free(h)


@pytest.mark.parametrize("bits,zp", [(4, True), (4, False), (8, False)])
def test_gemm_block_sums_bit_exact(bits, zp, oracle):
    """The per-(token, column, block) INT32 accumulators 256*S_hi + S_lo."""
    N, K, M = 144, 32 * 9, 131
    qw, sc, qz = _weights(N, K, bits, zp, True, 5)
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    qlc.set_hi_prec(True)
    try:
        a = outlier_activations(M, K, 2)
        hi, lo, _ = oracle.quantize_i16(a)
        expect = oracle.block_sums(qw, qz, N, K, bits, hi, lo)
        assert np.array_equal(qlc.block_sums_dev(h, a, N, K), expect)
    finally:
        qlc.free(h)


def test_gemm_edge_activations(oracle):
    """Zeros, subnormals, infinities, NaN and saturating values through the GEMM."""
    N, K, M = 160, 32 * 6, 150
    qw, sc, qz = _weights(N, K, 4, True, True, 9)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    try:
        for hp in (True, False):
            qlc.set_hi_prec(hp)
            a = edge_activations(M, K, 4)
            assert bits_equal(qlc.matmul_dev(h, a, N), oracle.matmul(qw, sc, qz, N, K, 4, a, hi_prec=hp))
    finally:
        qlc.free(h)


@pytest.mark.parametrize("N,K,bits,M", [(256, 4096, 4, 256), (384, 2048, 8, 200), (1024, 512, 4, 1000)])
def test_gemm_larger_shapes(N, K, bits, M, oracle):
    """Long K (many stages per tile), several waves of tiles per CTA."""
    qw, sc, qz = _weights(N, K, bits, bits == 4, True, N + M)
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    qlc.set_hi_prec(True)
    try:
        a = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
        assert bits_equal(qlc.matmul_dev(h, a, N), oracle.matmul(qw, sc, qz, N, K, bits, a))
        assert bits_equal(qlc.matmul_host(h, a, N), oracle.matmul(qw, sc, qz, N, K, bits, a))
    finally:
        qlc.free(h)


@pytest.mark.parametrize("hp", [True, False])
def test_gemm_workspace_sizes_and_kernel_rerun(hp, prefill_kernel, oracle):
    """INT4 with fp16 scales: the full workspace (FP16-operand GEMM), the
    activation-records-only workspace (the per-tile-unpack GEMM) and
    ql_prefill_gemm_dev re-running the GEMM on the prepared workspace all give
    the oracle's bits."""
    import torch
    lib = qlc.lib()
    N, K, M = 272, 640, 300
    qw, sc, qz = _weights(N, K, 4, True, True, 33)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    qlc.set_hi_prec(hp)
    try:
        a = outlier_activations(M, K, 7)
        expect = oracle.matmul(qw, sc, qz, N, K, 4, a, hi_prec=hp)
        dA = torch.from_numpy(a).cuda()
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        full = lib.ql_workspace_bytes(ctypes.c_void_p(h), M)
        small = lib.ql_act_workspace_bytes(M, K)
        assert full >= small
        for nbytes in (full, small):
            ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
            c = torch.full((M, N), -1.0, device="cuda")
            assert lib.ql_matmul_dev_ws(ctypes.c_void_p(h), dA.data_ptr(), M, c.data_ptr(), ws.data_ptr(), nbytes,
                                        s) == 0
            torch.cuda.synchronize()
            assert bits_equal(c.cpu().numpy(), expect), nbytes
            c2 = torch.full((M, N), -1.0, device="cuda")
            rc = lib.ql_prefill_gemm_dev(ctypes.c_void_p(h), ws.data_ptr(), nbytes, M, int(hp), c2.data_ptr(), s)
            torch.cuda.synchronize()
            if prefill_kernel == "auto" and nbytes == full:
                assert rc == 0 and bits_equal(c2.cpu().numpy(), expect)
            else:
                assert rc in (qlc.L.QL_ENOTSUP, qlc.L.QL_EINVAL)
    finally:
        qlc.free(h)


def test_gemm_quantize_once_matches_matmul():
    """ql_quantize_act_dev + ql_matmul_quantized_dev (shared activations) give
    the same bits as ql_matmul_dev_ws for a prefill-sized token count."""
    import torch
    lib = qlc.lib()
    N, K, M = 400, 640, 333
    qw, sc, qz = _weights(N, K, 4, True, True, 21)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    try:
        for hp in (True, False):
            qlc.set_hi_prec(hp)
            a = torch.randn(M, K, device="cuda")
            ref = torch.from_numpy(qlc.matmul_dev(h, a.cpu().numpy(), N))
            need = lib.ql_act_workspace_bytes(M, K)
            assert need <= lib.ql_workspace_bytes(h, M)     # the one-call form may add FP16 operands
            ws = torch.empty(need, dtype=torch.uint8, device="cuda")
            c = torch.empty(M, N, device="cuda")
            s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            assert lib.ql_quantize_act_dev(a.data_ptr(), M, K, int(hp), ws.data_ptr(), need, s) == 0
            assert lib.ql_matmul_quantized_dev(h, ws.data_ptr(), M, int(hp), c.data_ptr(), s) == 0
            torch.cuda.synchronize()
            assert torch.equal(c.cpu().view(torch.int32), ref.view(torch.int32))
    finally:
        qlc.free(h)


@pytest.fixture(scope="module")
def prefill_weights():
    """configs[2]'s layer (K = 5120, N = 17408): N(0, 0.02) weights RTN-packed
    to INT4 with zero points, built once for the module."""
    from breeze_engine_b200.quant import quantize_matmul_nbits
    K, N = 5120, 17408
    rng = np.random.default_rng(K + N)
    w = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    return quantize_matmul_nbits(w, bits=4, symmetric=False)


@pytest.mark.slow
@pytest.mark.parametrize("M", [128, 512, 2048])
def test_gemm_prefill_full_size_sampled_columns(M, prefill_weights, oracle):
    """The prefill configuration (K = 5120, N = 17408, INT4, M in {128, 512,
    2048} tokens with 1% outlier channels): a random sample of 16-column groups
    matches the oracle bit for bit (each column slice of the MatMulNBits arrays
    is an exact sub-problem)."""
    K, N = 5120, 17408
    qw, sc, qz = prefill_weights
    rng = np.random.default_rng(K + N + M)
    a = outlier_activations(M, K, 3)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    qlc.set_hi_prec(True)
    try:
        c = qlc.matmul_dev(h, a, N)
    finally:
        qlc.free(h)
    nblk = K // 32
    qz2 = qz.reshape(N, -1)
    for g in np.sort(rng.choice(N // 16, size=8, replace=False)):
        rows = slice(16 * g, 16 * g + 16)
        expect = oracle.matmul(qw.reshape(N, -1)[rows], sc.reshape(N, nblk)[rows], qz2[rows], 16, K, 4, a)
        assert bits_equal(c[:, rows], expect), f"columns {16 * g}..{16 * g + 15}"
    assert np.isfinite(c).all()
