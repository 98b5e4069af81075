"""GPU parity of libbreeze_ql.so against the oracle and the reference goldens.

Every call goes through the C ABI (tests/qlc.py).  The bar is bit-exact: the
activation planes and scales, the per-block INT32 accumulators, and the FP32
outputs (the kernels run each output's rescale chain in reference block order).
"""
import ctypes

import numpy as np
import pytest

import qlc
from cases import all_cases, edge_activations, fixture_weights, outlier_activations
from conftest import bits_equal

pytestmark = pytest.mark.gpu

CASES = sorted(all_cases())


@pytest.fixture(autouse=True)
def _mode_reset():
    yield
    qlc.set_hi_prec(False)
    assert qlc.device_error() == 0


# ---------------------------------------------------------------- quantizer

@pytest.mark.parametrize("M,K,kind", [(1, 32, "normal"), (5, 256, "edge"), (9, 4096, "outliers"),
                                      (64, 5120, "normal"), (300, 96, "normal")])
def test_quantizer_bit_exact(M, K, kind, oracle):
    if kind == "edge":
        a = edge_activations(M, K, 3)
    elif kind == "outliers":
        a = outlier_activations(M, K, 4)
    else:
        a = np.random.default_rng(M + K).standard_normal((M, K)).astype(np.float32)
    hi, lo, asc = qlc.quantize_dev(a)
    ohi, olo, oasc = oracle.quantize_i16(a)
    assert np.array_equal(hi, ohi)
    assert np.array_equal(lo, olo)
    assert bits_equal(asc, oasc)


@pytest.mark.parametrize("name", [n for n in CASES])
def test_quantizer_matches_reference_planes(name, cases, golden):
    case = cases[name]()
    for i, (hp, a) in enumerate(case["acts"]):
        if f"{name}/hi{i}" not in golden.files:
            continue
        hi, lo, asc = qlc.quantize_dev(a)
        assert np.array_equal(hi, golden[f"{name}/hi{i}"])
        assert np.array_equal(lo, golden[f"{name}/lo{i}"])
        assert bits_equal(asc, golden[f"{name}/as{i}"])


# ---------------------------------------------------------------- goldens

@pytest.mark.parametrize("name", CASES)
def test_goldens_bit_exact(name, cases, golden):
    case = cases[name]()
    h = qlc.prepack(case["qweight"], case["scales"], case["qzeros"], case["N"], case["K"], case["bits"])
    try:
        for i, (hp, a) in enumerate(case["acts"]):
            qlc.set_hi_prec(hp)
            expect = golden[f"{name}/C{i}"]
            assert bits_equal(qlc.matmul_dev(h, a, case["N"]), expect), f"device path, set {i}"
            assert bits_equal(qlc.matmul_host(h, a, case["N"]), expect), f"i4_matmul, set {i}"
            if f"{name}/cs{i}" in golden.files:
                cs = qlc.block_sums_dev(h, a, case["N"], case["K"])
                assert np.array_equal(cs, golden[f"{name}/cs{i}"]), f"INT32 accumulators, set {i}"
    finally:
        qlc.free(h)


# ---------------------------------------------------------------- sweeps vs the oracle

def _weights(N, K, bits, zp, half, seed):
    rng = np.random.default_rng(seed)
    qw = rng.integers(0, 256, (N, K // 32, 4 * bits), dtype=np.uint8)
    sc = rng.uniform(1e-4, 0.03, (N, K // 32)).astype(np.float16 if half else np.float32)
    qz = rng.integers(0, 256, (N, (K // 32 + 1) // 2), dtype=np.uint8) if (zp and bits == 4) else None
    return qw, sc, qz


@pytest.mark.parametrize("bits,zp,half", [(4, False, True), (4, True, True), (4, True, False),
                                          (8, False, True), (8, False, False)])
@pytest.mark.parametrize("hp", [True, False])
def test_token_count_sweep(bits, zp, half, hp, oracle):
    N, K = 48, 320
    qw, sc, qz = _weights(N, K, bits, zp, half, 7)
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    qlc.set_hi_prec(hp)
    try:
        for M in (1, 2, 3, 7, 8, 9, 15, 16, 17, 31, 33, 63, 64, 65, 129):
            a = outlier_activations(M, K, M)
            expect = oracle.matmul(qw, sc, qz, N, K, bits, a, hi_prec=hp)
            assert bits_equal(qlc.matmul_dev(h, a, N), expect), f"M={M}"
            if hp and M in (3, 17, 65):
                hi, lo, _ = oracle.quantize_i16(a)
                cs = oracle.block_sums(qw, qz, N, K, bits, hi, lo)
                assert np.array_equal(qlc.block_sums_dev(h, a, N, K), cs), f"cs M={M}"
    finally:
        qlc.free(h)


@pytest.mark.parametrize("N,K", [(16, 32), (16, 96), (32, 32 * 37), (4096, 64), (9600, 64), (19200, 64),
                                 (160, 32 * 41)])
@pytest.mark.parametrize("bits", [4, 8])
def test_shapes_cover_every_launch_config(N, K, bits, oracle):
    """Row-group counts that select 1/2/4 groups per CTA, odd block counts, K tails."""
    qw, sc, qz = _weights(N, K, bits, bits == 4, True, N + K)
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    qlc.set_hi_prec(True)
    try:
        for M in (1, 12):
            a = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
            expect = oracle.matmul(qw, sc, qz, N, K, bits, a)
            assert bits_equal(qlc.matmul_dev(h, a, N), expect), f"M={M}"
    finally:
        qlc.free(h)


def test_library_workspace_variant(oracle):
    qw, sc, qz = _weights(64, 512, 4, True, True, 3)
    h = qlc.prepack(qw, sc, qz, 64, 512, 4)
    qlc.set_hi_prec(True)
    try:
        for M in (4, 70, 2):          # grows, then reuses the library workspace
            a = np.random.default_rng(M).standard_normal((M, 512)).astype(np.float32)
            assert bits_equal(qlc.matmul_dev(h, a, 64, workspace=False),
                              oracle.matmul(qw, sc, qz, 64, 512, 4, a))
    finally:
        qlc.free(h)


# ---------------------------------------------------------------- legacy VNNI prepack

def _vnni_layout(qw, sc, qz, N, K, bits):
    """The reference's legacy VNNI layout, restated from breeze/cpu_backend.py:171-227."""
    nblk, ntiles = K // 32, N // 16
    tile16 = lambda x: np.ascontiguousarray(x.reshape(ntiles, 16, nblk).transpose(0, 2, 1))
    s = tile16(np.asarray(sc, np.float32).reshape(N, nblk))
    if bits == 8:
        b = (qw.reshape(N, nblk, 32).astype(np.int16) - 128).astype(np.int8)
        Bv = np.ascontiguousarray(b.reshape(ntiles, 16, nblk, 8, 4).transpose(0, 2, 3, 1, 4).reshape(ntiles, nblk, 8, 64))
        corr = tile16((128 * b.astype(np.int32).sum(axis=2)).astype(np.int32))
        return Bv.view(np.uint8), s, None, corr
    q = np.empty((N, nblk, 32), np.uint8)
    q[:, :, 0::2] = qw.reshape(N, nblk, 16) & 15
    q[:, :, 1::2] = qw.reshape(N, nblk, 16) >> 4
    if qz is not None:
        z2 = np.empty((N, 2 * ((nblk + 1) // 2)), np.uint8)
        z2[:, 0::2] = qz.reshape(N, -1) & 15
        z2[:, 1::2] = qz.reshape(N, -1) >> 4
        zp = z2[:, :nblk].astype(np.int32)
    else:
        zp = np.full((N, nblk), 8, np.int32)
    w2 = q.reshape(ntiles, 16, nblk, 8, 4).transpose(0, 2, 3, 1, 4).reshape(ntiles, nblk, 8, 64)
    Bv = np.ascontiguousarray((w2[..., 0::2] | (w2[..., 1::2] << 4)).astype(np.uint8))
    corr = tile16((128 * (q.astype(np.int32).sum(axis=2) - 32 * zp)).astype(np.int32))
    return Bv, s, tile16(zp.astype(np.int8)), corr


@pytest.mark.parametrize("bits,zp", [(4, False), (4, True), (8, False)])
def test_legacy_vnni_prepack_matches_onnx_prepack(bits, zp):
    N, K = 48, 96
    qw, sc, qz = fixture_weights(N, K, bits, np.float32, zp)
    qz = qz if bits == 4 else None
    B, s, z, corr = _vnni_layout(qw, sc, qz, N, K, bits)
    lib = qlc.lib()
    h_old = lib.i4_prepack(B.ctypes.data, s.ctypes.data, z.ctypes.data if z is not None else None,
                           corr.ctypes.data, N, K, K // 32, bits)
    assert h_old
    h_new = qlc.prepack(qw, sc, qz, N, K, bits)
    qlc.set_hi_prec(True)
    try:
        a = np.random.default_rng(5).standard_normal((9, K)).astype(np.float32)
        assert bits_equal(qlc.matmul_dev(h_old, a, N), qlc.matmul_dev(h_new, a, N))
    finally:
        qlc.free(h_old)
        qlc.free(h_new)


# ---------------------------------------------------------------- device API contract

def test_device_api_rejects_bad_calls():
    import torch
    lib = qlc.lib()
    qw, sc, qz = _weights(32, 64, 4, False, True, 1)
    h = qlc.prepack(qw, sc, qz, 32, 64, 4)
    try:
        a = torch.zeros((2, 64 + 4), dtype=torch.float32, device="cuda")
        c = torch.zeros((2, 32), dtype=torch.float32, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        assert lib.ql_matmul_dev(h, a.data_ptr() + 4, 2, c.data_ptr(), s) == 1        # misaligned A
        need = lib.ql_workspace_bytes(h, 2)
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        assert lib.ql_matmul_dev_ws(h, a.data_ptr(), 2, c.data_ptr(), ws.data_ptr(), need - 1, s) == 1
        assert lib.ql_matmul_dev_ws(h, a.data_ptr(), 0, c.data_ptr(), ws.data_ptr(), need, s) == 0
        assert lib.ql_matmul_dev_ws(h, a.data_ptr(), -1, c.data_ptr(), ws.data_ptr(), need, s) == 1
    finally:
        qlc.free(h)


# ---------------------------------------------------------------- full-size properties

@pytest.mark.slow
def test_config1_full_size_bit_exact(oracle):
    """The benchmark spec's first config (INT4, M=1, K=N=4096) against the oracle on every output."""
    from breeze_engine_b200.quant import quantize_matmul_nbits
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, (4096, 4096)).astype(np.float32)
    qw, sc, qz = quantize_matmul_nbits(w, bits=4)
    a = rng.standard_normal((1, 4096)).astype(np.float32)
    h = qlc.prepack(qw, sc, qz, 4096, 4096, 4)
    qlc.set_hi_prec(True)
    try:
        assert bits_equal(qlc.matmul_dev(h, a, 4096), oracle.matmul(qw, sc, qz, 4096, 4096, 4, a))
    finally:
        qlc.free(h)


@pytest.mark.slow
@pytest.mark.parametrize("K,N,bits,M", [(4096, 151936, 8, 16), (12288, 4096, 8, 16), (5120, 17408, 4, 64)])
def test_full_size_sampled_columns(K, N, bits, M, oracle):
    """Full benchmark-spec shapes: every output column of a random sample matches the
    oracle bit for bit (outputs are independent per column, so a column slice of
    the MatMulNBits arrays is an exact sub-problem)."""
    from breeze_engine_b200.quant import quantize_matmul_nbits
    rng = np.random.default_rng(K + N)
    w = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    qw, sc, qz = quantize_matmul_nbits(w, bits=bits, per_channel=(bits == 8))
    del w
    a = outlier_activations(M, K, 9)
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    qlc.set_hi_prec(True)
    try:
        c = qlc.matmul_dev(h, a, N)
    finally:
        qlc.free(h)
    groups = np.sort(rng.choice(N // 16, size=12, replace=False))
    nblk = K // 32
    for g in groups:
        rows = slice(16 * g, 16 * g + 16)
        sub_qw = qw.reshape(N, -1)[rows]
        sub_sc = sc.reshape(N, nblk)[rows]
        expect = oracle.matmul(sub_qw, sub_sc, None, 16, K, bits, a)
        assert bits_equal(c[:, rows], expect), f"columns {16 * g}..{16 * g + 15}"
    assert np.isfinite(c).all()


@pytest.mark.parametrize("M,N,K,bits", [(16, 16384, 256, 4), (64, 12288, 128, 8), (130, 4096, 256, 4),
                                         (300, 2000, 224, 4), (9, 151936, 64, 8)])
def test_host_call_output_chunks(M, N, K, bits):
    """i4_matmul splits large outputs into column chunks whose device->host
    copies overlap the next chunk's matmul; the result must be bit-identical to
    the single device call (ql_matmul_dev_ws) for decode and prefill sizes,
    ragged last chunks included."""
    rng = np.random.default_rng(M + N)
    nblk = K // 32
    qw = rng.integers(0, 256, (N, nblk, 4 * bits), dtype=np.uint8)
    sc = rng.uniform(1e-3, 2e-2, (N, nblk)).astype(np.float16)
    h = qlc.prepack(qw, sc, None, N, K, bits)
    qlc.set_hi_prec(True)
    try:
        a = rng.standard_normal((M, K)).astype(np.float32)
        assert bits_equal(qlc.matmul_host(h, a, N), qlc.matmul_dev(h, a, N))
    finally:
        qlc.set_hi_prec(False)
        qlc.free(h)


@pytest.mark.parametrize("bits,half,N,K,M,cfg", [
    (8, False, 96, 5120, 64, None), (8, False, 96, 5120, 57, None), (8, True, 96, 5120, 64, None),
    (8, False, 32, 2048, 64, None), (8, False, 96, 5120, 64, "1,4,2,4"), (8, False, 96, 5120, 64, "2,4,2,8"),
    (4, True, 96, 5120, 64, "1,4,2,8"), (4, True, 96, 5120, 64, "1,8,2,8")])
def test_split_k_relay_repeatable(bits, half, N, K, M, cfg, oracle, monkeypatch):
    """K split across warps with one sub-chunk per stage (each warp hands its
    stage back before it waits for the relay): the last token groups must be
    right on every run.  These shapes and tuning overrides once failed
    intermittently (rows 48-63), until every stage release was preceded by an
    async-proxy fence."""
    import torch
    if cfg:
        monkeypatch.setenv("BREEZE_QL_DECODE_CONFIG", cfg)
    qw, sc, qz = fixture_weights(N, K, bits, np.float16 if half else np.float32, False)
    a = outlier_activations(M, K, 43 + M)
    ref = oracle.matmul(qw, sc, qz, N, K, bits, a)
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    lib = qlc.lib()
    try:
        qlc.set_hi_prec(True)
        dA = torch.from_numpy(a).cuda()
        n = lib.ql_act_workspace_bytes(M, K)
        ws = torch.empty(n, dtype=torch.uint8, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        assert lib.ql_quantize_act_dev(dA.data_ptr(), M, K, 1, ws.data_ptr(), n, s) == 0
        for _ in range(10):
            c = torch.full((M, N), -1.0, device="cuda")
            assert lib.ql_matmul_quantized_dev(ctypes.c_void_p(h), ws.data_ptr(), M, 1, c.data_ptr(), s) == 0
            torch.cuda.synchronize()
            assert bits_equal(c.cpu().numpy(), ref)
    finally:
        qlc.free(h)


@pytest.mark.parametrize("zp,half", [(False, True), (True, True), (True, False), (False, False)])
@pytest.mark.parametrize("hp", [True, False])
@pytest.mark.parametrize("K", [64, 800, 4096])
def test_dp4a_decode_kernel(zp, half, hp, K, oracle):
    """INT4 at one and two tokens on layers of >= 8192 rows run the dp4a
    decode kernel (ql_gemv4.cu): outputs and per-block INT32 accumulators
    bit-exact against the oracle, with explicit zero points, fp16/fp32 scales,
    both activation modes, and K from 2 blocks (no K split) to 128 (split,
    relayed accumulators).  N = 8208 leaves a partial last quad of row groups;
    the activations include edge values (zeros, outliers)."""
    from cases import edge_activations
    N = 8208
    qw, sc, qz = _weights(N, K, 4, zp, half, K + 2 * zp + half)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    qlc.set_hi_prec(hp)
    try:
        for M in (1, 2, 1):
            a = np.random.default_rng(M + K).standard_normal((M, K)).astype(np.float32)
            if K >= 800:
                a[:, : K // 4] = edge_activations(M, K // 4, 3)
            assert bits_equal(qlc.matmul_dev(h, a, N), oracle.matmul(qw, sc, qz, N, K, 4, a, hi_prec=hp)), M
            if hp:
                hi, lo, _ = oracle.quantize_i16(a)
                assert np.array_equal(qlc.block_sums_dev(h, a, N, K), oracle.block_sums(qw, qz, N, K, 4, hi, lo))
    finally:
        qlc.free(h)


@pytest.mark.parametrize("zp,half", [(False, True), (True, True), (True, False), (False, False)])
@pytest.mark.parametrize("hp", [True, False])
@pytest.mark.parametrize("N,K", [(16, 32), (48, 800), (1040, 5120), (5120, 17408)])
def test_dp4a_chain_kernel(zp, half, hp, N, K, oracle):
    """INT4 at one and two tokens on layers of fewer than 8192 rows run the
    chain variant of the dp4a decode kernel (one row group per CTA, f values
    through a shared-memory ring, one warp running the ordered FP32 chain):
    bit-exact against the oracle from one row group and one block up to the
    27B-class down projection (17408 x 5120), with explicit zero points,
    fp16/fp32 scales, both activation modes and edge-valued activations."""
    from cases import edge_activations
    qw, sc, qz = _weights(N, K, 4, zp, half, N + K + 2 * zp + half)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    qlc.set_hi_prec(hp)
    try:
        for M in (1, 2):
            a = np.random.default_rng(M + K).standard_normal((M, K)).astype(np.float32)
            if K >= 800:
                a[:, : K // 4] = edge_activations(M, K // 4, 3)
            assert bits_equal(qlc.matmul_dev(h, a, N), oracle.matmul(qw, sc, qz, N, K, 4, a, hi_prec=hp)), M
    finally:
        qlc.free(h)
        qlc.set_hi_prec(False)


@pytest.mark.parametrize("cfg", ["1,4,16,4,4,1", "2,4,16,0,0,2", "4,4,16,0,0,4", "1,2,5,2,2,2", "2,8,7,8,8,4",
                                 "4,1,3,1,1,1", "1,3,16,6,3,3", "4,4,24,4,4,2", "1,4,32,0,8,4", "1,4,8,12,4,3"])
@pytest.mark.parametrize("N", [1008, 8208])
def test_dp4a_chain_configs(cfg, N, oracle, monkeypatch):
    """Every carve-up of the chain kernel gives the same bits: one, two or
    four row groups per CTA (a partial last CTA when N / 16 is not a multiple),
    one to eight consumer warps, one to four producer warps, stages of 3 to
    32 blocks (partial last stages), rings from one slot to twelve that wrap
    many times; on a small layer and, forced with BREEZE_QL_DP4A_KERNEL=chain,
    on a wide one."""
    K = 2848                        # 89 blocks: no stage size divides it
    qw, sc, qz = _weights(N, K, 4, True, True, 9)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    qlc.set_hi_prec(True)
    monkeypatch.setenv("BREEZE_QL_DP4A_KERNEL", "chain")
    monkeypatch.setenv("BREEZE_QL_DP4A_CHAIN", cfg)
    try:
        for M in (1, 2):
            a = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
            assert bits_equal(qlc.matmul_dev(h, a, N), oracle.matmul(qw, sc, qz, N, K, 4, a, hi_prec=True)), M
    finally:
        qlc.free(h)
        qlc.set_hi_prec(False)


@pytest.mark.parametrize("bits,half", [(8, False), (8, True), (4, True)])
@pytest.mark.parametrize("cfg", ["0,0,0,0,2", "0,0,0,0,4", "4,1,0,0,4", "1,4,0,0,2", "2,2,0,0,4", "1,2,0,0,4"])
def test_decode_kernel_producers(bits, half, cfg, oracle, monkeypatch):
    """The tensor-core decode kernel with two or four producer warps (each
    issuing every PROD-th stage of the ring) gives the same bits at 1, 5, 16
    and 64 tokens, with and without a K split (partial last stages: 159
    blocks)."""
    N, K = 208, 5088
    monkeypatch.setenv("BREEZE_QL_DECODE_CONFIG", cfg)
    monkeypatch.setenv("BREEZE_QL_DECODE_DP4A", "0")
    qw, sc, qz = _weights(N, K, bits, False, half, 11 + bits)
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    qlc.set_hi_prec(True)
    try:
        for M in (1, 5, 16, 64):
            a = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
            assert bits_equal(qlc.matmul_dev(h, a, N), oracle.matmul(qw, sc, qz, N, K, bits, a, hi_prec=True)), M
    finally:
        qlc.free(h)
        qlc.set_hi_prec(False)


@pytest.mark.parametrize("cfg", ["0,0,0,0,2", "0,0,0,0,4", "1,2,8,4,2", "2,4,8,8,4", "1,4,16,4,4", "1,1,5,2,2"])
@pytest.mark.parametrize("N", [8208, 1008])
def test_dp4a_relay_producers(cfg, N, oracle, monkeypatch):
    """The relay variant of the dp4a decode kernel with one to four producer
    warps (each issuing every PROD-th stage) gives the same bits at one and two
    tokens: a wide layer (a partial last quad) and, forced with
    BREEZE_QL_DP4A_KERNEL=relay, a small one; 89 blocks, so stages end
    partial."""
    K = 2848
    qw, sc, qz = _weights(N, K, 4, True, True, 13)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    qlc.set_hi_prec(True)
    monkeypatch.setenv("BREEZE_QL_DP4A_KERNEL", "relay")
    monkeypatch.setenv("BREEZE_QL_DP4A_CONFIG", cfg)
    try:
        for M in (1, 2):
            a = np.random.default_rng(M + 3).standard_normal((M, K)).astype(np.float32)
            assert bits_equal(qlc.matmul_dev(h, a, N), oracle.matmul(qw, sc, qz, N, K, 4, a, hi_prec=True)), M
    finally:
        qlc.free(h)
        qlc.set_hi_prec(False)
