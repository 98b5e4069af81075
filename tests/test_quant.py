"""The RTN MatMulNBits packer (CPU only): layout, round trip, reference acceptance."""
import numpy as np
import pytest

from breeze_engine_b200.quant import (dequantize_matmul_nbits, quantize_matmul_nbits,
                                      quantize_matmul_nbits_torch)
from oracle.oracle import Reference


@pytest.mark.parametrize("bits,symmetric,per_channel", [(4, True, False), (4, False, False),
                                                        (8, True, False), (8, True, True)])
def test_packer_layout_and_round_trip(bits, symmetric, per_channel):
    rng = np.random.default_rng(bits)
    K, N = 256, 48
    w = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    qw, sc, qz = quantize_matmul_nbits(w, bits=bits, symmetric=symmetric, per_channel=per_channel)
    nblk = K // 32
    assert qw.dtype == np.uint8 and qw.shape == (N, nblk, 4 * bits)
    assert sc.dtype == np.float16 and sc.shape == (N * nblk,)
    if bits == 4 and not symmetric:
        assert qz.dtype == np.uint8 and qz.shape == (N * ((nblk + 1) // 2),)
    else:
        assert qz is None
    if per_channel:
        s = sc.reshape(N, nblk)
        assert (s == s[:, :1]).all()
    deq = dequantize_matmul_nbits(qw, sc, qz, bits=bits, block_size=32, K=K, N=N)
    step = np.repeat(sc.astype(np.float32).reshape(N, nblk), 32, axis=1).T   # [K, N]
    # half a step for symmetric codes; a rounded zero point can clip one extra step
    bound = 0.5 if symmetric else 1.0
    assert np.all(np.abs(deq - w) <= bound * step * (1 + 1e-3) + 1e-12)


def test_torch_packer_matches_numpy():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(7)
    w = rng.normal(0, 0.02, (512, 64)).astype(np.float32)
    for bits, pc in ((4, False), (8, False), (8, True)):
        a = quantize_matmul_nbits(w, bits=bits, per_channel=pc)
        b = quantize_matmul_nbits_torch(torch.from_numpy(w), bits=bits, per_channel=pc)
        assert np.array_equal(a[0], b[0].numpy())
        assert np.array_equal(a[1].view(np.uint16), b[1].numpy().view(np.uint16))


@pytest.mark.skipif(not Reference.available(), reason="oracle/_ref not built")
def test_reference_prepack_accepts_packer_output():
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (128, 32)).astype(np.float32)
    ref = Reference()
    for bits, sym in ((4, True), (4, False), (8, True)):
        qw, sc, qz = quantize_matmul_nbits(w, bits=bits, symmetric=sym)
        h = ref.prepack(qw, sc, qz, 128, 32, bits)
        a = rng.standard_normal((2, 128)).astype(np.float32)
        c = ref.matmul(h, a, 32, hi_prec=True, threads=1)
        ref.free(h)
        dense = a @ dequantize_matmul_nbits(qw, sc, qz, bits=bits, block_size=32, K=128, N=32)
        cos = float((c * dense).sum() / (np.linalg.norm(c) * np.linalg.norm(dense)))
        assert cos > 0.9999
