"""GPU parity of the Python call surface the reference's callers use.

* ``backend.prepack`` with torch CUDA tensors runs ``ql_prepack_onnx_dev``
  (the path every bench weight takes): its packed bytes must equal those of
  the host entry ``i4_prepack_onnx`` and its outputs the oracle's.
* ``breeze_engine_b200.cpu_backend`` imported the way ``breeze/ops.py:118-131``
  (``_matmul_nbits``) and ``breeze/qwen35_cpu.py:71-89`` use
  ``breeze.cpu_backend``: ``prepack(qweight, scales, qzeros, K, N, bits=,
  block_size=)``, ``matmul(handle, a2d, N)`` on a reshaped activation, ``free``.
* ``linear.backend/prepare_weight/linear`` (``breeze/linear.py:25-46``), with
  MatMulNBits tuples and dense weights, NumPy and torch CUDA activations.

Every output is compared bit for bit with the oracle (NaN positions only).
"""
import ctypes

import numpy as np
import pytest

import qlc
from conftest import bits_equal

pytestmark = pytest.mark.gpu

_vp = ctypes.c_void_p


@pytest.fixture(autouse=True)
def _mode_reset():
    yield
    qlc.set_hi_prec(False)
    assert qlc.device_error() == 0


def _rtn(K, N, bits, seed, symmetric=True):
    from breeze_engine_b200.quant import quantize_matmul_nbits
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    return quantize_matmul_nbits(w, bits=bits, symmetric=symmetric, per_channel=bits == 8)


def _serialized(h):
    lib = qlc.lib()
    n = lib.ql_weight_serialized_bytes(_vp(h))
    buf = np.empty(n, np.uint8)
    assert lib.ql_weight_serialize(_vp(h), buf.ctypes.data, n) == 0
    return buf


@pytest.mark.parametrize("bits,symmetric,half", [(4, True, True), (4, False, True), (4, False, False),
                                                 (8, True, True), (8, True, False)])
def test_device_prepack_matches_host_prepack_and_oracle(bits, symmetric, half, oracle):
    """``backend.prepack`` on CUDA tensors (``ql_prepack_onnx_dev``): the packed
    records are byte-identical to the host entry's, and matmuls through the
    handle match the oracle at decode and prefill token counts."""
    import torch
    from breeze_engine_b200 import backend
    K, N = 640, 272
    qw, sc, qz = _rtn(K, N, bits, 100 + bits + 2 * symmetric, symmetric=symmetric)
    if not half:
        sc = sc.astype(np.float32)
    if bits == 8:
        qz = None
    h_host = backend.prepack(qw, sc, qz, K, N, bits=bits)
    h_dev = backend.prepack(torch.from_numpy(qw).cuda(), torch.from_numpy(sc).cuda(),
                            None if qz is None else torch.from_numpy(qz).cuda(), K, N, bits=bits)
    try:
        assert np.array_equal(_serialized(h_dev), _serialized(h_host))
        rng = np.random.default_rng(5)
        for hp in (True, False):
            backend.set_hi_prec(hp)
            for M in (1, 7, 130):
                a = rng.standard_normal((M, K)).astype(np.float32)
                got = backend.matmul(h_dev, torch.from_numpy(a).cuda(), N)
                torch.cuda.synchronize()
                expect = oracle.matmul(qw, sc, qz, N, K, bits, a, hi_prec=hp)
                assert bits_equal(got.cpu().numpy(), expect), (hp, M)
    finally:
        backend.free(h_host)
        backend.free(h_dev)


def test_cpu_backend_as_the_reference_callers_use_it(oracle):
    """The ``_matmul_nbits`` pattern of ``breeze/ops.py:118-131``: a
    ``[batch, seq, K]`` activation reshaped to 2-D, ``cpu_backend.matmul``,
    reshaped back; prepack keyword arguments as ``Qwen35CpuModel._build``
    passes them (``breeze/qwen35_cpu.py:78-80``)."""
    from breeze_engine_b200 import cpu_backend
    assert cpu_backend.available()
    K, N = 512, 96
    qw, sc, qz = _rtn(K, N, 4, 3, symmetric=False)
    cpu_backend.set_threads(4)
    cpu_backend.set_hi_prec(True)
    h = cpu_backend.prepack(qw, sc, qz, int(K), int(N), bits=4, block_size=32)
    assert h
    try:
        a = np.random.default_rng(1).standard_normal((2, 3, K)).astype(np.float32)
        a2d = a.reshape(-1, a.shape[-1])
        out = cpu_backend.matmul(h, a2d, N).reshape(*a.shape[:-1], N)
        assert out.shape == (2, 3, N) and out.dtype == np.float32
        assert bits_equal(out.reshape(-1, N), oracle.matmul(qw, sc, qz, N, K, 4, a2d))
        with pytest.raises(ValueError):
            cpu_backend.prepack(qw, sc, qz, K, N, bits=4, block_size=64)
    finally:
        cpu_backend.free(h)


@pytest.mark.parametrize("hp", [True, False])
def test_linear_surface(hp, oracle):
    """``linear.prepare_weight`` with a MatMulNBits tuple and with a dense
    ``[K, N]`` weight (packed by the RTN packer), ``linear.linear`` on NumPy and
    torch CUDA activations with leading dimensions."""
    import torch
    from breeze_engine_b200 import backend, linear
    from breeze_engine_b200.quant import quantize_matmul_nbits
    assert linear.backend() == "cuda-sm100a-quantized"
    backend.set_hi_prec(hp)
    K, N = 256, 160
    rng = np.random.default_rng(9)
    qw, sc, qz = _rtn(K, N, 4, 11, symmetric=False)
    w4 = linear.prepare_weight((qw, sc, qz, K, N, 4))
    dense = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    w8 = linear.prepare_weight(dense)                      # 8-bit per-channel RTN
    q8, s8, z8 = quantize_matmul_nbits(dense, bits=8, symmetric=True, per_channel=True)
    try:
        assert w4.shape == (K, N) and w8.bits == 8
        a = rng.standard_normal((3, 5, K)).astype(np.float32)
        got = linear.linear(a, w4)
        assert got.shape == (3, 5, N)
        assert bits_equal(got.reshape(-1, N), oracle.matmul(qw, sc, qz, N, K, 4, a.reshape(-1, K), hi_prec=hp))
        got8 = linear.linear(torch.from_numpy(a).cuda(), w8)
        torch.cuda.synchronize()
        assert tuple(got8.shape) == (3, 5, N)
        assert bits_equal(got8.cpu().numpy().reshape(-1, N),
                          oracle.matmul(q8, s8, None, N, K, 8, a.reshape(-1, K), hi_prec=hp))
    finally:
        w4.close()
        w8.close()
