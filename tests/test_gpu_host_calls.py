"""Repeated synchronous host-pointer calls (``i4_matmul``) on pinned buffers.

A decoder calls ``i4_matmul`` with the same weight, token count and pinned
scratch rows every step: new data in the same buffers must give new, exact
results on every call -- one output copy, column-chunked outputs whose copies
overlap the next chunk's matmul, and the prefill path -- across activation
modes, and a weight freed and re-packed behind the same buffers (its handle
may reuse the freed one's address) must compute with its own records.  Every
result is compared bit for bit with the oracle or the device entry point.
"""
import ctypes

import numpy as np
import pytest

import qlc
from breeze_engine_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _pack(N, K, bits, seed):
    rng = np.random.default_rng(seed)
    qw = rng.integers(0, 256, (N, K // 32, 4 * bits), dtype=np.uint8)
    sc = rng.uniform(1e-3, 2e-2, (N, K // 32)).astype(np.float16)
    return qw, sc, qlc.prepack(qw, sc, None, N, K, bits)


@pytest.mark.parametrize("M,N,K,bits", [
    (1, 4096, 512, 8),        # one copy out, decode kernel
    (2, 8192, 256, 4),        # INT4 dp4a decode
    (16, 32768, 256, 8),      # 2 MB of output: column chunks with overlapped copies
    (128, 4096, 512, 4),      # prefill on FP16 operands, 2 MB chunked output
])
def test_repeated_pinned_calls_are_exact(M, N, K, bits, oracle):
    import torch
    lib = L.load()
    qw, sc, h = _pack(N, K, bits, M + N)
    a = torch.empty((M, K), dtype=torch.float32).pin_memory()
    c = torch.empty((M, N), dtype=torch.float32).pin_memory()
    rng = np.random.default_rng(7)
    try:
        for hp in (True, False, True):
            qlc.set_hi_prec(hp)
            for it in range(4):
                a.copy_(torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)))
                c.fill_(-1.0)
                lib.i4_matmul(ctypes.c_void_p(h), ctypes.c_void_p(a.data_ptr()), M, ctypes.c_void_p(c.data_ptr()))
                assert lib.ql_last_status() == 0, (hp, it)
                want = oracle.matmul(qw, sc, None, N, K, bits, a.numpy(), hi_prec=hp)
                assert np.array_equal(c.numpy().view(np.uint32), want.view(np.uint32)), (hp, it)
    finally:
        qlc.free(h)
        qlc.set_hi_prec(False)
        assert lib.ql_device_error(1) == 0


def test_repacked_weight_behind_the_same_buffers():
    """A new weight behind the same pinned buffers (its handle may even reuse
    the freed one's address) computes with its own records."""
    import torch
    lib = L.load()
    M, N, K = 4, 2048, 512
    a = torch.randn((M, K), dtype=torch.float32).pin_memory()
    c = torch.empty((M, N), dtype=torch.float32).pin_memory()
    qlc.set_hi_prec(True)
    try:
        outs = []
        for seed in (1, 2, 3):
            qw, sc, h = _pack(N, K, 8, seed)
            try:
                for _ in range(3):
                    lib.i4_matmul(ctypes.c_void_p(h), ctypes.c_void_p(a.data_ptr()), M, ctypes.c_void_p(c.data_ptr()))
                    assert lib.ql_last_status() == 0
                want = qlc.matmul_dev(h, a.numpy(), N)
                assert np.array_equal(c.numpy().view(np.uint32), want.view(np.uint32)), seed
                outs.append(c.numpy().copy())
            finally:
                qlc.free(h)
        assert not np.array_equal(outs[0], outs[1])
    finally:
        qlc.set_hi_prec(False)


@pytest.mark.parametrize("bits", [8, 4])
def test_pinned_input_aligned_or_not(bits, oracle):
    """A pinned, 16-byte aligned A is read by the quantizer directly (no copy
    in); one that starts 4 bytes into its allocation is copied in as usual;
    pageable A is copied in.  Same bits every way."""
    import torch
    lib = L.load()
    M, N, K = 3, 4096, 512
    qw, sc, h = _pack(N, K, bits, 11)
    buf = torch.empty(M * K + 8, dtype=torch.float32).pin_memory()
    c = torch.empty((M, N), dtype=torch.float32).pin_memory()
    rng = np.random.default_rng(5)
    qlc.set_hi_prec(True)
    try:
        for off in (0, 1, 4, None):
            x = rng.standard_normal((M, K)).astype(np.float32)
            if off is None:
                a_ptr, keep = x.ctypes.data, x                       # pageable
            else:
                a = buf[off:off + M * K].view(M, K)
                a.copy_(torch.from_numpy(x))
                a_ptr, keep = a.data_ptr(), a
            c.fill_(-1.0)
            lib.i4_matmul(ctypes.c_void_p(h), ctypes.c_void_p(a_ptr), M, ctypes.c_void_p(c.data_ptr()))
            assert lib.ql_last_status() == 0, off
            want = oracle.matmul(qw, sc, None, N, K, bits, x, hi_prec=True)
            assert np.array_equal(c.numpy().view(np.uint32), want.view(np.uint32)), off
            del keep
    finally:
        qlc.free(h)
        qlc.set_hi_prec(False)
