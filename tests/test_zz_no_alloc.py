"""ql_matmul_dev_noalloc: the entry point for callers that cannot allocate
device memory when they run a layer (under a serving runtime whose allocator
owns all of HBM, or in a per-token loop that cannot pay for an allocation or
the synchronisation a free implies).  It keeps the quantized activations in a
fixed scratch array compiled into the library instead of a caller or library
workspace.

The test drives it through the C ABI and compares it with the workspace entry
point (ql_matmul_dev_ws) and with the oracle on calls in a row, over the
decode kernel (M <= 64) and the tensor-core GEMM (M > 64, which also fits the
scratch at K = 4096); outputs must be bit-identical, the same bar as every
other parity test here.  The file is named so pytest collects it last, and it
needs no state from earlier tests.
"""
import ctypes

import numpy as np
import pytest

import qlc
from conftest import bits_equal

pytestmark = pytest.mark.gpu

_vp = ctypes.c_void_p


def _noalloc(h, a, N):
    import torch
    lib = qlc.lib()
    dA = torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    dC = torch.full((a.shape[0], N), -12345.0, dtype=torch.float32, device="cuda")
    rc = lib.ql_matmul_dev_noalloc(_vp(h), dA.data_ptr(), a.shape[0], dC.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, dC.cpu().numpy()


def test_noalloc_matches_workspace_entry_point_on_two_calls(oracle):
    from breeze_engine_b200.quant import quantize_matmul_nbits
    rng = np.random.default_rng(42)
    K, N = 4096, 1024
    w = rng.normal(0, 0.02, (K, N)).astype(np.float32)
    qw, sc, qz = quantize_matmul_nbits(w, bits=4)
    h = qlc.prepack(qw, sc, qz, N, K, 4)
    qlc.set_hi_prec(True)
    try:
        # calls in a row: each reuses the scratch the previous one left behind;
        # 128 tokens take the tensor-core GEMM, whose records also fit
        for M in (16, 3, 128, 128):
            assert qlc.lib().ql_act_workspace_bytes(M, K) <= 8 << 20     # the records the scratch holds
            a = rng.standard_normal((M, K)).astype(np.float32)
            rc, got = _noalloc(h, a, N)
            assert rc == 0, qlc.lib().ql_error_string(rc)
            assert bits_equal(got, qlc.matmul_dev(h, a, N))
            assert bits_equal(got, oracle.matmul(qw, sc, qz, N, K, 4, a))
        assert qlc.device_error() == 0
    finally:
        qlc.free(h)
        qlc.set_hi_prec(False)


def test_noalloc_rejects_requests_beyond_its_scratch():
    rng = np.random.default_rng(7)
    K, N = 4096, 64
    qw = rng.integers(0, 256, (N, K // 32, 16), dtype=np.uint8)
    sc = rng.uniform(1e-3, 2e-2, (N, K // 32)).astype(np.float16)
    h = qlc.prepack(qw, sc, None, N, K, 4)
    try:
        M = 4096   # needs more than the 8 MiB scratch
        assert qlc.lib().ql_workspace_bytes(_vp(h), M) > 8 << 20
        rc, out = _noalloc(h, np.zeros((M, K), np.float32), N)
        assert rc == 7                     # QL_ESCRATCH
        assert (out == -12345.0).all()     # nothing was launched
    finally:
        qlc.free(h)
