"""GPU parity of the 27B-class decoder-layer projection set (configs[3] of the benchmark spec).

Hidden size 5120, INT4 weights (N(0, 0.02), RTN-packed with fp16 scales):
Q 5120x6144, K 5120x1024, V 5120x1024, O 6144x5120, gate/up 5120x17408,
down 17408x5120, run as one sequence of 7 calls enqueued back to back on one
stream with one shared workspace (Q/K/V/gate/up read the layer input; O reads
an attention-sized input; down reads an MLP-sized one), at M = 1 and M = 512.
At M = 1 every output is compared with the oracle; at M = 512 a random sample
of 16-column groups per layer (each column slice of the MatMulNBits arrays is
an exact sub-problem).  Bit-exact, NaN positions only.
"""
import ctypes

import numpy as np
import pytest

import qlc
from conftest import bits_equal

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

H = 5120
LAYERS = [("q", H, 6144, "x"), ("k", H, 1024, "x"), ("v", H, 1024, "x"), ("o", 6144, H, "attn"),
          ("gate", H, 17408, "x"), ("up", H, 17408, "x"), ("down", 17408, H, "mlp")]


@pytest.fixture(scope="module")
def layer_set():
    from breeze_engine_b200.quant import quantize_matmul_nbits
    out = {}
    for i, (name, K, N, _) in enumerate(LAYERS):
        rng = np.random.default_rng(2700 + i)
        w = rng.normal(0, 0.02, (K, N)).astype(np.float32)
        out[name] = quantize_matmul_nbits(w, bits=4, symmetric=True)
    return out


@pytest.mark.parametrize("M", [1, 512])
def test_layer_set_seven_calls(M, layer_set, oracle):
    import torch
    lib = qlc.lib()
    rng = np.random.default_rng(M)
    inputs = {"x": rng.standard_normal((M, H)).astype(np.float32),
              "attn": rng.standard_normal((M, 6144)).astype(np.float32),
              "mlp": rng.standard_normal((M, 17408)).astype(np.float32)}
    handles = {}
    qlc.set_hi_prec(True)
    try:
        for name, K, N, _ in LAYERS:
            qw, sc, qz = layer_set[name]
            handles[name] = qlc.prepack(qw, sc, qz, N, K, 4)
        dev_in = {k: torch.from_numpy(v).cuda() for k, v in inputs.items()}
        outs = {name: torch.full((M, N), -1.0, device="cuda") for name, _, N, _ in LAYERS}
        need = max(lib.ql_workspace_bytes(ctypes.c_void_p(handles[n]), M) for n, _, _, _ in LAYERS)
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        for name, K, N, src in LAYERS:          # one sequence, one stream, no sync in between
            rc = lib.ql_matmul_dev_ws(ctypes.c_void_p(handles[name]), dev_in[src].data_ptr(), M,
                                      outs[name].data_ptr(), ws.data_ptr(), need, s)
            assert rc == 0, lib.ql_error_string(rc)
        torch.cuda.synchronize()
        assert qlc.device_error() == 0
        for name, K, N, src in LAYERS:
            qw, sc, qz = layer_set[name]
            got = outs[name].cpu().numpy()
            if M == 1:
                expect = oracle.matmul(qw, sc, qz, N, K, 4, inputs[src])
                assert bits_equal(got, expect), name
                continue
            nblk = K // 32
            for g in np.sort(rng.choice(N // 16, size=4, replace=False)):
                rows = slice(16 * g, 16 * g + 16)
                expect = oracle.matmul(qw.reshape(N, -1)[rows], sc.reshape(N, nblk)[rows], None, 16, K, 4,
                                       inputs[src])
                assert bits_equal(got[:, rows], expect), (name, int(g))
    finally:
        for h in handles.values():
            qlc.free(h)
        qlc.set_hi_prec(False)
