"""Failure detection on one GPU without a GPU fault.

A bounded wait is made to run out on purpose: the peer exchange waits for a
flag that nothing sets.  A second process on the same GPU only allocates an
exchange region and shares its CUDA IPC handle; it never calls the gather, so
this process's gather waits for a peer that never posts.  With the peer wait
limit set to 200 ms the kernel gives up, records QL_ETIMEOUT in the device
error word and returns; the host sees the code, promptly.  Only one kernel
ever waits (no two launches depend on each other), nothing traps and no
address is invalid.

The same expired wait then checks the reporting of the synchronous host entry
point: ``i4_matmul`` reads the device error word after its work, reports it
through ``ql_last_status()`` and clears it, so the following call is clean.
"""
import ctypes
import os
import subprocess
import sys
import textwrap
import time

import numpy as np
import pytest

import qlc
from breeze_engine_b200 import _lib as L

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# The silent peer: allocates an exchange region on cuda:0, prints its IPC
# handle, waits for a line on stdin, frees the region and exits.
_PEER = textwrap.dedent("""
    import ctypes, sys
    sys.path.insert(0, {root!r})
    from breeze_engine_b200 import _lib as L
    lib = L.load()
    h = (ctypes.c_uint8 * 64)()
    x = ctypes.c_void_p()
    rc = lib.ql_peer_exchange_create(1 << 16, ctypes.byref(h), ctypes.byref(x))
    print(("OK " + bytes(h).hex()) if rc == 0 else ("ERR %d" % rc), flush=True)
    sys.stdin.readline()
    lib.ql_peer_exchange_destroy(x)
""")


@pytest.fixture
def silent_peer():
    proc = subprocess.Popen([sys.executable, "-c", _PEER.format(root=ROOT)], stdin=subprocess.PIPE,
                            stdout=subprocess.PIPE, text=True)
    try:
        line = proc.stdout.readline().split()
        assert line and line[0] == "OK", line
        yield bytes.fromhex(line[1])
    finally:
        try:
            proc.stdin.write("\n")
            proc.stdin.flush()
            proc.wait(timeout=60)
        except Exception:  # noqa: BLE001 - make sure the child is gone
            proc.kill()


def test_peer_wait_runs_out_and_is_reported(silent_peer, oracle):
    import torch
    torch.cuda.set_device(0)
    lib = L.load()
    assert lib.ql_device_error(1) == 0
    own = (ctypes.c_uint8 * 64)()
    x = ctypes.c_void_p()
    assert lib.ql_peer_exchange_create(1 << 16, ctypes.byref(own), ctypes.byref(x)) == 0
    h = None
    try:
        handles = (ctypes.c_uint8 * 128).from_buffer_copy(bytes(own) + silent_peer)
        assert lib.ql_peer_exchange_connect(x, 0, 2, ctypes.byref(handles)) == 0
        assert lib.ql_set_wait_limits(0, 200_000_000) == 0          # 200 ms for peer flags
        shard = torch.ones((4, 64), dtype=torch.float32, device="cuda")
        t0 = time.perf_counter()
        assert lib.ql_peer_allgather_cols_dev(x, ctypes.c_void_p(shard.data_ptr()), 4, 64,
                                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert elapsed < 3.0, elapsed                                 # two 200 ms waits, not 5 s
        assert lib.ql_device_error(0) == L.QL_ETIMEOUT                # read, left set

        # i4_matmul reads the word after its work: it reports the expired wait
        # and clears it; the next call is clean and its output exact.
        rng = np.random.default_rng(3)
        K, N = 256, 64
        qw = rng.integers(0, 256, (N, K // 32, 16), dtype=np.uint8)
        sc = rng.uniform(1e-3, 2e-2, (N, K // 32)).astype(np.float16)
        h = qlc.prepack(qw, sc, None, N, K, 4)
        qlc.set_hi_prec(True)
        a = rng.standard_normal((2, K)).astype(np.float32)
        c = np.zeros((2, N), np.float32)
        lib.i4_matmul(ctypes.c_void_p(h), a.ctypes.data, 2, c.ctypes.data)
        assert lib.ql_last_status() == L.QL_ETIMEOUT
        assert lib.ql_device_error(0) == 0
        c = qlc.matmul_host(h, a, N)                                  # asserts status OK
        assert np.array_equal(c.view(np.uint32), oracle.matmul(qw, sc, None, N, K, 4, a).view(np.uint32))
    finally:
        lib.ql_set_wait_limits(L.DEFAULT_WAIT_NS, L.DEFAULT_PEER_WAIT_NS)
        if h is not None:
            qlc.free(h)
        qlc.set_hi_prec(False)
        lib.ql_peer_exchange_destroy(x)
        lib.ql_device_error(1)


def test_backend_check_device_raises_on_a_set_word(silent_peer):
    """backend.check_device / PeerExchange-style checks raise QLError(QL_ETIMEOUT)."""
    import torch
    from breeze_engine_b200 import backend
    torch.cuda.set_device(0)
    lib = L.load()
    own = (ctypes.c_uint8 * 64)()
    x = ctypes.c_void_p()
    assert lib.ql_peer_exchange_create(1 << 16, ctypes.byref(own), ctypes.byref(x)) == 0
    try:
        handles = (ctypes.c_uint8 * 128).from_buffer_copy(bytes(own) + silent_peer)
        assert lib.ql_peer_exchange_connect(x, 0, 2, ctypes.byref(handles)) == 0
        backend.set_wait_limits(peer_wait_ns=100_000_000)
        shard = torch.ones((1, 16), dtype=torch.float32, device="cuda")
        assert lib.ql_peer_allgather_cols_dev(x, ctypes.c_void_p(shard.data_ptr()), 1, 16,
                                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        with pytest.raises(L.QLError) as ei:
            backend.check_device("gather")
        assert ei.value.code == L.QL_ETIMEOUT
        backend.check_device()                                        # cleared
    finally:
        backend.set_wait_limits(L.DEFAULT_WAIT_NS, L.DEFAULT_PEER_WAIT_NS)
        lib.ql_peer_exchange_destroy(x)
        lib.ql_device_error(1)
