"""Packed-layout cache: ql_weight_serialize / ql_weight_deserialize and the
Python save_packed / load_packed helpers.

The reference repacks every MatMulNBits weight on each model load
(breeze/qwen35_cpu.py:71-89 -> kernel/quantized_matmul.cpp:505-520); here a
packed handle can be written to a file once and restored with one host ->
device copy.  A restored handle must give bit-identical outputs, and a file
from another layout version, a truncated file or a corrupted payload must be
rejected (QL_EINVAL / ValueError) before any device memory is touched.
"""
import ctypes
import struct

import numpy as np
import pytest

import qlc
from breeze_engine_b200 import _lib as L
from conftest import bits_equal

HEADER = struct.Struct("<8sII6iQQ")      # magic, version, header_bytes, N K bits half zp REC, payload, checksum


def _checksum(payload):
    """Host restatement of the header checksum (wrapping sum of 64-bit words
    times odd weights, then the tail bytes)."""
    s = 0x9E3779B97F4A7C15
    n = len(payload) // 8 * 8
    words = np.frombuffer(payload[:n], dtype=np.uint64)
    with np.errstate(over="ignore"):
        s = (s + int((words * (2 * np.arange(words.size, dtype=np.uint64) + 1)).sum(dtype=np.uint64))) % (1 << 64)
    for i in range(n, len(payload)):
        s = (s + (payload[i] << ((i & 7) * 8))) % (1 << 64)
    return s


def _blob(N=32, K=64, bits=4, half=1, zp=0, payload=None, checksum=None, magic=b"QLPACK1\0", version=1):
    rec = (256 if bits == 4 else 512) + (32 if half else 64) + (16 if zp else 0)
    size = (N // 16) * (K // 32) * rec
    if payload is None:
        payload = np.random.default_rng(0).integers(0, 256, size, dtype=np.uint8).tobytes()
    if checksum is None:
        checksum = _checksum(payload)
    return HEADER.pack(magic, version, HEADER.size, N, K, bits, half, zp, rec, size, checksum) + payload


def _deserialize(blob):
    lib = qlc.lib()
    buf = np.frombuffer(blob, dtype=np.uint8).copy()
    out = ctypes.c_void_p()
    rc = lib.ql_weight_deserialize(buf.ctypes.data, buf.size, ctypes.byref(out))
    return rc, out.value


@pytest.mark.parametrize("change", ["magic", "version", "short", "checksum", "geometry", "int8_zp"])
def test_rejects_bad_files_without_touching_the_device(change):
    """Every malformed input is refused by the header checks alone (this runs
    without a GPU: the checks precede any CUDA call)."""
    good = _blob()
    blob = {
        "magic": _blob(magic=b"QLPACK9\0"),
        "version": _blob(version=2),
        "short": good[:-1],
        "checksum": _blob(checksum=_checksum(good[HEADER.size:]) ^ 1),
        "geometry": HEADER.pack(b"QLPACK1\0", 1, HEADER.size, 32, 64, 4, 1, 0, 304, 2 * 2 * 304, 0) + bytes(1216),
        "int8_zp": _blob(bits=8, zp=1),
    }[change]
    rc, h = _deserialize(blob)
    assert rc == L.QL_EINVAL and not h


def test_header_checksum_restatement():
    """The Python restatement matches the checksum the library accepts: a
    blob built with it passes every host check and reaches the device
    allocation (which fails with QL_ENOMEM / QL_ECUDA where there is no GPU)."""
    assert HEADER.size == 56
    lib = qlc.lib()
    assert lib.ql_weight_serialized_bytes(None) == 0
    assert lib.ql_weight_serialize(None, None, 0) == L.QL_EINVAL
    rc, h = _deserialize(_blob())
    if h:
        qlc.free(h)
    assert rc in (L.QL_OK, L.QL_ENOMEM, L.QL_ECUDA), rc


@pytest.mark.gpu
@pytest.mark.parametrize("bits,zp,half", [(4, False, True), (4, True, True), (8, False, False)])
def test_roundtrip_bit_identical(bits, zp, half, oracle, tmp_path):
    from breeze_engine_b200 import backend
    rng = np.random.default_rng(bits + zp)
    N, K = 272, 320
    qw = rng.integers(0, 256, (N, K // 32, 4 * bits), dtype=np.uint8)
    sc = rng.uniform(1e-3, 2e-2, (N, K // 32)).astype(np.float16 if half else np.float32)
    qz = rng.integers(0, 256, (N, (K // 32 + 1) // 2), dtype=np.uint8) if zp else None
    h = qlc.prepack(qw, sc, qz, N, K, bits)
    path = tmp_path / "w.qlpack"
    try:
        n = backend.save_packed(h, path)
        assert n == qlc.lib().ql_weight_serialized_bytes(ctypes.c_void_p(h)) == path.stat().st_size
        h2 = backend.load_packed(path)
        try:
            qlc.set_hi_prec(True)
            for M in (1, 70):
                a = rng.standard_normal((M, K)).astype(np.float32)
                ref = qlc.matmul_dev(h, a, N)
                assert bits_equal(qlc.matmul_dev(h2, a, N), ref)
                assert bits_equal(ref, oracle.matmul(qw, sc, qz, N, K, bits, a))
            # the restored records serialise to the same bytes
            path2 = tmp_path / "w2.qlpack"
            backend.save_packed(h2, path2)
            assert path.read_bytes() == path2.read_bytes()
        finally:
            qlc.set_hi_prec(False)
            qlc.free(h2)
        blob = bytearray(path.read_bytes())
        blob[-5] ^= 0x40                                    # one payload bit
        path.write_bytes(bytes(blob))
        with pytest.raises(ValueError):
            backend.load_packed(path)
    finally:
        qlc.free(h)
