"""The C-ABI library loads, exports what include/breeze_ql.h declares, and
enforces the reference's contract checks before touching a GPU (CPU only)."""
import ctypes
import os
import re

import numpy as np
import pytest

from breeze_engine_b200 import _lib as L
from breeze_engine_b200 import backend as ib
from cases import fixture_weights

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "breeze_ql.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^[\w\s\*]+?\b(\w+)\s*\(", text, flags=re.M)) - {"if", "defined"})


def test_header_declares_the_reference_entry_points():
    names = declared_functions()
    for ref_name in ("i4_set_threads", "i4_set_numa_split", "i4_set_hi_prec", "i4_prepack_onnx",
                     "i4_prepack", "i4_free", "i4_matmul"):
        assert ref_name in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(L.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_the_header():
    bound = {name for name, _, _ in L.SIGNATURES}
    assert set(declared_functions()) == bound


def test_settings_round_trip_without_a_gpu():
    lib = L.load()
    assert lib.ql_version() >= 1
    lib.i4_set_threads(3)
    lib.i4_set_numa_split(1 << 30)
    ib.set_hi_prec(True)
    assert ib.get_hi_prec() is True
    ib.set_hi_prec(False)
    assert ib.get_hi_prec() is False
    assert lib.ql_error_string(0) == b"ok"


def test_null_safe_entry_points():
    lib = L.load()
    lib.i4_free(None)
    ib.free(0)
    assert lib.ql_workspace_bytes(None, 4) == 0
    lib.i4_matmul(None, None, 1, None)
    assert lib.ql_last_status() == L.QL_EINVAL
    assert lib.ql_matmul_dev(None, None, 1, None, None) == L.QL_EINVAL
    assert lib.ql_block_sums_dev(None, None, 1, None, None) == L.QL_EINVAL
    assert lib.ql_weight_info(None, None, None, None, None, None) == L.QL_EINVAL
    out = ctypes.c_void_p(123)
    assert lib.ql_prepack_onnx_dev(None, None, None, 16, 32, 4, 16, None, ctypes.byref(out)) == L.QL_EINVAL
    assert out.value is None


@pytest.mark.parametrize("N,K,bits,scale_bits", [(0, 32, 4, 32), (16, 0, 4, 32), (17, 32, 4, 32),
                                                 (16, 33, 4, 32), (16, 32, 3, 32), (16, 32, 4, 64)])
def test_native_rejects_bad_contract(N, K, bits, scale_bits):
    """Mirrors tests/test_cpu_packing.py:185-190 of the reference."""
    qw, sc, _ = fixture_weights(16, 32, 4, np.float32, False)
    lib = L.load()
    assert not lib.i4_prepack_onnx(qw.ctypes.data, sc.ctypes.data, None, N, K, bits, scale_bits)
    assert lib.ql_last_status() == L.QL_EINVAL      # a bad contract, not an allocation failure


def test_int8_with_zero_points_rejected_natively():
    qw, sc, _ = fixture_weights(16, 32, 8, np.float32, False)
    zeros = np.full(16, 128, np.uint8)
    assert not L.load().i4_prepack_onnx(qw.ctypes.data, sc.ctypes.data, zeros.ctypes.data, 16, 32, 8, 32)


def test_legacy_prepack_rejects_bad_contract():
    lib = L.load()
    b = np.zeros(16 * 8 * 32, np.uint8)
    s = np.zeros(16, np.float32)
    z = np.zeros(16, np.int8)
    c = np.zeros(16, np.int32)
    assert not lib.i4_prepack(b.ctypes.data, s.ctypes.data, None, c.ctypes.data, 16, 32, 1, 4)
    assert not lib.i4_prepack(b.ctypes.data, s.ctypes.data, z.ctypes.data, c.ctypes.data, 16, 32, 2, 4)
    z[3] = 16   # INT4 zero points must be 0..15
    assert not lib.i4_prepack(b.ctypes.data, s.ctypes.data, z.ctypes.data, c.ctypes.data, 16, 32, 1, 4)


@pytest.mark.parametrize("fault", ["weights", "scales", "zeros", "zero_dtype", "fractional_dim", "overflow_dim",
                                   "bool_dim", "weight_dtype"])
def test_reject_malformed_inputs(fault):
    """Mirrors tests/test_cpu_packing.py:171-182 of the reference."""
    qw, sc, qz = fixture_weights(16, 32, 4, np.float32, True)
    K, N = 32, 16
    if fault == "weights": qw = qw.reshape(-1)[:-1]
    elif fault == "scales": sc = sc.reshape(-1)[:-1]
    elif fault == "zeros": qz = qz.reshape(-1)[:-1]
    elif fault == "zero_dtype": qz = qz.astype(np.int32)
    elif fault == "fractional_dim": N = 16.0
    elif fault == "overflow_dim": K = 2**32 + 32
    elif fault == "bool_dim": N = True
    elif fault == "weight_dtype": qw = qw.astype(np.int16)
    with pytest.raises(ValueError):
        ib.prepack(qw, sc, qz, K, N)


def test_reject_quantization_mismatch():
    """Mirrors tests/test_qwen35_cpu.py:211-216 of the reference."""
    qw = np.zeros((16, 1, 32), np.uint8)
    with pytest.raises(ValueError, match="block_size"):
        ib.prepack(qw, np.ones(16), None, 32, 16, block_size=128)
    with pytest.raises(ValueError, match="zero point"):
        ib.prepack(qw, np.ones(16), np.zeros(16, np.uint8), 32, 16, bits=8)


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="unavailable"):
        L.load(str(tmp_path / "nope.so"))


def test_available_reports_no_device_on_a_cpu_host():
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        has_gpu = False
    assert ib.available() == has_gpu
