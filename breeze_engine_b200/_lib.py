"""ctypes binding of libbreeze_ql.so (the C ABI in include/breeze_ql.h).

The library path defaults to the in-tree build next to this file and can be
overridden with ``BREEZE_B200_KERNEL`` (the counterpart of the reference's
``BREEZE_KERNEL``, ``breeze/cpu_backend.py:11``).  There is no fallback: if
the library cannot be loaded every compute entry point raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("BREEZE_B200_KERNEL", os.path.join(HERE, "libbreeze_ql.so"))

QL_OK, QL_EINVAL, QL_ENOMEM, QL_ECUDA, QL_ETIMEOUT, QL_EDEVICE, QL_ENOTSUP, QL_ESCRATCH = range(8)
DEFAULT_WAIT_NS = 1_000_000_000        # QL_DEFAULT_WAIT_NS of include/breeze_ql.h
DEFAULT_PEER_WAIT_NS = 5_000_000_000   # QL_DEFAULT_PEER_WAIT_NS

_vp = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t

# (name, restype, argtypes) for every symbol declared in include/breeze_ql.h.
SIGNATURES = [
    ("i4_set_threads", None, [_i]),
    ("i4_set_numa_split", None, [_i]),
    ("i4_set_hi_prec", None, [_i]),
    ("i4_prepack_onnx", _vp, [_vp, _vp, _vp, _i, _i, _i, _i]),
    ("i4_prepack", _vp, [_vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    ("i4_free", None, [_vp]),
    ("i4_matmul", None, [_vp, _vp, _i, _vp]),
    ("i4_matmul_region", None, [_vp, _vp, _i, _vp, _vp, _vp]),
    ("ql_version", _i, []),
    ("ql_device_count", _i, []),
    ("ql_get_hi_prec", _i, []),
    ("ql_set_prefill_kernel", _i, [_i]),
    ("ql_last_status", _i, []),
    ("ql_error_string", ctypes.c_char_p, [_i]),
    ("ql_last_cuda_error_string", ctypes.c_char_p, []),
    ("ql_device_error", _i, [_i]),
    ("ql_set_wait_limits", _i, [ctypes.c_ulonglong, ctypes.c_ulonglong]),
    ("ql_prepack_onnx_dev", _i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, ctypes.POINTER(_vp)]),
    ("ql_weight_info", _i, [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i),
                            ctypes.POINTER(_i), ctypes.POINTER(ctypes.c_ulonglong)]),
    ("ql_workspace_bytes", _sz, [_vp, _i]),
    ("ql_matmul_dev_ws", _i, [_vp, _vp, _i, _vp, _vp, _sz, _vp]),
    ("ql_matmul_dev", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ql_matmul_dev_noalloc", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ql_act_workspace_bytes", _sz, [_i, _i]),
    ("ql_quantize_act_dev", _i, [_vp, _i, _i, _i, _vp, _sz, _vp]),
    ("ql_matmul_quantized_dev", _i, [_vp, _vp, _i, _i, _vp, _vp]),
    ("ql_norm_act_workspace_bytes", _sz, [_i, _i]),
    ("ql_quantize_act_rmsnorm_dev", _i, [_vp, _vp, ctypes.c_float, _i, _i, _i, _vp, _sz, _vp, _vp]),
    ("ql_matmul_rmsnorm_dev", _i, [_vp, _vp, _vp, ctypes.c_float, _i, _vp, _vp]),
    ("ql_quantize_act_silu_mul_dev", _i, [_vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp, _vp]),
    ("ql_matmul_silu_mul_dev", _i, [_vp, _vp, _vp, _i, _i, _vp, _vp]),
    ("ql_weight_concat", _i, [ctypes.POINTER(_vp), _i, ctypes.POINTER(_vp)]),
    ("ql_peer_exchange_create", _i, [_sz, _vp, ctypes.POINTER(_vp)]),
    ("ql_peer_exchange_connect", _i, [_vp, _i, _i, _vp]),
    ("ql_peer_exchange_output", _vp, [_vp]),
    ("ql_peer_allgather_cols_dev", _i, [_vp, _vp, _i, _i, _vp]),
    ("ql_peer_exchange_destroy", _i, [_vp]),
    ("ql_weight_serialized_bytes", _sz, [_vp]),
    ("ql_weight_serialize", _i, [_vp, _vp, _sz]),
    ("ql_weight_deserialize", _i, [_vp, _sz, ctypes.POINTER(_vp)]),
    ("ql_block_sums_dev", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ql_prefill_gemm_dev", _i, [_vp, _vp, _sz, _i, _i, _vp, _vp]),
    ("ql_quantize_dev", _i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
]

_lib = None
_load_error = None


def load(path=None):
    """Load (once) and return the library; raises RuntimeError if unavailable."""
    global _lib, _load_error
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    try:
        lib = ctypes.CDLL(p)
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
    except (OSError, AttributeError) as exc:
        _load_error = f"{p}: {exc}"
        raise RuntimeError(f"breeze_engine_b200 CUDA library unavailable ({_load_error}); "
                           "build it with `python -m breeze_engine_b200.build`") from exc
    if path is None:
        _lib = lib
    return lib


def try_load():
    try:
        return load()
    except RuntimeError:
        return None


class QLError(RuntimeError):
    def __init__(self, code, what=""):
        lib = try_load()
        msg = lib.ql_error_string(code).decode() if lib else str(code)
        detail = ""
        if lib is not None and code == QL_ECUDA:
            detail = ": " + lib.ql_last_cuda_error_string().decode()
        super().__init__(f"{what}: {msg}{detail}" if what else msg + detail)
        self.code = code


def check(code, what=""):
    if code != QL_OK:
        if code == QL_ENOMEM:
            raise MemoryError(f"{what}: device allocation failed")
        if code == QL_EINVAL:
            raise ValueError(f"{what}: invalid argument")
        raise QLError(code, what)
    return code
