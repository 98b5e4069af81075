"""GPU quantized-linear backend with Breeze's ``cpu_backend`` call surface.

Mirrors ``breeze/cpu_backend.py:57-242`` -- ``available``, ``set_threads``,
``set_hi_prec``, ``prepack``, ``matmul``, ``free`` -- with the same argument
meaning, validation and exceptions (``ValueError`` for a contract violation,
``MemoryError`` for a null handle, ``RuntimeError`` when the native library is
unavailable), so a caller such as ``ops._matmul_nbits`` (``breeze/ops.py:118-131``)
or ``Qwen35CpuModel._build`` (``breeze/qwen35_cpu.py:71-89``) switches by
changing its import.  All arithmetic runs in libbreeze_ql.so on the GPU;
there is no CPU fallback.

Inputs may be NumPy arrays (copied to the GPU, result returned as NumPy, as
the reference does) or torch CUDA tensors (zero-copy, result returned as a
CUDA tensor on the current stream).
"""
import ctypes

import numpy as np

from . import _lib as L

_INT32_MAX = np.iinfo(np.int32).max


def _torch():
    try:
        import torch
        return torch
    except Exception:  # noqa: BLE001 - torch is optional for the NumPy path
        return None


def _is_cuda_tensor(x):
    t = _torch()
    return t is not None and isinstance(x, t.Tensor) and x.is_cuda


def available():
    """True when the CUDA library loads and a CUDA device is visible."""
    lib = L.try_load()
    return lib is not None and lib.ql_device_count() > 0


def set_threads(n):
    """Accepted for compatibility (``breeze/cpu_backend.py:61-68``); results never depend on it."""
    lib = L.try_load()
    if lib is not None:
        lib.i4_set_threads(int(n))


def set_hi_prec(on):
    """Select process-global int16 two-pass (True) versus int8 single-pass activations.

    Same contract as ``breeze/cpu_backend.py:71-78``: configure before
    inference; the setting is process-global and calls must be serialised
    against it.
    """
    lib = L.try_load()
    if lib is not None:
        lib.i4_set_hi_prec(1 if on else 0)


def get_hi_prec():
    return bool(L.load().ql_get_hi_prec())


def device_error(clear=True):
    """Synchronise the current CUDA device and return its device error word:
    0, or the code (``QL_ETIMEOUT``) a kernel recorded when one of its bounded
    waits gave up.  ``clear`` resets it.  The synchronous NumPy path of
    :func:`matmul` checks it after every call; callers of the asynchronous
    torch path check it here after they synchronise."""
    return int(L.load().ql_device_error(1 if clear else 0))


def check_device(what="device"):
    """Raise :class:`breeze_engine_b200._lib.QLError` when the device error
    word is set (and clear it)."""
    code = device_error(clear=True)
    if code:
        raise L.QLError(code, what)


def set_wait_limits(wait_ns=0, peer_wait_ns=0):
    """Limits of the bounded device waits on the current device (0 keeps one):
    kernel-internal waits (1 s by default) and waits on another GPU's flags in
    the peer exchange (5 s by default)."""
    L.check(L.load().ql_set_wait_limits(int(wait_ns), int(peer_wait_ns)), "set_wait_limits")


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _validate(qweight, scales, qzeros, K, N, bits, block_size):
    """The MatMulNBits contract checks of ``breeze/cpu_backend.py:128-156``."""
    if bits not in (4, 8) or block_size != 32:
        raise ValueError("quantized prepack requires 4/8-bit weights and block_size=32")
    if (not isinstance(N, (int, np.integer)) or not isinstance(K, (int, np.integer))
            or isinstance(N, (bool, np.bool_)) or isinstance(K, (bool, np.bool_))
            or N > _INT32_MAX or K > _INT32_MAX):
        raise ValueError("Prepack dimensions must be signed 32-bit integers")
    N, K = int(N), int(K)
    if N <= 0 or K <= 0 or N % 16 or K % 32:
        raise ValueError(f"need N%16==0,K%32==0 (got N={N},K={K})")
    nblk = K // 32
    qdt = qweight.dtype
    if str(qdt) not in ("uint8", "torch.uint8"):
        raise ValueError("MatMulNBits packed weights must be uint8")
    if _numel(qweight) != N * nblk * (4 * bits):
        raise ValueError("Incorrect packed weight size for the supplied dimensions")
    if _numel(scales) != N * nblk:
        raise ValueError("Incorrect scale count for the supplied dimensions")
    if qzeros is not None and _numel(qzeros):
        if str(qzeros.dtype) not in ("uint8", "torch.uint8"):
            raise ValueError("Packed zero points must be uint8")
        if _numel(qzeros) != N * (nblk if bits == 8 else (nblk + 1) // 2):
            raise ValueError("Incorrect zero-point count for the supplied dimensions")
        if bits == 8:
            if bool((qzeros != 128).any()):
                raise ValueError("INT8 weights require symmetric zero point 128")
            qzeros = None
    else:
        qzeros = None
    return N, K, qzeros


def _numel(x):
    return int(x.numel()) if hasattr(x, "numel") and callable(x.numel) else int(np.size(x))


def prepack(qweight, scales, qzeros, K, N, bits=4, block_size=32):
    """Pack ONNX MatMulNBits weights into device memory; returns an opaque handle.

    Same signature and contract as ``breeze/cpu_backend.py:119-168``.  The
    handle (an integer address, like the reference's) owns its device memory
    on the current CUDA device and must be released with :func:`free`.
    """
    if not _is_cuda_tensor(qweight):
        qweight = np.asarray(qweight)
        scales = np.asarray(scales)
        if qzeros is not None:
            qzeros = np.asarray(qzeros)
    N, K, qzeros = _validate(qweight, scales, qzeros, K, N, bits, block_size)
    lib = L.load()
    if _is_cuda_tensor(qweight):
        return _prepack_device(lib, qweight, scales, qzeros, K, N, bits)
    qw = np.ascontiguousarray(qweight)
    scale_dtype = np.float16 if scales.dtype == np.float16 else np.float32
    sc = np.require(scales, dtype=scale_dtype, requirements=["C", "A"])
    qz = np.ascontiguousarray(qzeros) if qzeros is not None else None
    handle = lib.i4_prepack_onnx(_p(qw), _p(sc), _p(qz), N, K, int(bits), sc.itemsize * 8)
    if not handle:
        raise MemoryError(f"Could not allocate packed {bits}-bit weights (N={N}, K={K})")
    return handle


def _prepack_device(lib, qweight, scales, qzeros, K, N, bits):
    torch = _torch()
    dev = qweight.device
    qw = qweight.contiguous()
    sc = scales.to(dev)
    if sc.dtype != torch.float16:
        sc = sc.to(torch.float32)
    sc = sc.contiguous()
    qz = qzeros.to(dev).contiguous() if qzeros is not None else None
    out = ctypes.c_void_p()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        rc = lib.ql_prepack_onnx_dev(qw.data_ptr(), sc.data_ptr(), qz.data_ptr() if qz is not None else None,
                                     N, K, int(bits), 16 if sc.dtype == torch.float16 else 32,
                                     stream.cuda_stream, ctypes.byref(out))
        if rc == L.QL_ENOMEM or (rc == L.QL_OK and not out.value):
            raise MemoryError(f"Could not allocate packed {bits}-bit weights (N={N}, K={K})")
        L.check(rc, "prepack")
        stream.synchronize()          # inputs may be released by the caller afterwards
    return out.value


def weight_info(handle):
    """(N, K, bits, device, bytes) of a handle."""
    lib = L.load()
    n, k, b, d = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    nbytes = ctypes.c_ulonglong()
    L.check(lib.ql_weight_info(ctypes.c_void_p(handle), ctypes.byref(n), ctypes.byref(k), ctypes.byref(b),
                               ctypes.byref(d), ctypes.byref(nbytes)), "weight_info")
    return n.value, k.value, b.value, d.value, nbytes.value


def matmul(handle, a2d, N):
    """``a2d`` fp32 ``[M, K]`` -> fp32 ``[M, N]`` (``breeze/cpu_backend.py:230-237``).

    NumPy in, NumPy out (synchronous, through the reference-compatible
    ``i4_matmul``, which also reads the device error word: a kernel wait that
    gave up raises :class:`~breeze_engine_b200._lib.QLError`), or torch CUDA
    tensor in, CUDA tensor out (asynchronous on the current stream, through
    ``ql_matmul_dev_ws``; check :func:`check_device` after synchronising).
    """
    lib = L.load()
    hN, hK, _, hdev, _ = weight_info(handle)
    if int(N) != hN:
        raise ValueError(f"N={N} does not match the packed weight (N={hN})")
    if _is_cuda_tensor(a2d):
        return _matmul_device(lib, handle, a2d, hN, hK, hdev)
    a2d = np.ascontiguousarray(a2d, dtype=np.float32)
    if a2d.ndim != 2 or a2d.shape[1] != hK:
        raise ValueError(f"activations must be [M, {hK}]")
    M = a2d.shape[0]
    out = np.empty((M, hN), dtype=np.float32)
    lib.i4_matmul(ctypes.c_void_p(handle), _p(a2d), int(M), _p(out))
    L.check(lib.ql_last_status(), "matmul")
    return out


def _matmul_device(lib, handle, a, N, K, hdev, out=None, workspace=None):
    torch = _torch()
    if a.dim() != 2 or a.shape[1] != K:
        raise ValueError(f"activations must be [M, {K}]")
    if a.device.index != hdev:
        raise ValueError(f"activations on cuda:{a.device.index}, weights on cuda:{hdev}")
    a = a.to(torch.float32).contiguous()
    if a.data_ptr() % 16:             # 16-byte vector loads in the quantizer
        a = a.clone()
    M = a.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=a.device)
    if M == 0:
        return out
    need = lib.ql_workspace_bytes(ctypes.c_void_p(handle), int(M))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=a.device)
    with torch.cuda.device(a.device):
        stream = torch.cuda.current_stream(a.device).cuda_stream
        rc = lib.ql_matmul_dev_ws(ctypes.c_void_p(handle), a.data_ptr(), int(M), out.data_ptr(),
                                  workspace.data_ptr(), int(workspace.numel()), stream)
    L.check(rc, "matmul")
    return out


def rmsnorm_matmul(handle, x, norm_w, eps, N, out=None):
    """``matmul(rmsnorm(x, norm_w, eps))`` with the normalisation fused into
    the activation quantizer: the reference decoder's ``rmsnorm`` followed by
    ``i4_matmul`` on its output (``kernel/qwen35_decoder.cpp:133-141``, then
    ``:329``, ``:395``, ``:406-407``, ``:421``), bit for bit.  ``x`` fp32
    ``[M, K]`` and ``norm_w`` fp32 ``[K]`` are CUDA tensors on the handle's
    device; asynchronous on the current stream.  The activation mode is the
    process-wide one (:func:`set_hi_prec`)."""
    lib = L.load()
    torch = _torch()
    hN, hK, _, hdev, _ = weight_info(handle)
    if int(N) != hN:
        raise ValueError(f"N={N} does not match the packed weight (N={hN})")
    if not (_is_cuda_tensor(x) and _is_cuda_tensor(norm_w)):
        raise TypeError("rmsnorm_matmul takes CUDA tensors")
    if x.dim() != 2 or x.shape[1] != hK or tuple(norm_w.shape) != (hK,):
        raise ValueError(f"x must be [M, {hK}] and norm_w [{hK}]")
    if x.device.index != hdev or norm_w.device.index != hdev:
        raise ValueError(f"inputs must be on cuda:{hdev}, where the weights are")
    x = x.to(torch.float32).contiguous()
    norm_w = norm_w.to(torch.float32).contiguous()
    if x.data_ptr() % 16:
        x = x.clone()
    if norm_w.data_ptr() % 16:
        norm_w = norm_w.clone()
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, hN), dtype=torch.float32, device=x.device)
    if M == 0:
        return out
    hp = get_hi_prec()
    need = lib.ql_norm_act_workspace_bytes(int(M), int(hK))
    ws = torch.empty(need, dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device).cuda_stream
        L.check(lib.ql_quantize_act_rmsnorm_dev(x.data_ptr(), norm_w.data_ptr(), float(eps), int(M), int(hK),
                                                int(hp), ws.data_ptr(), need, None, stream), "rmsnorm_matmul")
        L.check(lib.ql_matmul_quantized_dev(ctypes.c_void_p(handle), ws.data_ptr(), int(M), int(hp),
                                            out.data_ptr(), stream), "rmsnorm_matmul")
    return out


def silu_mul_matmul(handle, gate, up, N, out=None):
    """``matmul(silu(gate) * up)`` with the SiLU and product fused into the
    activation quantizer: the reference decoder's ``g1 = siluf(g1) * g2``
    followed by ``i4_matmul`` of the down projection
    (``kernel/qwen35_decoder.cpp:408-409``), bit for bit (the host C library's
    ``expf`` is reproduced exactly).  ``gate`` and ``up`` are fp32 CUDA tensors of
    shape ``[M, K]`` on the handle's device whose rows share one stride (e.g. the
    two halves of a concatenated gate|up output); asynchronous on the current
    stream, in the process-wide activation mode (:func:`set_hi_prec`)."""
    lib = L.load()
    torch = _torch()
    hN, hK, _, hdev, _ = weight_info(handle)
    if int(N) != hN:
        raise ValueError(f"N={N} does not match the packed weight (N={hN})")
    if not (_is_cuda_tensor(gate) and _is_cuda_tensor(up)):
        raise TypeError("silu_mul_matmul takes CUDA tensors")
    if gate.dim() != 2 or tuple(gate.shape) != tuple(up.shape) or gate.shape[1] != hK:
        raise ValueError(f"gate and up must both be [M, {hK}]")
    if gate.device.index != hdev or up.device.index != hdev:
        raise ValueError(f"inputs must be on cuda:{hdev}, where the weights are")
    ok = (gate.dtype == torch.float32 and up.dtype == torch.float32 and gate.stride(1) == 1 and up.stride(1) == 1
          and gate.stride(0) == up.stride(0) and gate.stride(0) % 4 == 0 and gate.data_ptr() % 16 == 0
          and up.data_ptr() % 16 == 0)
    if not ok:
        gate = gate.to(torch.float32).contiguous().clone()
        up = up.to(torch.float32).contiguous().clone()
    M = gate.shape[0]
    if out is None:
        out = torch.empty((M, hN), dtype=torch.float32, device=gate.device)
    if M == 0:
        return out
    with torch.cuda.device(gate.device):
        stream = torch.cuda.current_stream(gate.device).cuda_stream
        L.check(lib.ql_matmul_silu_mul_dev(ctypes.c_void_p(handle), gate.data_ptr(), up.data_ptr(),
                                           int(gate.stride(0)), int(M), out.data_ptr(), stream), "silu_mul_matmul")
    return out


def concat_packed(handles):
    """One new handle stacking ``handles`` along N (same K, bits, scale type
    and zero points), e.g. gate and up, so projections that share an input run
    as one launch (the reference calls ``i4_matmul`` once per projection,
    ``kernel/qwen35_decoder.cpp:406-407``).  Output columns follow the order
    given; the sources stay valid and are freed separately."""
    lib = L.load()
    handles = list(handles)
    if not handles:
        raise ValueError("concat_packed needs at least one handle")
    arr = (ctypes.c_void_p * len(handles))(*handles)
    out = ctypes.c_void_p()
    rc = lib.ql_weight_concat(arr, len(handles), ctypes.byref(out))
    if rc == L.QL_EINVAL:
        raise ValueError("handles differ in K, bits, scale type, zero points or device")
    L.check(rc, "concat_packed")
    return out.value


def save_packed(handle, path):
    """Write a handle's packed device layout to ``path`` (a versioned header
    plus the records), so a later :func:`load_packed` skips the MatMulNBits
    repack.  The reference repacks on every load (``breeze/qwen35_cpu.py:71-89``)."""
    lib = L.load()
    n = lib.ql_weight_serialized_bytes(ctypes.c_void_p(handle))
    if n == 0:
        raise ValueError("invalid handle")
    buf = np.empty(n, dtype=np.uint8)
    L.check(lib.ql_weight_serialize(ctypes.c_void_p(handle), _p(buf), n), "save_packed")
    with open(path, "wb") as f:
        buf.tofile(f)
    return n


def load_packed(path):
    """Create a handle on the current CUDA device from a file written by
    :func:`save_packed`; ``ValueError`` for a corrupt or mismatched file."""
    lib = L.load()
    buf = np.fromfile(path, dtype=np.uint8)
    out = ctypes.c_void_p()
    rc = lib.ql_weight_deserialize(_p(buf), buf.size, ctypes.byref(out))
    if rc == L.QL_EINVAL:
        raise ValueError(f"{path}: not a packed weight of this library version (or corrupt)")
    if rc == L.QL_ENOMEM or (rc == L.QL_OK and not out.value):
        raise MemoryError(f"Could not allocate packed weights from {path}")
    L.check(rc, "load_packed")
    return out.value


def free(handle):
    """Release a handle (``breeze/cpu_backend.py:240-242``); null-safe."""
    lib = L.try_load()
    if lib is not None and handle:
        lib.i4_free(ctypes.c_void_p(handle))
