"""Test helpers that drive libbreeze_ql.so through its C ABI (include/breeze_ql.h).

Device memory comes from torch (plumbing only); every compute call goes
through the library's exported ``extern "C"`` entry points via ctypes.
"""
import ctypes

import numpy as np

from breeze_engine_b200 import _lib as L

_vp = ctypes.c_void_p


def lib():
    return L.load()


def prepack(qweight, scales, qzeros, N, K, bits):
    """i4_prepack_onnx with host arrays (the reference-compatible entry)."""
    qw = np.ascontiguousarray(qweight, np.uint8)
    s = np.asarray(scales)
    sc = np.ascontiguousarray(s if s.dtype == np.float16 else s.astype(np.float32))
    qz = None
    if qzeros is not None and bits == 4:
        qz = np.ascontiguousarray(qzeros, np.uint8)
    h = lib().i4_prepack_onnx(qw.ctypes.data, sc.ctypes.data, qz.ctypes.data if qz is not None else None,
                              N, K, bits, sc.itemsize * 8)
    assert h, f"i4_prepack_onnx failed: status {lib().ql_last_status()}"
    return h


def free(h):
    lib().i4_free(_vp(h))


def set_hi_prec(on):
    lib().i4_set_hi_prec(1 if on else 0)


def matmul_host(h, a, N):
    """i4_matmul: host pointers, synchronous."""
    a = np.ascontiguousarray(a, np.float32)
    c = np.full((a.shape[0], N), np.float32(-12345.0))
    lib().i4_matmul(_vp(h), a.ctypes.data, a.shape[0], c.ctypes.data)
    assert lib().ql_last_status() == 0, lib().ql_error_string(lib().ql_last_status())
    return c


def matmul_dev(h, a, N, workspace=True):
    """ql_matmul_dev_ws (or ql_matmul_dev) on torch device buffers."""
    import torch
    a = np.ascontiguousarray(a, np.float32)
    M = a.shape[0]
    dA = torch.from_numpy(a).cuda()
    dC = torch.full((M, N), -12345.0, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if workspace:
        need = lib().ql_workspace_bytes(_vp(h), M)
        ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
        rc = lib().ql_matmul_dev_ws(_vp(h), dA.data_ptr(), M, dC.data_ptr(), ws.data_ptr(), need, stream)
    else:
        rc = lib().ql_matmul_dev(_vp(h), dA.data_ptr(), M, dC.data_ptr(), stream)
    assert rc == 0, lib().ql_error_string(rc)
    torch.cuda.synchronize()
    return dC.cpu().numpy()


def block_sums_dev(h, a, N, K):
    import torch
    a = np.ascontiguousarray(a, np.float32)
    M = a.shape[0]
    dA = torch.from_numpy(a).cuda()
    dCS = torch.full((M, N, K // 32), -7, dtype=torch.int32, device="cuda")
    rc = lib().ql_block_sums_dev(_vp(h), dA.data_ptr(), M, dCS.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib().ql_error_string(rc)
    torch.cuda.synchronize()
    return dCS.cpu().numpy()


def quantize_dev(a):
    import torch
    a = np.ascontiguousarray(a, np.float32)
    M, K = a.shape
    dA = torch.from_numpy(a).cuda()
    hi = torch.empty((M, K), dtype=torch.uint8, device="cuda")
    lo = torch.empty((M, K), dtype=torch.uint8, device="cuda")
    asc = torch.empty((M, K // 32), dtype=torch.float32, device="cuda")
    rc = lib().ql_quantize_dev(dA.data_ptr(), M, K, hi.data_ptr(), lo.data_ptr(), asc.data_ptr(),
                               torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    return hi.cpu().numpy(), lo.cpu().numpy(), asc.cpu().numpy()


def device_error(clear=True):
    return lib().ql_device_error(1 if clear else 0)


def rmsnorm_quantize_dev(x, w, eps, hi_prec, want_hn=True):
    """ql_quantize_act_rmsnorm_dev: returns (workspace tensor, hn or None)."""
    import torch
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    dX = torch.from_numpy(x).cuda()
    dW = torch.from_numpy(np.ascontiguousarray(w, np.float32)).cuda()
    need = lib().ql_norm_act_workspace_bytes(M, K)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    hn = torch.full((M, K), -7.0, dtype=torch.float32, device="cuda") if want_hn else None
    rc = lib().ql_quantize_act_rmsnorm_dev(dX.data_ptr(), dW.data_ptr(), float(eps), M, K, 1 if hi_prec else 0,
                                           ws.data_ptr(), need, hn.data_ptr() if want_hn else None,
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib().ql_error_string(rc)
    torch.cuda.synchronize()
    return ws, (hn.cpu().numpy() if want_hn else None)


def matmul_quantized_dev(h, ws, M, hi_prec, N):
    """ql_matmul_quantized_dev over a workspace filled by a quantize call."""
    import torch
    dC = torch.full((M, N), -12345.0, dtype=torch.float32, device="cuda")
    rc = lib().ql_matmul_quantized_dev(_vp(h), ws.data_ptr(), M, 1 if hi_prec else 0, dC.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib().ql_error_string(rc)
    torch.cuda.synchronize()
    return dC.cpu().numpy()


def matmul_rmsnorm_dev(h, x, w, eps, N):
    """ql_matmul_rmsnorm_dev (library workspace, process-wide activation mode)."""
    import torch
    x = np.ascontiguousarray(x, np.float32)
    M = x.shape[0]
    dX = torch.from_numpy(x).cuda()
    dW = torch.from_numpy(np.ascontiguousarray(w, np.float32)).cuda()
    dC = torch.full((M, N), -12345.0, dtype=torch.float32, device="cuda")
    rc = lib().ql_matmul_rmsnorm_dev(_vp(h), dX.data_ptr(), dW.data_ptr(), float(eps), M, dC.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib().ql_error_string(rc)
    torch.cuda.synchronize()
    return dC.cpu().numpy()


def concat(handles):
    """ql_weight_concat: one handle stacking the weights along N."""
    arr = (_vp * len(handles))(*handles)
    out = _vp()
    rc = lib().ql_weight_concat(arr, len(handles), ctypes.byref(out))
    assert rc == 0 and out.value, lib().ql_error_string(rc)
    return out.value


def silu_quantize_dev(g, u, hi_prec, ld=None):
    """ql_quantize_act_silu_mul_dev: returns (workspace tensor, the products).
    With ld > K, gate and up sit side by side in one [M, ld] buffer (up at
    column K, as in a concatenated gate|up output)."""
    import torch
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    M, K = g.shape
    ld = ld or K
    if ld == K:
        buf = np.concatenate([g, u], axis=0)          # separate planes: gate rows, then up rows
    else:
        buf = np.zeros((M, ld), np.float32)
        buf[:, :K] = g
        buf[:, K:2 * K] = u
    dbuf = torch.from_numpy(np.ascontiguousarray(buf)).cuda()
    if ld == K:
        dG, dU = dbuf[:M], dbuf[M:]
    else:
        dG, dU = dbuf[:, :K], dbuf[:, K:2 * K]
    need = lib().ql_act_workspace_bytes(M, K)
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    out = torch.full((M, K), -7.0, dtype=torch.float32, device="cuda")
    rc = lib().ql_quantize_act_silu_mul_dev(dG.data_ptr(), dU.data_ptr(), ld, M, K, 1 if hi_prec else 0,
                                            ws.data_ptr(), need, out.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib().ql_error_string(rc)
    torch.cuda.synchronize()
    return ws, out.cpu().numpy()


def matmul_silu_dev(h, g, u, N, ld_pad=0):
    """ql_matmul_silu_mul_dev (library workspace, process-wide activation mode),
    gate and up in one [M, 2K + ld_pad] buffer."""
    import torch
    g = np.ascontiguousarray(g, np.float32)
    M, K = g.shape
    ld = 2 * K + ld_pad
    buf = np.zeros((M, ld), np.float32)
    buf[:, :K] = g
    buf[:, K:2 * K] = u
    dbuf = torch.from_numpy(buf).cuda()
    dC = torch.full((M, N), -12345.0, dtype=torch.float32, device="cuda")
    rc = lib().ql_matmul_silu_mul_dev(_vp(h), dbuf.data_ptr(), dbuf[:, K:].data_ptr(), ld, M, dC.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib().ql_error_string(rc)
    torch.cuda.synchronize()
    return dC.cpu().numpy()
