"""Parity checkers for the quantized-linear hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` legs may import this module, and only as the checker or
the timed CPU baseline.  The product (``breeze_engine_b200``) never imports it.

Two checkers live here:

* :class:`Oracle` wraps ``liboracle.so`` (``ql_oracle.c``), the scalar C
  restatement of ``kernel/quantized_matmul.cpp`` working on the MatMulNBits
  layout.  It is pinned against the committed golden fixtures in
  ``tests/golden`` (generated from the compiled reference) and, where the
  reference library was built, against the reference itself.
* :class:`Reference` wraps ``_ref/libbreeze_ref.so``: the reference's own
  ``kernel/quantized_matmul.cpp`` plus ``ref_probe.cpp``.  It exposes the
  reference C ABI (``i4_prepack_onnx``/``i4_matmul``/``i4_free``/
  ``i4_set_hi_prec``/``i4_set_threads``, ``kernel/quantized_matmul.cpp:472-574``)
  and the probes for its internal quantizer and per-block INT32 accumulators.

NumPy restatements (:func:`np_quantize_i16`, :func:`np_block_sums`) give an
independent, vectorised cross-check of the integer parts.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.environ.get("BREEZE_REF_KERNEL", os.path.join(HERE, "_ref", "libbreeze_ref.so"))

_vp = ctypes.c_void_p
_i = ctypes.c_int


def _p(a):
    return a.ctypes.data_as(_vp) if a is not None else None


def reference_checkout(reference=None):
    """The reference checkout to compile ``_ref`` from: ``reference``, else the
    ``BREEZE_REFERENCE`` environment variable, else a directory named
    ``reference`` beside this repository; None when none of them holds
    ``kernel/quantized_matmul.cpp`` (e.g. on a GPU box, which uses the
    prebuilt ``_ref`` files)."""
    for ref in (reference, os.environ.get("BREEZE_REFERENCE"),
                os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")):
        if ref and os.path.isfile(os.path.join(ref, "kernel", "quantized_matmul.cpp")):
            return ref
    return None


def build(reference=None):
    """Build ``liboracle.so`` (and ``_ref`` when the reference checkout exists)."""
    targets = ["oracle"]
    ref = reference_checkout(reference)
    if ref:
        targets.append("ref")
        if os.path.exists(os.path.join(os.path.dirname(HERE), "breeze_engine_b200", "libbreeze_ql.so")):
            targets.append("decoders")
    subprocess.run(["make", "-s", "-C", HERE, f"REF={ref or ''}", *targets], check=True)


def weight_scales_f32(scales):
    """fp16/fp32/other scales -> fp32 exactly as the reference bridge does.

    ``cpu_backend.prepack`` keeps fp16 as fp16 (widened exactly by
    ``_cvtsh_ss``) and converts anything else with ``np.require(..., float32)``
    (``breeze/cpu_backend.py:163-164``, ``kernel/quantized_matmul.cpp:156-159``).
    """
    s = np.asarray(scales)
    if s.dtype == np.float16:
        return np.ascontiguousarray(s.astype(np.float32)).reshape(-1)
    return np.ascontiguousarray(s.astype(np.float32)).reshape(-1)


class Oracle:
    """ctypes view of ``liboracle.so`` (the C restatement)."""

    def __init__(self, path=ORACLE_SO):
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        lib.ql_oracle_quantize_i16.argtypes = [_vp, _i, _i, _vp, _vp, _vp]
        lib.ql_oracle_quantize_i8.argtypes = [_vp, _i, _i, _vp, _vp]
        lib.ql_oracle_block_sums.argtypes = [_vp, _vp, _i, _i, _i, _vp, _vp, _i, _vp]
        lib.ql_oracle_rescale.argtypes = [_vp, _vp, _vp, _i, _i, _i, _vp]
        lib.ql_oracle_matmul.argtypes = [_vp, _vp, _vp, _i, _i, _i, _vp, _i, _vp, _vp, _vp, _vp]
        lib.ql_oracle_matmul_i8.argtypes = [_vp, _vp, _vp, _i, _i, _i, _vp, _i, _vp, _vp, _vp]
        lib.ql_oracle_rmsnorm.argtypes = [_vp, _vp, _i, _i, ctypes.c_float, _vp]
        lib.ql_expf_restated.restype = ctypes.c_float
        lib.ql_expf_restated.argtypes = [ctypes.c_float, _i]
        lib.ql_silu_mul_array.argtypes = [_vp, _vp, _vp, ctypes.c_longlong]
        lib.ql_expf_check.restype = ctypes.c_ulonglong
        lib.ql_expf_check.argtypes = [ctypes.c_uint32, ctypes.c_uint32, _i, ctypes.POINTER(ctypes.c_uint32)]
        self.lib = lib

    def quantize_i16(self, a):
        a = np.ascontiguousarray(a, np.float32)
        M, K = a.shape
        hi = np.empty((M, K), np.uint8)
        lo = np.empty((M, K), np.uint8)
        asc = np.empty((M, K // 32), np.float32)
        self.lib.ql_oracle_quantize_i16(_p(a), M, K, _p(hi), _p(lo), _p(asc))
        return hi, lo, asc

    def block_sums(self, qweight, qzeros, N, K, bits, hi, lo):
        qw = np.ascontiguousarray(qweight, np.uint8).reshape(-1)
        qz = None if qzeros is None else np.ascontiguousarray(qzeros, np.uint8).reshape(-1)
        M = hi.shape[0]
        cs = np.empty((M, N, K // 32), np.int32)
        self.lib.ql_oracle_block_sums(_p(qw), _p(qz), N, K, bits, _p(hi), _p(lo), M, _p(cs))
        return cs

    def rescale(self, cs, ascale, scales, N, K):
        M = cs.shape[0]
        bs = weight_scales_f32(scales)
        c = np.empty((M, N), np.float32)
        self.lib.ql_oracle_rescale(_p(np.ascontiguousarray(cs)), _p(np.ascontiguousarray(ascale)),
                                   _p(bs), M, N, K, _p(c))
        return c

    def matmul(self, qweight, scales, qzeros, N, K, bits, a, hi_prec=True):
        a = np.ascontiguousarray(a, np.float32).reshape(-1, K)
        M = a.shape[0]
        qw = np.ascontiguousarray(qweight, np.uint8).reshape(-1)
        qz = None if qzeros is None else np.ascontiguousarray(qzeros, np.uint8).reshape(-1)
        bs = weight_scales_f32(scales)
        c = np.empty((M, N), np.float32)
        asc = np.empty((M, K // 32), np.float32)
        if hi_prec:
            hi = np.empty((M, K), np.uint8)
            lo = np.empty((M, K), np.uint8)
            self.lib.ql_oracle_matmul(_p(qw), _p(bs), _p(qz), N, K, bits, _p(a), M, _p(c),
                                      _p(hi), _p(lo), _p(asc))
        else:
            q8 = np.empty((M, K), np.int8)
            self.lib.ql_oracle_matmul_i8(_p(qw), _p(bs), _p(qz), N, K, bits, _p(a), M, _p(c),
                                         _p(q8), _p(asc))
        return c


    def silu_mul(self, g, u):
        """silu(g) * u element by element as the reference decoder computes it
        (``kernel/qwen35_decoder.cpp:129, 408``), on the restated exponential
        of ``expf_ref.c``."""
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        assert g.shape == u.shape
        out = np.empty_like(g)
        self.lib.ql_silu_mul_array(_p(g), _p(u), _p(out), g.size)
        return out

    def expf_check(self, lo=0, hi=0xFFFFFFFF, fused=True):
        """(mismatches, first mismatching bit pattern) of the restated expf
        against this host's C library over the float bit patterns lo..hi."""
        first = ctypes.c_uint32()
        bad = self.lib.ql_expf_check(lo, hi, 1 if fused else 0, ctypes.byref(first))
        return int(bad), int(first.value)

    def rmsnorm(self, x, w, eps):
        """hn = rmsnorm(x) as the reference decoder computes it
        (``kernel/qwen35_decoder.cpp:133-141``)."""
        x = np.ascontiguousarray(x, np.float32)
        M, K = x.shape
        out = np.empty((M, K), np.float32)
        self.lib.ql_oracle_rmsnorm(_p(x), _p(np.ascontiguousarray(w, np.float32)), M, K, float(eps), _p(out))
        return out


class Reference:
    """ctypes view of the compiled reference (``_ref/libbreeze_ref.so``)."""

    def __init__(self, path=REF_SO):
        lib = ctypes.CDLL(path)
        lib.i4_prepack_onnx.restype = _vp
        lib.i4_prepack_onnx.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i]
        lib.i4_matmul.argtypes = [_vp, _vp, _i, _vp]
        lib.i4_free.argtypes = [_vp]
        lib.i4_set_threads.argtypes = [_i]
        lib.i4_set_hi_prec.argtypes = [_i]
        lib.i4_set_numa_split.argtypes = [_i]
        lib.refprobe_quantize_i16.argtypes = [_vp, _i, _i, _vp, _vp, _vp]
        lib.refprobe_block_sums.argtypes = [_vp, _vp, _vp, _i, _vp]
        lib.refprobe_block_sums.restype = _i
        lib.refprobe_replay.argtypes = [_vp, _vp, _vp, _i, _vp]
        lib.refprobe_replay.restype = _i
        lib.refprobe_rmsnorm.argtypes = [_vp, _vp, _vp, _i, _i, ctypes.c_float]
        lib.refprobe_silu_mul.argtypes = [_vp, _vp, _vp, ctypes.c_longlong]
        self.lib = lib
        lib.i4_set_numa_split(1 << 30)

    @staticmethod
    def available(path=REF_SO):
        return os.path.exists(path)

    def prepack(self, qweight, scales, qzeros, K, N, bits=4):
        """Mirror of ``cpu_backend.prepack``'s native branch (``breeze/cpu_backend.py:162-168``)."""
        qw = np.ascontiguousarray(qweight, np.uint8)
        s = np.asarray(scales)
        sdt = np.float16 if s.dtype == np.float16 else np.float32
        sc = np.require(s, dtype=sdt, requirements=["C", "A"])
        qz = None
        if qzeros is not None and np.size(qzeros) and bits == 4:
            qz = np.ascontiguousarray(qzeros, np.uint8)
        h = self.lib.i4_prepack_onnx(_p(qw), _p(sc), _p(qz), N, K, bits, sc.itemsize * 8)
        if not h:
            raise MemoryError("reference prepack returned null")
        return h

    def matmul(self, handle, a, N, hi_prec=True, threads=None):
        a = np.ascontiguousarray(a, np.float32)
        if threads is not None:
            self.lib.i4_set_threads(int(threads))
        self.lib.i4_set_hi_prec(1 if hi_prec else 0)
        c = np.empty((a.shape[0], N), np.float32)
        self.lib.i4_matmul(_vp(handle), _p(a), a.shape[0], _p(c))
        return c

    def free(self, handle):
        if handle:
            self.lib.i4_free(_vp(handle))

    def quantize_i16(self, a):
        a = np.ascontiguousarray(a, np.float32)
        M, K = a.shape
        hi = np.empty((M, K), np.uint8)
        lo = np.empty((M, K), np.uint8)
        asc = np.empty((M, K // 32), np.float32)
        self.lib.refprobe_quantize_i16(_p(a), M, K, _p(hi), _p(lo), _p(asc))
        return hi, lo, asc

    def block_sums(self, handle, hi, lo, N, K):
        M = hi.shape[0]
        cs = np.empty((M, N, K // 32), np.int32)
        assert self.lib.refprobe_block_sums(_vp(handle), _p(hi), _p(lo), M, _p(cs)) == 0
        return cs

    def silu_mul(self, g, u):
        """The reference decoder's own ``siluf(g) * u`` (``kernel/qwen35_decoder.cpp:129, 408``),
        compiled from its source file by ``oracle/ref_norm_probe.cpp``."""
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        assert g.shape == u.shape
        out = np.empty_like(g)
        self.lib.refprobe_silu_mul(_p(out), _p(g), _p(u), g.size)
        return out

    def rmsnorm(self, x, w, eps):
        """The reference decoder's own rmsnorm (``kernel/qwen35_decoder.cpp:133-141``),
        compiled from its source file by ``oracle/ref_norm_probe.cpp``."""
        x = np.ascontiguousarray(x, np.float32)
        M, K = x.shape
        out = np.empty((M, K), np.float32)
        self.lib.refprobe_rmsnorm(_p(out), _p(x), _p(np.ascontiguousarray(w, np.float32)), M, K, float(eps))
        return out

    def replay(self, handle, cs, ascale, N):
        M = cs.shape[0]
        c = np.empty((M, N), np.float32)
        assert self.lib.refprobe_replay(_vp(handle), _p(np.ascontiguousarray(cs)),
                                        _p(np.ascontiguousarray(ascale)), M, _p(c)) == 0
        return c


def np_quantize_i16(a):
    """Vectorised NumPy restatement of ``quantize_A_i16`` (kernel/quantized_matmul.cpp:237-258)."""
    a = np.ascontiguousarray(a, np.float32)
    M, K = a.shape
    blk = a.reshape(M, K // 32, 32)
    absv = np.abs(blk)
    amax = np.where(np.isnan(absv), np.float32(0), absv).max(axis=2).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        scale = (amax / np.float32(32767.0)).astype(np.float32)
        inv = np.where(scale > 0, np.float32(1.0) / np.where(scale > 0, scale, 1), 0).astype(np.float32)
        x = (blk * inv[:, :, None]).astype(np.float32)
        ok = np.abs(x) < np.float32(2.0 ** 31)
        q = np.where(ok, np.rint(np.where(ok, x, 0)), 0).astype(np.int64)
    q = np.clip(q, -32767, 32767)
    u = (q + 32768).astype(np.uint32).reshape(M, K)
    return (u >> 8).astype(np.uint8), (u & 0xFF).astype(np.uint8), scale


def np_weights(qweight, qzeros, N, K, bits):
    """Signed weights ``w - zp`` as int32 ``[N, K]`` (breeze/quant.py:9-58 semantics)."""
    nblk = K // 32
    if bits == 8:
        return np.ascontiguousarray(qweight, np.uint8).reshape(N, K).astype(np.int32) - 128
    qw = np.ascontiguousarray(qweight, np.uint8).reshape(N, nblk, 16)
    q = np.empty((N, nblk, 32), np.int32)
    q[:, :, 0::2] = qw & 15
    q[:, :, 1::2] = qw >> 4
    if qzeros is not None and np.size(qzeros):
        qz = np.ascontiguousarray(qzeros, np.uint8).reshape(N, (nblk + 1) // 2)
        zp = np.empty((N, 2 * qz.shape[1]), np.int32)
        zp[:, 0::2] = qz & 15
        zp[:, 1::2] = qz >> 4
        zp = zp[:, :nblk]
    else:
        zp = np.full((N, nblk), 8, np.int32)
    return (q - zp[:, :, None]).reshape(N, K)


def np_block_sums(qweight, qzeros, N, K, bits, hi, lo):
    """cs[m, n, b] = sum_k q16 * (w - zp) as int32 ``[M, N, nblk]``."""
    q16 = 256 * (hi.astype(np.int64) - 128) + lo.astype(np.int64)
    w = np_weights(qweight, qzeros, N, K, bits).astype(np.int64)
    M = hi.shape[0]
    nblk = K // 32
    cs = np.einsum("mbj,nbj->mnb", q16.reshape(M, nblk, 32), w.reshape(N, nblk, 32))
    return cs.astype(np.int32)
