"""The reference's native decoders, unchanged, on this library.

``oracle/_ref/libdecoders_ql.so`` is the reference's ``kernel/phi35_decoder.cpp``
and ``kernel/qwen35_decoder.cpp`` compiled from where they lie and linked with
``--no-undefined`` against ``breeze_engine_b200/libbreeze_ql.so`` in place of
``kernel/quantized_matmul.cpp`` (``oracle/Makefile``, target ``decoders``).
It is built where the reference checkout exists and travels with the
repository; the tests skip when it is absent.

CPU: the library loads, its matmul imports resolve to libbreeze_ql.so, and it
exports the decoders' C ABI (``i4_forward``, ``i4_qwen_forward``, ...).

GPU: the tiny Phi forward of the reference's own test
(``tests/test_public_api.py:40-88``: one layer, H = 32, four heads of 8,
intermediate 64, vocabulary 32, 1 or 8 tokens, both activation modes) runs
through ``i4_forward`` -- whose projections call ``i4_matmul_region`` from
inside the decoder's persistent OpenMP region -- and gives the closed-form
logits; with random weights and embeddings its logits equal, bit for bit,
those of the reference's own library (``oracle/_ref/libbreeze_ref.so``, the
same decoder on the AVX-512 ``i4_matmul``).
"""
import ctypes
import os

import numpy as np
import pytest

from breeze_engine_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEC_SO = os.path.join(ROOT, "oracle", "_ref", "libdecoders_ql.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libbreeze_ref.so")

needs_decoders = pytest.mark.skipif(not os.path.exists(DEC_SO),
                                    reason="oracle/_ref/libdecoders_ql.so not built (needs the reference checkout)")

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float


def _bind(lib):
    lib.i4_prepack_onnx.restype = _vp
    lib.i4_prepack_onnx.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i]
    lib.i4_free.argtypes = [_vp]
    lib.i4_set_hi_prec.argtypes = [_i]
    lib.i4_set_threads.argtypes = [_i]
    lib.i4_model_new.restype = _vp
    lib.i4_model_new.argtypes = [_i, _i, _i, _i, _i, _i, _f, _f, _i]
    lib.i4_model_set_embed.argtypes = [_vp, _vp]
    lib.i4_model_set_rotary.argtypes = [_vp, _vp, _vp]
    lib.i4_model_set_layer.argtypes = [_vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp]
    lib.i4_model_set_final.argtypes = [_vp, _vp, _vp]
    lib.i4_model_free.argtypes = [_vp]
    lib.i4_forward.argtypes = [_vp, _vp, _i, _vp]
    return lib


@needs_decoders
def test_decoders_link_against_this_library():
    dec = ctypes.CDLL(DEC_SO)
    ql = L.load()
    for name in ("i4_forward", "i4_model_new", "i4_qwen_forward", "i4_qwen_new", "i4_qwen_set_linear",
                 "i4_qwen_set_full", "i4_causal_conv", "i4_linear_attention"):
        assert hasattr(dec, name), name
    # the decoders' matmul imports are this library's entry points
    for name in ("i4_matmul", "i4_matmul_region", "i4_prepack_onnx", "i4_free", "i4_set_hi_prec"):
        assert ctypes.cast(getattr(dec, name), _vp).value == ctypes.cast(getattr(ql, name), _vp).value, name


class _TinyPhi:
    """The one-layer Phi model of the reference's tiny forward, built through
    one library's C ABI (its i4_prepack_onnx and i4_model_* entry points)."""
    L_, H, NH, HS, INTER, VOCAB, ROT = 1, 32, 4, 8, 64, 32, 8

    def __init__(self, lib, random_seed=None):
        self.lib = _bind(lib)
        self.keep, self.handles = [], []
        rng = np.random.default_rng(random_seed) if random_seed is not None else None
        H, I, V = self.H, self.INTER, self.VOCAB
        self.m = lib.i4_model_new(self.L_, H, self.NH, self.HS, I, V, 1e-5, 8 ** -0.5, self.ROT)
        assert self.m
        if rng is None:
            embed = np.full((V, H), 0.5, np.float16)
            cos, sin = np.ones((8, self.ROT // 2), np.float32), np.zeros((8, self.ROT // 2), np.float32)
            norm = np.ones(H, np.float32)
        else:
            embed = rng.standard_normal((V, H)).astype(np.float16)
            ang = rng.uniform(0, np.pi, (8, self.ROT // 2))
            cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
            norm = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        lib.i4_model_set_embed(self.m, self._vec(embed))
        lib.i4_model_set_rotary(self.m, self._vec(cos), self._vec(sin))
        nv = self._vec(norm)
        proj = lambda k, n, packed=0x88: self._proj(k, n, packed, rng)  # noqa: E731
        lib.i4_model_set_layer(self.m, 0, proj(H, 3 * H), proj(H, H), proj(H, I), proj(H, I), proj(I, H), nv, nv)
        lib.i4_model_set_final(self.m, nv, proj(H, V, 0x99))

    def _vec(self, a):
        a = np.ascontiguousarray(a)
        self.keep.append(a)
        return a.ctypes.data

    def _proj(self, K, N, packed, rng):
        if rng is None:
            qw = np.full((N, K // 32, 16), packed, np.uint8)
            sc = np.full(N * (K // 32), 0.125, np.float32)
        else:
            qw = rng.integers(0, 256, (N, K // 32, 16), dtype=np.uint8)
            sc = rng.uniform(0.01, 0.05, N * (K // 32)).astype(np.float32)
        h = self.lib.i4_prepack_onnx(qw.ctypes.data, sc.ctypes.data, None, N, K, 4, 32)
        assert h
        self.handles.append(h)
        return h

    def forward(self, tokens):
        ids = np.ascontiguousarray(tokens, np.int64)
        logits = np.empty((ids.size, self.VOCAB), np.float32)
        self.lib.i4_forward(self.m, ids.ctypes.data, int(ids.size), logits.ctypes.data)
        return logits

    def close(self):
        for h in self.handles:
            self.lib.i4_free(h)
        self.lib.i4_model_free(self.m)


@pytest.mark.gpu
@needs_decoders
@pytest.mark.parametrize("high_precision", [False, True])
@pytest.mark.parametrize("tokens", [1, 8])
def test_phi_tiny_forward_on_the_gpu_library(high_precision, tokens):
    dec = ctypes.CDLL(DEC_SO)
    ql = L.load()
    ql.i4_set_hi_prec(1 if high_precision else 0)
    model = _TinyPhi(dec)
    try:
        actual = model.forward([1] * tokens)
        assert ql.ql_last_status() == 0
        expected = 32 * 0.125 * 0.5 / np.sqrt(0.25 + 1e-5)
        assert actual.shape == (tokens, 32)
        np.testing.assert_allclose(actual, expected, rtol=1e-5, atol=1e-5)
    finally:
        model.close()
        ql.i4_set_hi_prec(0)
        assert ql.ql_device_error(1) == 0


@pytest.mark.gpu
@needs_decoders
@pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref/libbreeze_ref.so not built")
@pytest.mark.parametrize("high_precision", [False, True])
@pytest.mark.parametrize("tokens", [1, 3, 8])
def test_phi_random_forward_matches_the_reference_build(high_precision, tokens):
    """Random weights, embeddings, rotary tables and norms: the GPU-linked
    decoder's logits equal the reference library's bit for bit."""
    dec = ctypes.CDLL(DEC_SO)
    ref = _bind(ctypes.CDLL(REF_SO))
    ql = L.load()
    ql.i4_set_hi_prec(1 if high_precision else 0)
    ref.i4_set_hi_prec(1 if high_precision else 0)
    ref.i4_set_threads(2)
    ids = np.random.default_rng(tokens).integers(0, 32, tokens)
    ours, theirs = _TinyPhi(dec, random_seed=77), _TinyPhi(ref, random_seed=77)
    try:
        got, want = ours.forward(ids), theirs.forward(ids)
        assert ql.ql_last_status() == 0
        assert np.isfinite(want).all()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    finally:
        ours.close()
        theirs.close()
        ql.i4_set_hi_prec(0)
        ref.i4_set_hi_prec(0)
        assert ql.ql_device_error(1) == 0
