"""Quantized linear with the call surface of ``breeze/linear.py``.

The reference module (``breeze/linear.py:25-46``) stores a dequantized
``[K, N]`` weight in fp16/fp32 and runs a dense GEMM.  Here the same three
functions keep the weight quantized on the GPU and run the INT16 x INT4/INT8
kernels:

* :func:`backend` names the backend.
* :func:`prepare_weight` accepts either MatMulNBits arrays
  ``(qweight, scales, qzeros, K, N, bits)`` -- packed as they are, the exact
  reference numerics -- or a dense fp32 ``[K, N]`` weight, which is first packed
  by this package's round-to-nearest MatMulNBits packer
  (:func:`breeze_engine_b200.quant.quantize_matmul_nbits`; 8-bit per-channel
  by default), so the result is the quantized layer, not the dense product.
* :func:`linear` computes ``a @ w`` for ``[..., K]`` activations and returns
  fp32 ``[..., N]`` (NumPy in, NumPy out; torch CUDA in, torch CUDA out).

The activation mode is the process-global one of
:func:`breeze_engine_b200.backend.set_hi_prec` (two-pass INT16 when on).
"""
import numpy as np

from . import backend as _backend
from .quant import quantize_matmul_nbits


def backend():
    return "cuda-sm100a-quantized"


class QuantizedWeight:
    """A packed device weight (owns its handle)."""

    def __init__(self, handle, K, N, bits):
        self.handle, self.K, self.N, self.bits = handle, int(K), int(N), int(bits)
        self.shape = (self.K, self.N)

    def close(self):
        if self.handle:
            _backend.free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def prepare_weight(w, *, bits=8, symmetric=True, per_channel=True):
    """Pack a weight for :func:`linear` (see the module docstring)."""
    if isinstance(w, (tuple, list)):
        qweight, scales, qzeros, K, N, nbits = w
        h = _backend.prepack(qweight, scales, qzeros, K, N, bits=nbits)
        return QuantizedWeight(h, K, N, nbits)
    dense = np.ascontiguousarray(w, np.float32)
    if dense.ndim != 2:
        raise ValueError("dense weight must be [K, N]")
    K, N = dense.shape
    qweight, scales, qzeros = quantize_matmul_nbits(dense, bits=bits, symmetric=symmetric,
                                                    per_channel=per_channel and bits == 8)
    h = _backend.prepack(qweight, scales, qzeros, K, N, bits=bits)
    return QuantizedWeight(h, K, N, bits)


def linear(a, w):
    """``a @ w`` for ``[..., K]`` activations, returning fp32 ``[..., N]``."""
    lead = tuple(a.shape[:-1])
    m = a.reshape(-1, a.shape[-1])
    out = _backend.matmul(w.handle, m, w.N)
    return out.reshape(*lead, w.N)
