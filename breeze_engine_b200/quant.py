"""MatMulNBits weight formats: round-to-nearest packer and the dequantizer.

The reference consumes ONNX ``com.microsoft`` MatMulNBits weights
(``breeze/quant.py:9-58`` decodes them; ``breeze/cpu_backend.py:119-168``
validates them) but ships no FP32 -> MatMulNBits packer.  :func:`quantize_matmul_nbits`
is this package's seeded, deterministic round-to-nearest packer producing
exactly that layout, so synthetic layers (tests, ``bench.py``) can be built
from FP32 weights drawn from N(0, 0.02):

* 4-bit: ``qweight`` uint8 ``[N, K/32, 16]``, low nibble = even k;
  ``scales`` ``[N * K/32]`` (fp16 by default); symmetric packing leaves
  ``qzeros`` ``None`` (zero point 8), asymmetric packing returns packed 4-bit
  zero points uint8 ``[N * ceil(nblk/2)]``, low nibble = even block.
* 8-bit: ``qweight`` uint8 ``[N, K/32, 32]``, zero point 128 (the only one the
  reference accepts, ``breeze/cpu_backend.py:152-153``); ``per_channel=True``
  repeats one scale per output row across its blocks.

:func:`dequantize_matmul_nbits` restates the reference decode
``w = (q - zp) * scale`` and returns a dense ``[K, N]`` fp32 matrix.
"""
import numpy as np

BLOCK = 32


def _round_scale(x, scale_dtype):
    s = np.asarray(x, np.float32).astype(scale_dtype)
    return s


def quantize_matmul_nbits(w, *, bits=4, symmetric=True, per_channel=False,
                          scale_dtype=np.float16):
    """Pack a dense fp32 ``[K, N]`` weight into MatMulNBits arrays.

    Returns ``(qweight, scales, qzeros)``.  ``K`` must be a multiple of 32.
    Rounding is numpy ``rint`` (ties to even) on ``w / scale`` with the scale
    already rounded to ``scale_dtype``, so the codes are reproducible.
    """
    w = np.asarray(w, np.float32)
    if w.ndim != 2:
        raise ValueError("weight must be [K, N]")
    K, N = w.shape
    if K % BLOCK:
        raise ValueError("K must be a multiple of 32")
    if bits not in (4, 8):
        raise ValueError("bits must be 4 or 8")
    nblk = K // BLOCK
    wb = np.ascontiguousarray(w.T).reshape(N, nblk, BLOCK)           # [N, nblk, 32]
    if bits == 8:
        if per_channel:
            amax = np.abs(wb).max(axis=(1, 2), keepdims=False)        # [N]
            amax = np.repeat(amax[:, None], nblk, axis=1)
        else:
            amax = np.abs(wb).max(axis=2)                             # [N, nblk]
        scale = _round_scale(amax / 127.0, scale_dtype)
        s32 = scale.astype(np.float32)
        with np.errstate(divide="ignore", invalid="ignore"):
            q = np.where(s32[:, :, None] > 0, np.rint(wb / s32[:, :, None]), 0)
        q = np.clip(q + 128, 0, 255).astype(np.uint8)
        return q.reshape(N, nblk, 32), scale.reshape(-1), None
    if symmetric:
        amax = np.abs(wb).max(axis=2)
        scale = _round_scale(amax / 7.0, scale_dtype)
        s32 = scale.astype(np.float32)
        with np.errstate(divide="ignore", invalid="ignore"):
            q = np.where(s32[:, :, None] > 0, np.rint(wb / s32[:, :, None]), 0)
        q = np.clip(q + 8, 0, 15).astype(np.uint8)
        zeros = None
    else:
        lo = np.minimum(wb.min(axis=2), 0.0)
        hi = np.maximum(wb.max(axis=2), 0.0)
        scale = _round_scale((hi - lo) / 15.0, scale_dtype)
        s32 = scale.astype(np.float32)
        with np.errstate(divide="ignore", invalid="ignore"):
            zp = np.where(s32 > 0, np.rint(-lo / s32), 8)
            zp = np.clip(zp, 0, 15).astype(np.int32)
            q = np.where(s32[:, :, None] > 0, np.rint(wb / s32[:, :, None]) + zp[:, :, None],
                         zp[:, :, None])
        q = np.clip(q, 0, 15).astype(np.uint8)
        packed_cols = (nblk + 1) // 2
        zpad = np.zeros((N, packed_cols * 2), np.uint8)
        zpad[:, :nblk] = zp
        zeros = (zpad[:, 0::2] | (zpad[:, 1::2] << 4)).astype(np.uint8).reshape(-1)
    qweight = (q[:, :, 0::2] | (q[:, :, 1::2] << 4)).astype(np.uint8)  # [N, nblk, 16]
    return qweight, scale.reshape(-1), zeros


def quantize_matmul_nbits_torch(w, *, bits=4, symmetric=True, per_channel=False):
    """:func:`quantize_matmul_nbits` for a torch ``[K, N]`` fp32 tensor, on its device.

    Same rounding rules (fp16 scales, ``round`` ties to even on ``w / scale``)
    and the same output layout, so synthetic layers can be built directly in
    device memory.  Returns ``(qweight uint8, scales fp16, qzeros uint8 or None)``.
    """
    import torch
    K, N = w.shape
    if K % BLOCK:
        raise ValueError("K must be a multiple of 32")
    nblk = K // BLOCK
    wb = w.t().contiguous().reshape(N, nblk, BLOCK).float()
    if bits == 8:
        if per_channel:
            amax = wb.abs().amax(dim=(1, 2)).unsqueeze(1).expand(N, nblk)
        else:
            amax = wb.abs().amax(dim=2)
        scale = (amax / 127.0).to(torch.float16)
        s32 = scale.float().unsqueeze(2)
        q = torch.where(s32 > 0, torch.round(wb / torch.where(s32 > 0, s32, 1.0)), 0.0)
        q = torch.clamp(q + 128, 0, 255).to(torch.uint8)
        return q.reshape(N, nblk, 32).contiguous(), scale.reshape(-1).contiguous(), None
    if not symmetric:
        raise NotImplementedError("torch packer: symmetric INT4 only")
    amax = wb.abs().amax(dim=2)
    scale = (amax / 7.0).to(torch.float16)
    s32 = scale.float().unsqueeze(2)
    q = torch.where(s32 > 0, torch.round(wb / torch.where(s32 > 0, s32, 1.0)), 0.0)
    q = torch.clamp(q + 8, 0, 15).to(torch.uint8)
    qweight = (q[:, :, 0::2] | (q[:, :, 1::2] << 4)).contiguous()
    return qweight, scale.reshape(-1).contiguous(), None


def dequantize_matmul_nbits(qweight, scales, qzeros, *, bits, block_size, K, N):
    """Dense fp32 ``[K, N]`` from MatMulNBits arrays (reference ``breeze/quant.py:9-58``)."""
    if bits not in (4, 8):
        raise NotImplementedError(f"MatMulNBits bits={bits} not supported (only 4, 8).")
    n_blocks = (K + block_size - 1) // block_size
    scales = np.asarray(scales, dtype=np.float32).reshape(N, n_blocks)
    if bits == 8:
        q = np.ascontiguousarray(qweight).reshape(N, n_blocks, block_size).astype(np.float32)
        if qzeros is not None and np.size(qzeros) > 0:
            zp = np.ascontiguousarray(qzeros).reshape(N, n_blocks).astype(np.float32)
        else:
            zp = np.full((N, n_blocks), 128.0, np.float32)
    else:
        qw = np.ascontiguousarray(qweight).reshape(N, n_blocks, block_size // 2)
        q = np.empty((N, n_blocks, block_size), np.uint8)
        q[:, :, 0::2] = qw & 0x0F
        q[:, :, 1::2] = qw >> 4
        q = q.astype(np.float32)
        if qzeros is not None and np.size(qzeros) > 0:
            packed = (n_blocks + 1) // 2
            qz = np.ascontiguousarray(qzeros).reshape(N, packed)
            zp = np.empty((N, packed * 2), np.uint8)
            zp[:, 0::2] = qz & 0x0F
            zp[:, 1::2] = qz >> 4
            zp = zp[:, :n_blocks].astype(np.float32)
        else:
            zp = np.full((N, n_blocks), 8.0, np.float32)
    w = (q - zp[:, :, None]) * scales[:, :, None]
    w = w.reshape(N, n_blocks * block_size)[:, :K]
    return np.ascontiguousarray(w.T)
