"""Column- and row-parallel quantized linear over the GPUs of one node.

One process per GPU, ``torch.distributed`` with NCCL over NVLink/NVSwitch.
The reference has no multi-device path; this shards one MatMulNBits layer the
two ways the benchmark spec asks for:

* **Column-parallel** (output features N split, ``N % (16 P) == 0``): rank r
  packs output rows ``[r N/P, (r+1) N/P)``, computes ``C[:, N_r]`` from the
  replicated activations and the shards are all-gathered.  Every output's
  block chain stays on one GPU, so the result is bit-identical to the
  unsharded layer (and to the reference).
* **Row-parallel** (input features K split, ``(K/32) % P == 0``): rank r packs
  blocks ``[r nblk/P, (r+1) nblk/P)`` and quantizes only its K slice of the
  activations (per-block quantization makes those planes identical to the
  unsharded ones), producing an FP32 partial ``[M, N]``; partials are summed by
  reduce-scatter (each rank keeps one contiguous 1/P of the flattened output)
  or all-reduce.  The per-block INT32 accumulators are exact; the FP32 sum
  order differs from one chain, so outputs agree within a tolerance.

The slicing and assembly helpers are pure functions of NumPy/torch arrays so
the host logic can be exercised on CPU ranks (gloo).
"""
import ctypes

import numpy as np

from . import _lib as L
from . import backend


# ---------------------------------------------------------------- pure helpers

def column_bounds(N, world, rank):
    if N % (16 * world):
        raise ValueError(f"column-parallel needs N % (16*P) == 0 (N={N}, P={world})")
    n = N // world
    return rank * n, (rank + 1) * n


def block_bounds(K, world, rank):
    nblk = K // 32
    if K % 32 or nblk % world:
        raise ValueError(f"row-parallel needs (K/32) % P == 0 (K={K}, P={world})")
    b = nblk // world
    return rank * b, (rank + 1) * b


def _as_2d(x, rows):
    return x.reshape(rows, -1)


def column_shard(qweight, scales, qzeros, K, N, bits, world, rank):
    """MatMulNBits arrays of output rows [n0, n1) (a plain row slice of every array)."""
    n0, n1 = column_bounds(N, world, rank)
    qw = _as_2d(qweight, N)[n0:n1]
    sc = _as_2d(scales, N)[n0:n1]
    qz = None if qzeros is None else _as_2d(qzeros, N)[n0:n1]
    return qw, sc, qz, n1 - n0


def _unpack_zeros(qz, N, nblk):
    qz = np.asarray(qz).reshape(N, -1)
    z = np.empty((N, 2 * qz.shape[1]), np.uint8)
    z[:, 0::2] = qz & 15
    z[:, 1::2] = qz >> 4
    return z[:, :nblk]


def _pack_zeros(z):
    N, nblk = z.shape
    pad = np.zeros((N, 2 * ((nblk + 1) // 2)), np.uint8)
    pad[:, :nblk] = z
    return (pad[:, 0::2] | (pad[:, 1::2] << 4)).astype(np.uint8)


def row_shard(qweight, scales, qzeros, K, N, bits, world, rank):
    """MatMulNBits arrays of input blocks [b0, b1); INT4 zero points are
    re-packed two per byte starting at the shard's first block."""
    b0, b1 = block_bounds(K, world, rank)
    nblk = K // 32
    qw = np.asarray(qweight).reshape(N, nblk, -1)[:, b0:b1]
    sc = np.asarray(scales).reshape(N, nblk)[:, b0:b1]
    qz = None
    if qzeros is not None and bits == 4:
        qz = _pack_zeros(_unpack_zeros(qzeros, N, nblk)[:, b0:b1])
    return np.ascontiguousarray(qw), np.ascontiguousarray(sc), qz, 32 * (b1 - b0)


def assemble_columns(gathered):
    """[P, M, N/P] all-gather buffer -> [M, N] (rank-major column blocks)."""
    P, M, n = gathered.shape
    return gathered.permute(1, 0, 2).reshape(M, P * n) if hasattr(gathered, "permute") \
        else np.ascontiguousarray(gathered.transpose(1, 0, 2).reshape(M, P * n))


def scatter_bounds(M, N, world, rank):
    """Flat-index range of the output a rank keeps after reduce-scatter."""
    total = M * N
    if total % world:
        raise ValueError("M*N must be divisible by P for reduce-scatter")
    c = total // world
    return rank * c, (rank + 1) * c


# ---------------------------------------------------------------- collectives

def _dist():
    import torch.distributed as dist
    return dist


def gather_columns(local, group=None):
    """All-gather column shards [M, N/P] -> full [M, N] (NCCL all_gather_into_tensor)."""
    import torch
    dist = _dist()
    world = dist.get_world_size(group)
    if world == 1:
        return local
    M, n = local.shape
    buf = torch.empty((world, M, n), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, local.contiguous(), group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), local.contiguous(), group=group)
    return assemble_columns(buf)


class _DeviceArray:
    """``__cuda_array_interface__`` view of library-owned device memory, so
    torch can wrap it without a copy."""

    def __init__(self, ptr, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """One-shot all-gather of column-parallel outputs over peer memory.

    Each GPU stores its ``[M, N/P]`` slice straight into every GPU's output
    buffer over NVLink (CUDA IPC mappings, plain stores), then the GPUs
    hand-shake through flags in the same buffers (``ql_peer_allgather_cols_dev``).
    At decode sizes this replaces an NCCL all-gather whose cost is latency.
    Every rank of ``group`` builds one with the same ``max_bytes`` (capacity of
    the full ``[M, N]`` fp32 output) and makes the same sequence of
    :meth:`gather` calls.  The tensor :meth:`gather` returns is a view of this
    GPU's buffer: valid until the next call, for work on the same stream.
    """

    def __init__(self, max_bytes, group=None):
        import torch
        dist = _dist()
        self.lib = L.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("peer exchange supports up to 8 GPUs")
        max_bytes = (int(max_bytes) + 15) // 16 * 16
        handle = (ctypes.c_uint8 * 64)()
        x = ctypes.c_void_p()
        L.check(self.lib.ql_peer_exchange_create(max_bytes, ctypes.byref(handle), ctypes.byref(x)),
                "peer exchange create")
        self.x = x
        self.max_bytes = max_bytes
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        flat = (ctypes.c_uint8 * (64 * self.world)).from_buffer_copy(b"".join(handles))
        L.check(self.lib.ql_peer_exchange_connect(self.x, self.rank, self.world, ctypes.byref(flat)),
                "peer exchange connect")
        dist.barrier(group=group)
        self.out_ptr = self.lib.ql_peer_exchange_output(self.x)
        self._torch = torch

    def gather(self, local, check=False):
        """Full ``[M, N]`` from this GPU's ``[M, N/P]`` slice (contiguous fp32, CUDA).

        Asynchronous on the current stream (and capturable in a CUDA graph).
        Its flag waits are bounded: a peer that never makes the matching call
        leaves ``QL_ETIMEOUT`` in the device error word and a partly filled
        output.  ``check=True`` synchronises and raises on that; otherwise call
        :meth:`check` after synchronising (e.g. after a graph replay)."""
        torch = self._torch
        M, n = local.shape
        if local.dtype != torch.float32 or not local.is_contiguous() or local.data_ptr() % 16:
            local = local.to(torch.float32).contiguous().clone()
        if M * n * self.world * 4 > self.max_bytes:
            raise ValueError("output larger than the exchange's capacity")
        stream = torch.cuda.current_stream(local.device).cuda_stream
        L.check(self.lib.ql_peer_allgather_cols_dev(self.x, ctypes.c_void_p(local.data_ptr()), M, n,
                                                    ctypes.c_void_p(stream)), "peer all-gather")
        out = torch.as_tensor(_DeviceArray(self.out_ptr, (M, n * self.world)), device=local.device)
        if check:
            self.check()
        return out

    def check(self):
        """Synchronise this GPU and raise ``QLError`` (``QL_ETIMEOUT``) if a
        gather's bounded wait for a peer ran out since the last check; the
        device error word is cleared."""
        code = int(self.lib.ql_device_error(1))
        if code:
            raise L.QLError(code, "peer all-gather")

    def close(self):
        if self.x:
            self.lib.ql_peer_exchange_destroy(self.x)
            self.x = None


def reduce_partials(partial, mode="all", group=None):
    """Sum FP32 partials across ranks: ``mode='all'`` -> full [M, N] on every
    rank (all-reduce); ``mode='scatter'`` -> this rank's contiguous 1/P of the
    flattened output (reduce-scatter)."""
    import torch
    dist = _dist()
    world = dist.get_world_size(group)
    if world == 1:
        return partial if mode == "all" else partial.reshape(-1)
    if mode == "all":
        out = partial.contiguous()
        dist.all_reduce(out, group=group)
        return out
    flat = partial.contiguous().reshape(-1)
    rank = dist.get_rank(group)
    lo, hi = scatter_bounds(partial.shape[0], partial.shape[1], world, rank)
    if dist.get_backend(group) == "nccl":
        out = torch.empty(hi - lo, dtype=flat.dtype, device=flat.device)
        dist.reduce_scatter_tensor(out, flat, group=group)
        return out
    full = flat.clone()
    dist.all_reduce(full, group=group)
    return full[lo:hi].clone()


# ---------------------------------------------------------------- layers

class _Sharded:
    def __init__(self, group):
        dist = _dist()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.handle = None

    def close(self):
        if self.handle:
            backend.free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class ColumnParallelLinear(_Sharded):
    """``y = a @ W`` with W's N output features split across the group."""

    def __init__(self, qweight, scales, qzeros, K, N, bits=4, group=None):
        super().__init__(group)
        self.K, self.N, self.bits = int(K), int(N), bits
        qw, sc, qz, n = column_shard(np.asarray(qweight), np.asarray(scales),
                                     None if qzeros is None else np.asarray(qzeros),
                                     K, N, bits, self.world, self.rank)
        self.n_local = n
        self.handle = backend.prepack(np.ascontiguousarray(qw), np.ascontiguousarray(sc),
                                      None if qz is None else np.ascontiguousarray(qz), K, n, bits)

    def local(self, a):
        return backend.matmul(self.handle, a, self.n_local)

    def __call__(self, a):
        return gather_columns(self.local(a), self.group)


class RowParallelLinear(_Sharded):
    """``y = a @ W`` with W's K input features split across the group."""

    def __init__(self, qweight, scales, qzeros, K, N, bits=4, group=None):
        super().__init__(group)
        self.K, self.N, self.bits = int(K), int(N), bits
        qw, sc, qz, k = row_shard(qweight, scales, qzeros, K, N, bits, self.world, self.rank)
        self.k0 = self.rank * k
        self.k_local = k
        self.handle = backend.prepack(qw, sc, qz, k, N, bits)

    def local(self, a):
        """FP32 partial [M, N] over this rank's K slice of the full activations."""
        return backend.matmul(self.handle, a[:, self.k0:self.k0 + self.k_local].contiguous(), self.N)

    def __call__(self, a, mode="all"):
        return reduce_partials(self.local(a), mode, self.group)
