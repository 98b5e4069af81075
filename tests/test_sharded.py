"""Multi-GPU sharding host logic on CPU ranks (gloo, world_size 2).

The slicing (column_shard / row_shard, INT4 zero points re-packed at an odd
block boundary) and the assembly collectives (gather_columns, reduce_partials)
of breeze_engine_b200/sharded.py run on 2 CPU processes; each rank's local
compute is the oracle (test-only stand-in for the GPU kernel).  Column shards
must reassemble bit-exactly; row shards agree within 1e-5 relative per row
(FP32 sum order), while their per-block INT32 accumulators are exact slices of
the unsharded ones.
"""
import os
import socket

import numpy as np
import pytest

from breeze_engine_b200 import sharded


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _case(seed=3):
    rng = np.random.default_rng(seed)
    N, K, bits = 64, 6 * 32, 4          # 6 blocks: rank 1 of 2 starts at block 3 (odd)
    nblk = K // 32
    qw = rng.integers(0, 256, (N, nblk, 16), dtype=np.uint8)
    sc = rng.uniform(1e-3, 2e-2, (N, nblk)).astype(np.float16)
    qz = rng.integers(0, 256, (N, (nblk + 1) // 2), dtype=np.uint8)
    a = rng.standard_normal((5, K)).astype(np.float32)
    return qw, sc, qz, N, K, bits, a


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.oracle import Oracle
        o = Oracle()
        qw, sc, qz, N, K, bits, a = _case()
        full = o.matmul(qw, sc, qz, N, K, bits, a)
        hi, lo, asc = o.quantize_i16(a)
        cs_full = o.block_sums(qw, qz, N, K, bits, hi, lo)
        out = {}
        # column-parallel: shard rows of the MatMulNBits arrays, gather outputs
        cqw, csc, cqz, n = sharded.column_shard(qw, sc, qz, K, N, bits, world, rank)
        local = o.matmul(cqw, csc, cqz, n, K, bits, a)
        got = sharded.gather_columns(torch.from_numpy(local)).numpy()
        out["col_exact"] = bool(np.array_equal(got.view(np.uint32), full.view(np.uint32)))
        # row-parallel: shard K blocks, each rank quantizes its K slice
        rqw, rsc, rqz, k = sharded.row_shard(qw, sc, qz, K, N, bits, world, rank)
        k0 = rank * k
        a_loc = np.ascontiguousarray(a[:, k0:k0 + k])
        partial = o.matmul(rqw, rsc, rqz, N, k, bits, a_loc)
        hi_l, lo_l, _ = o.quantize_i16(a_loc)
        cs_loc = o.block_sums(rqw, rqz, N, k, bits, hi_l, lo_l)
        b0 = k0 // 32
        out["row_int32_exact"] = bool(np.array_equal(cs_loc, cs_full[:, :, b0:b0 + k // 32]))
        summed = sharded.reduce_partials(torch.from_numpy(partial.copy()), "all").numpy()
        rel = np.abs(summed - full).max(axis=1) / np.abs(full).max(axis=1)
        out["row_rel"] = float(rel.max())
        chunk = sharded.reduce_partials(torch.from_numpy(partial.copy()), "scatter").numpy()
        lo_i, hi_i = sharded.scatter_bounds(full.shape[0], full.shape[1], world, rank)
        out["scatter_rel"] = float(np.abs(chunk - full.reshape(-1)[lo_i:hi_i]).max() / np.abs(full).max())
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_sharding_on_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out in results.items():
        assert out["col_exact"], rank
        assert out["row_int32_exact"], rank
        assert out["row_rel"] <= 1e-5, out
        assert out["scatter_rel"] <= 1e-5, out


def test_shard_bounds_and_zero_point_repacking():
    qw, sc, qz, N, K, bits, a = _case()
    with pytest.raises(ValueError):
        sharded.column_bounds(48, 2, 0)            # 48 % (16*2) != 0
    with pytest.raises(ValueError):
        sharded.block_bounds(5 * 32, 2, 0)         # 5 blocks over 2 ranks
    # re-packed zero points of rank 1 (blocks 3..5) decode to the original nibbles
    _, _, rqz, k = sharded.row_shard(qw, sc, qz, K, N, bits, 2, 1)
    full = sharded._unpack_zeros(qz, N, K // 32)
    part = sharded._unpack_zeros(rqz, N, k // 32)
    assert np.array_equal(part, full[:, 3:6])
    # column shards concatenate back to the original arrays
    pieces = [sharded.column_shard(qw, sc, qz, K, N, bits, 4, r) for r in range(4)]
    assert np.array_equal(np.concatenate([p[0] for p in pieces]), qw.reshape(N, -1))
    assert np.array_equal(np.concatenate([p[2] for p in pieces]), qz.reshape(N, -1))
