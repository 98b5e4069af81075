"""Host-side checks of bench.py's multi-GPU plans (no GPU needed).

The driver runs `bench.py --gpus N` for N = 1, 2, 4, 8 with the default
decode workload.  At N > 1 only the LM head is column-sharded (NCCL
all-gather); the 50 MB layers stay whole and their calls are dealt to the
GPUs.  These tests pin that plan and the divisibility every sharded workload
needs at each N (output rows in whole 16-row groups per GPU, input blocks of 32
in equal shares for row-parallel layers).
"""
import collections

import pytest

import bench


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_decode_plan(world):
    wl = bench.DecodeWorkload
    plan = wl.plan(world)
    assert len(plan) == len(wl.shapes)
    owned = collections.Counter()
    for (K, N), (mode, owners) in zip(wl.shapes, plan):
        big = N * K * wl.bits // 8 >= wl.SHARD_BYTES
        if world == 1 or big:
            assert mode == "col" and owners is None
            assert N % (16 * world) == 0
        else:
            assert mode == "whole" and len(owners) == len(wl.Ms)
            assert all(0 <= o < world for o in owners)
            owned.update(owners)
    if world > 1:
        # every call of a whole layer runs on exactly one GPU, and the GPUs
        # get equal shares up to one call
        assert sum(owned.values()) == len(wl.Ms) * sum(1 for m, _ in plan if m == "whole")
        counts = [owned.get(r, 0) for r in range(world)]
        assert max(counts) - min(counts) <= 1


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_sharded_shapes_divide(world):
    """Every layer the other workloads column-shard (prefill, the 27B-class
    layer set, configs[4]'s column-parallel layer) splits into whole 16-row
    groups, and configs[4]'s row-parallel layer into whole 32-wide blocks."""
    col = [(bench.PrefillWorkload.K, bench.PrefillWorkload.N), (8192, 65536)]
    col += [(K, N) for _, K, N in bench.LayerSetWorkload.shapes]
    for K, N in col:
        assert N % (16 * world) == 0, (K, N, world)
    assert (65536 // 32) % world == 0


def test_mlp_front_workload_streams_from_hbm():
    """The fused MLP-front bench: decode-size batches (one decode launch per
    call), a concatenated width in whole 16-row groups, and rotated weight
    copies whose total is well above the 126 MB L2 so each call reads HBM."""
    wl = bench.MlpFrontWorkload
    assert max(wl.Ms) <= 64
    assert (2 * wl.INTER) % 16 == 0 and wl.H % 32 == 0
    one = bench.alg_bytes(0, wl.H, 2 * wl.INTER, wl.bits)
    assert wl.copies * one > 2 * bench.L2_BYTES
    assert wl().step_amount() == sum(bench.alg_bytes(M, wl.H, 2 * wl.INTER, wl.bits) + 4 * wl.H for M in wl.Ms)
