"""Host-side checks of bench.py's multi-GPU plans (no GPU needed).

The driver runs `bench.py --gpus N` for N = 1, 2, 4, 8 with the default
decode workload.  At N > 1 only large layers are sharded: the LM head
column-parallel (all-gather), configs[4]'s layers column- and row-parallel;
the decode sweep's 50 MB layers stay whole and their calls are dealt to the
GPUs; the prefill layer and the 27B-class layer set run as replicas (every
rank the whole layer on its own inputs, no collective).  These tests pin those
plans and the divisibility every sharded workload needs at each N (output
rows in whole 16-row groups per GPU, input blocks of 32 in equal shares for
row-parallel layers).
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
    """configs[4]'s column-parallel layer splits into whole 16-row groups and
    its row-parallel layer into whole 32-wide blocks at every N."""
    assert 65536 % (16 * world) == 0
    assert (65536 // 32) % world == 0


def test_small_layer_workloads_are_replicas():
    """Layers that are not large run whole on every rank at N > 1: the prefill
    layer and the layer set are replicas; the decode sweep and configs[4]
    shard."""
    assert bench.PrefillWorkload.replicas and bench.LayerSetWorkload.replicas
    assert not getattr(bench.DecodeWorkload, "replicas", False)
    assert not getattr(bench.ShardedWorkload, "replicas", False)


@pytest.mark.parametrize("mode,n_local,k_local", [("col", 4352, 5120), ("row", 17408, 1280),
                                                  ("whole", 17408, 5120), ("replica", 17408, 5120)])
def test_layer_geometry_per_mode(mode, n_local, k_local):
    """Rank 2 of 4: its slice of a 5120 x 17408 layer in each mode (no packing)."""
    layer = bench.Layer(None, 5120, 17408, 4, 4, 2, 0, 1, mode=mode, build=False)
    assert (layer.n_local, layer.k_local) == (n_local, k_local)
    assert layer.k0 == (2 * 1280 if mode == "row" else 0)


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
