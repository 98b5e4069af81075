#!/usr/bin/env python
"""Benchmark of the B200 quantized-linear hot path (one JSON line on rank 0).

Workloads (``--workload``):

* ``decode`` (default; configs[1] of the benchmark spec): the INT8 decode GEMV sweep --
  batch M in {1, 4, 8, 16} x (K, N) in {(4096, 12288), (12288, 4096),
  (4096, 151936)}, weights N(0, 0.02) packed to INT8 per output channel,
  activations N(0, 1) quantized to two-pass INT16.  One *step* is the 12 calls
  of the sweep.  ``value`` is the whole-job HBM throughput: algorithmic bytes of
  the 12 calls (``N*K*bits/8 + 2*N*K/32 + 4*M*K + 4*M*N`` each) / device time
  of the step, max over ranks.
* ``prefill``: the INT4 prefill GEMM -- M in {128, 512, 2048}
  tokens, K = 5120, N = 17408, weights N(0, 0.02) RTN-packed to INT4 with fp16
  scales, activations N(0, 1) with 1% of the channels scaled x20 (outliers),
  two-pass INT16.  One step is the 3 calls.  ``value`` is INT8 tera-operations
  per second counted as the headline metric does: ``4*M*N*K`` per call (two
  INT8 passes of 2*M*N*K each).  The default ``decode`` line also carries this
  workload's measurement under ``secondary.prefill``, and configs[3]'s INT4
  layer set at M = 1 under ``secondary.layer_m1``, and with ``--gpus P > 1``
  configs[4]'s sharded layers under ``secondary.sharded_m1`` /
  ``secondary.sharded_m2048`` (``--no-secondary`` skips them all), so one
  driver run measures both halves of the metric.
* ``mlp_front``: the front of a Qwen3.5-27B MLP block at decode batch sizes
  (M in {1, 4, 8, 16}; H = 5120, intermediate 17408, INT4 with fp16 scales):
  the RMSNorm fused into the activation quantizer, then one decode launch over
  the concatenated [gate; up] weight.  ``value`` is HBM GB/s of the step's
  algorithmic bytes; ``parts`` times the same step with gate and up as two
  launches and with the norm left out.  The reference arm runs the
  reference's own rmsnorm and two i4_matmul per M.  ``--gpus P`` runs P
  replicas.

With ``--gpus P`` (total work fixed, "strong" scaling) the decode sweep
column-shards the LM head (N/P per GPU; the output is all-gathered by the
library's one-shot peer-memory exchange, or by NCCL with ``--exchange nccl``)
and deals the calls of the two 50 MB layers round-robin over the GPUs as
whole, independent calls.  The calls of a step are independent, so each call's
collective runs on a second stream while the next call's matmul runs
(``--no-overlap`` serialises them);
``sharded_m1`` / ``sharded_m2048`` shard one layer column-parallel
and one row-parallel.  Layers that are not large -- ``prefill``'s 44.6 MB and
the 3-50 MB projections of ``layer_m1`` / ``layer_m512`` -- run whole on every
GPU, each rank on its own inputs (replicas, "weak" scaling, no collective).  Every
other config is also a parity-test case (tests/).

Inputs stay resident in HBM; every call streams its weights from HBM because
each layer is packed into several copies that are rotated (the working set of
a step is far above the 126 MB L2).

``--impl reference`` times the reference's own VNNI/OpenMP ``i4_matmul``
(oracle/_ref, built from kernel/quantized_matmul.cpp) on the host cores for the
same workload and metric; under torchrun only rank 0 runs it.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
DATA = ("synthetic: seeded N(0,0.02) weights RTN-packed to MatMulNBits (fp16 scales), "
        "seeded N(0,1) activations; identical in both arms")
FALLBACK_HBM_GBS = 6650.0
NOMINAL_INT8_TOPS = 4500.0           # dense INT8, B200 (NVIDIA's figure without sparsity)
SMS = 148


def alg_bytes(M, K, N, bits):
    """Algorithmic bytes of one call (the decode metric's formula, fp16 scales)."""
    return N * K * bits // 8 + 2 * N * (K // 32) + 4 * M * K + 4 * M * N


def decode_kernel_bytes(M, K, N, bits):
    """Algorithmic bytes of the weight-streaming kernel alone: packed weights,
    fp16 scales, the two INT8 activation planes and their scales, FP32 output."""
    return N * K * bits // 8 + 2 * N * (K // 32) + 2 * M * K + 4 * M * (K // 32) + 4 * M * N


def prefill_ops(M, K, N):
    """Algorithmic INT8 operations of one call: two INT8 passes of 2*M*N*K."""
    return 4 * M * N * K


# ------------------------------------------------------------------ helpers

def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak():
    """Dense 16-bit tensor peak from MEASURED_PEAKS.json (cuBLAS bf16 GEMM
    burst; FP16 runs at the same rate), else the profiling fallback."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured: cuBLAS bf16 GEMM 8192^3 burst (MEASURED_PEAKS.json)"
    except Exception:  # noqa: BLE001
        return 1590.0, "fallback: earlier bf16 measurement on this pool"


def measure_int8_tops(n=8192, iters=10):
    """Dense INT8 tensor-core peak of this GPU, measured now: cuBLASLt INT8
    GEMM (torch._int_mm, int32 output) on n^3, best of `iters` CUDA-event runs."""
    import torch
    try:
        a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda").t().contiguous().t()
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = None
        for _ in range(iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1) / 1e3
            best = t if best is None else min(best, t)
        del a, b
        torch.cuda.empty_cache()
        return 2.0 * n ** 3 / best / 1e12, f"measured: cuBLASLt INT8 GEMM (torch._int_mm) {n}^3, best of {iters}"
    except Exception as exc:  # noqa: BLE001
        return NOMINAL_INT8_TOPS, f"nominal dense INT8 (measurement failed: {type(exc).__name__})"


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the GPU is under load."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:  # noqa: BLE001
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "samples": len(sm), "reasons": sorted(reasons)}



class Layer:
    """One packed weight (possibly several rotation copies) of a (K, N) layer shard.

    ``mode='col'``: rank r keeps output rows [r N/P, (r+1) N/P) (column-parallel);
    ``mode='row'``: rank r keeps input blocks [r K/P, (r+1) K/P) (row-parallel);
    ``mode='whole'``: the full layer, packed only where ``build`` is true (the
    ranks that run one of its calls);
    ``mode='replica'``: the full layer on every rank, which runs its own calls
    (independent token streams, no collective)."""

    def __init__(self, lib, K, N, bits, world, rank, seed, copies, mode="col", build=True):
        import torch
        from breeze_engine_b200 import backend
        from breeze_engine_b200.quant import quantize_matmul_nbits_torch
        self.K, self.N, self.bits, self.mode = K, N, bits, mode
        if mode in ("whole", "replica"):
            world, rank = 1, 0
        self.n_local = N // world if mode != "row" else N
        self.k_local = K if mode != "row" else K // world
        self.k0 = 0 if mode != "row" else rank * self.k_local
        self.handles = []
        self.shard_bytes = self.n_local * self.k_local * bits // 8 + 2 * self.n_local * (self.k_local // 32)
        if not build:
            return
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        w = torch.randn((K, N), generator=g, device="cuda", dtype=torch.float32).mul_(0.02)
        qw, sc, qz = quantize_matmul_nbits_torch(w, bits=bits, per_channel=(bits == 8))
        del w
        nblk = K // 32
        if mode == "col":
            n0 = rank * self.n_local
            qw = qw[n0:n0 + self.n_local].contiguous()
            sc = sc.reshape(N, nblk)[n0:n0 + self.n_local].contiguous()
        elif mode == "row":
            b0, nb = self.k0 // 32, self.k_local // 32
            qw = qw.reshape(N, nblk, -1)[:, b0:b0 + nb].contiguous()
            sc = sc.reshape(N, nblk)[:, b0:b0 + nb].contiguous()
        self.handles = [backend.prepack(qw, sc, None, self.k_local, self.n_local, bits) for _ in range(copies)]
        del qw, sc
        torch.cuda.empty_cache()

    def free(self):
        from breeze_engine_b200 import backend
        for h in self.handles:
            backend.free(h)


# ------------------------------------------------------------------ workloads

def _outlier_acts(M, K, seed, dev="cuda"):
    """N(0, 1) activations with 1% of the channels scaled x20 (the outlier
    channels exercise the INT16 hi/lo split); seeded, on the device."""
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    a = torch.randn((M, K), generator=g, device=dev, dtype=torch.float32)
    ch = torch.randperm(K, generator=g, device=dev)[: max(1, K // 100)]
    a[:, ch] *= 20.0
    return a


def _to_host(acts):
    return {k: v.cpu().numpy() for k, v in acts.items()}


class DecodeWorkload:
    name = "decode"
    metric = "decode GEMV HBM throughput (INT8 weights, two-pass INT16 activations)"
    unit = "GB/s"
    shapes = [(4096, 12288), (12288, 4096), (4096, 151936)]   # (K, N)
    Ms = [1, 4, 8, 16]
    bits = 8
    kernel = "decode_kernel (ql_gemv.cu)"

    # Layers of at least this many weight bytes are column-sharded across the
    # GPUs (all-gather of the outputs); smaller layers stay whole and their
    # calls -- independent units of the sweep -- are dealt round-robin to the
    # GPUs, so only sharded shapes have a collective.
    SHARD_BYTES = 256 << 20

    @classmethod
    def plan(cls, world):
        """Per shape: ("col", None) -- column-sharded over all GPUs -- or
        ("whole", owners) with the owning GPU of each of its calls (one per M),
        dealt round-robin over the small layers' calls."""
        out, small = [], 0
        for K, N in cls.shapes:
            if world > 1 and N * K * cls.bits // 8 < cls.SHARD_BYTES:
                out.append(("whole", [(small + j) % world for j in range(len(cls.Ms))]))
                small += len(cls.Ms)
            else:
                out.append(("col", None))
        return out

    def build(self, lib, world, rank):
        import torch
        layers = []
        self.owners = {}
        for i, ((K, N), (mode, owners)) in enumerate(zip(self.shapes, self.plan(world))):
            if mode == "whole":
                shard = N * K
                copies = int(min(len(self.Ms), max(1, -(-2 * L2_BYTES // shard))))
                layer = Layer(lib, K, N, self.bits, world, rank, 1000 + i, copies, mode="whole",
                              build=rank in owners)
                for M, o in zip(self.Ms, owners):
                    self.owners[(id(layer), M)] = o
            else:
                shard = (N // world) * K + 2 * (N // world) * (K // 32)
                copies = int(min(len(self.Ms), max(1, -(-2 * L2_BYTES // shard))))
                layer = Layer(lib, K, N, self.bits, world, rank, 1000 + i, copies)
            layers.append(layer)
        acts = self.make_acts("cuda")
        calls = []
        for layer in layers:
            for j, M in enumerate(self.Ms):
                h = layer.handles[j % len(layer.handles)] if layer.handles else None
                calls.append((layer, h, M))
        return layers, acts, calls

    def step_amount(self, calls):
        return sum(alg_bytes(M, layer.K, layer.N, layer.bits) for layer, _, M in calls)

    def value(self, amount, seconds):
        return amount / seconds / 1e9

    def kernel_amount(self, M, K, n_local, bits):
        return decode_kernel_bytes(M, K, n_local, bits)

    def roofline(self, achieved, kern_amount_avg, calls, clock_mhz):
        peak, kind = measured_peaks()
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "decode_traffic.json")
        if self.name == "decode" and os.path.exists(tpath):     # captured on the INT8 sweep
            try:
                tr = json.load(open(tpath))
                traffic = round(tr["dram_bytes"] / tr["alg_bytes"] * kern_amount_avg)
            except Exception:  # noqa: BLE001
                traffic = None
        return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "peak_kind": kind,
                "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic}

    def config(self, world):
        return {"workload": "configs[1]: INT8 decode GEMV sweep", "M": self.Ms,
                "shapes_KN": self.shapes, "weights": "INT8 per-channel RTN, fp16 scales",
                "activations": "two-pass INT16 (hi_prec=1)",
                "l2": "rotated weight copies; step working set > L2",
                "timing": "CUDA graph of one step (12 quantize+matmul calls), CUDA events",
                "parallelism": ("1 GPU" if world == 1 else
                                f"LM head (661 MB) column-parallel N/{world} + NCCL all-gather; the 50 MB "
                                f"layers whole, their 8 calls dealt round-robin over the {world} GPUs")}

    def make_acts(self, dev):
        import torch
        g = torch.Generator(device=dev)
        g.manual_seed(7)
        acts = {}
        for K in sorted({k for k, _ in self.shapes}):
            for M in self.Ms:
                acts[(M, K)] = torch.randn((M, K), generator=g, device=dev, dtype=torch.float32)
        return acts

    def host_acts(self):
        return _to_host(self.make_acts(_gen_device()))

    def cpu_calls(self):
        """(K, N, bits, Ms, weight seed) of the bounded reference sample: the full sweep."""
        return [(K, N, self.bits, self.Ms, 1000 + i) for i, (K, N) in enumerate(self.shapes)]

    ref_calls = cpu_calls
    cpu_sample = "full decode sweeps (12 i4_matmul calls each)"


class PrefillWorkload:
    name = "prefill"
    metric = "prefill GEMM INT8 TOPS (INT4 weights, two-pass INT16 activations; 4*M*N*K per call)"
    unit = "TOPS"
    K, N, Ms, bits = 5120, 17408, [128, 512, 2048], 4
    kernel = "gemmw_kernel (ql_gemmw.cu, tcgen05 kind::f16 on per-call FP16-dequantized weights)"

    # A 44.6 MB weight is not a large layer: on several GPUs every rank runs the
    # whole layer on its own token batch (no collective; weak scaling).
    replicas = True

    def build(self, lib, world, rank):
        layer = Layer(lib, self.K, self.N, self.bits, world, rank, 3000, len(self.Ms),
                      mode="replica" if world > 1 else "col")
        acts = self.make_acts("cuda")
        calls = [(layer, layer.handles[j % len(layer.handles)], M) for j, M in enumerate(self.Ms)]
        return [layer], acts, calls

    def make_acts(self, dev):
        return {(M, self.K): _outlier_acts(M, self.K, 11 + M, dev) for M in self.Ms}

    def host_acts(self):
        return _to_host(self.make_acts(_gen_device()))

    def step_amount(self, calls):
        return sum(prefill_ops(M, layer.K, layer.N) for layer, _, M in calls)

    def value(self, amount, seconds):
        return amount / seconds / 1e12

    def kernel_amount(self, M, K, n_local, bits):
        return prefill_ops(M, K, n_local)

    def roofline(self, achieved, kern_amount_avg, calls, clock_mhz):
        # INT4 weights with fp16 scales in two-pass mode run gemmw_kernel: per
        # 32-wide block one K = 64 FP16 MMA (h and l/256 planes) = exactly the
        # 4*M*N*K operations counted here, on the FP16 tensor pipe.  Its roofline
        # is the measured dense 16-bit tensor peak; the INT8 peak (the metric
        # headline metric names) is reported beside it.
        f16_peak, f16_kind = measured_tensor_peak()
        int8_peak, int8_kind = measure_int8_tops()
        out = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(f16_peak, 1),
               "peak_kind": f16_kind, "unit": "TFLOP/s (FP16 tensor pipe; = counted INT8 TOPS)",
               "frac": round(achieved / f16_peak, 4), "traffic": None,
               "int8_peak": round(int8_peak, 1), "int8_peak_kind": int8_kind,
               "int8_peak_frac": round(achieved / int8_peak, 4)}
        # FP32 work of the epilogue: RN(D * 256*bscale) and fma(ascale, ., acc),
        # 2 operations per output per 32-wide block on the 128-lane FP32 pipe.
        if clock_mhz:
            fp32_ops_s = SMS * 128 * clock_mhz * 1e6
            ops_per_tops = 2.0 / (32 * 4)           # FP32 ops per counted op (4*M*N*K)
            out["fp32_epilogue_bound_tops"] = round(fp32_ops_s / ops_per_tops / 1e12, 1)
            out["fp32_epilogue_frac"] = round(achieved / out["fp32_epilogue_bound_tops"], 4)
        return out

    def config(self, world):
        return {"workload": "configs[2]: INT4 prefill GEMM", "M": self.Ms, "K": self.K, "N": self.N,
                "weights": "INT4 symmetric RTN, fp16 scales (block 32)",
                "activations": "two-pass INT16 (hi_prec=1); N(0,1), 1% channels x20",
                "l2": "3 rotated weight copies; step working set > L2",
                "timing": "CUDA graph of one step (3 quantize+GEMM calls), CUDA events",
                "parallelism": "1 GPU" if world == 1 else f"replicas on {world} GPUs (no collective)"}

    def cpu_calls(self):
        return [(self.K, self.N, self.bits, [128], 3000)]

    def ref_calls(self):
        return [(self.K, self.N, self.bits, self.Ms, 3000)]

    cpu_sample = "i4_matmul calls at M=128 (the smallest prefill size)"


class _OpsOrBytes:
    """Shared metric logic: HBM bytes for decode-sized M, INT8 ops for prefill-sized M."""
    bits = 4

    def __init__(self):
        self.unit = "GB/s" if self.M <= 64 else "TOPS"
        self.kernel = ("decode_dp4a_kernel (ql_gemv4.cu) for layers of >= 8192 rows at M <= 2, "
                       "decode_kernel (ql_gemv.cu) otherwise" if self.M <= 64
                       else "gemmw_kernel (ql_gemmw.cu, tcgen05 kind::f16 on per-call FP16-dequantized weights)")

    def step_amount(self, calls):
        if self.unit == "GB/s":
            return sum(alg_bytes(M, layer.K, layer.N, layer.bits) for layer, _, M in calls)
        return sum(prefill_ops(M, layer.K, layer.N) for layer, _, M in calls)

    def value(self, amount, seconds):
        return amount / seconds / (1e9 if self.unit == "GB/s" else 1e12)

    def kernel_amount(self, M, K, n_local, bits):
        return decode_kernel_bytes(M, K, n_local, bits) if self.unit == "GB/s" else prefill_ops(M, K, n_local)

    def roofline(self, achieved, kern_amount_avg, calls, clock_mhz):
        if self.unit == "GB/s":
            return DecodeWorkload.roofline(self, achieved, kern_amount_avg, calls, clock_mhz)
        return PrefillWorkload.roofline(self, achieved, kern_amount_avg, calls, clock_mhz)


class LayerSetWorkload(_OpsOrBytes):
    """the 27B-class decoder-layer projection set, 7 sequential calls."""
    shapes = [("q", 5120, 6144), ("k", 5120, 1024), ("v", 5120, 1024), ("o", 6144, 5120),
              ("gate", 5120, 17408), ("up", 5120, 17408), ("down", 17408, 5120)]

    def __init__(self, M):
        self.M = M
        self.name = f"layer_m{M}"
        super().__init__()
        self.metric = (f"27B-class layer projection set, M={M}: "
                       + ("HBM throughput" if self.unit == "GB/s" else "INT8 TOPS (4*M*N*K per call)"))

    # The projections (3-50 MB) are not large layers: on several GPUs every rank
    # runs the whole sequence on its own tokens (no collective; weak scaling).
    replicas = True

    def build(self, lib, world, rank):
        total = sum(K * N // 2 for _, K, N in self.shapes)
        copies = int(min(4, max(1, -(-2 * L2_BYTES // total))))
        layers = [Layer(lib, K, N, self.bits, world, rank, 4000 + i, copies, mode="replica" if world > 1 else "col")
                  for i, (_, K, N) in enumerate(self.shapes)]
        acts = {(self.M, K): _outlier_acts(self.M, K, 21 + K) for K in sorted({K for _, K, _ in self.shapes})}
        calls = [(layer, layer.handles[0], self.M) for layer in layers]
        self._rot = copies
        return layers, acts, calls

    def config(self, world):
        return {"workload": f"configs[3]: 27B-class layer projection set, M={self.M}",
                "layers_KN": {n: [K, N] for n, K, N in self.shapes},
                "weights": "INT4 symmetric RTN, fp16 scales (block 32)",
                "activations": "two-pass INT16 (hi_prec=1); N(0,1), 1% channels x20",
                "l2": "7-call step touches > L2 (192 MB of weights)",
                "timing": "CUDA graph of one step (7 quantize+matmul calls), CUDA events",
                "parallelism": "1 GPU" if world == 1 else f"replicas on {world} GPUs (no collective)"}

    def host_acts(self):
        dev = _gen_device()
        Ks = sorted({K for _, K, _ in self.shapes})
        return _to_host({(m, K): _outlier_acts(m, K, 21 + K, dev) for m in {self.M, min(self.M, 128)} for K in Ks})

    def cpu_calls(self):
        return [(K, N, self.bits, [min(self.M, 128)], 4000 + i) for i, (_, K, N) in enumerate(self.shapes)]

    def ref_calls(self):
        return [(K, N, self.bits, [self.M], 4000 + i) for i, (_, K, N) in enumerate(self.shapes)]

    @property
    def cpu_sample(self):
        return f"7-call layer sets at M={min(self.M, 128)}"


class ShardedWorkload(_OpsOrBytes):
    """column-parallel K=8192, N=65536 (all-gather of C) and
    row-parallel K=65536, N=8192 (reduce-scatter of FP32 partials), INT4."""

    def __init__(self, M):
        self.M = M
        self.name = f"sharded_m{M}"
        super().__init__()
        self.metric = (f"sharded INT4 linear (column- and row-parallel), M={M}: "
                       + ("HBM throughput" if self.unit == "GB/s" else "INT8 TOPS (4*M*N*K per call)"))

    def build(self, lib, world, rank):
        shard = (8192 * 65536 // 2) // world
        copies = int(min(4, max(1, -(-2 * L2_BYTES // (2 * shard)))))
        col = Layer(lib, 8192, 65536, self.bits, world, rank, 5000, copies, mode="col")
        row = Layer(lib, 65536, 8192, self.bits, world, rank, 5001, copies, mode="row")
        acts = {(self.M, 8192): _outlier_acts(self.M, 8192, 31), (self.M, 65536): _outlier_acts(self.M, 65536, 32)}
        calls = [(col, col.handles[0], self.M), (row, row.handles[0], self.M)]
        return [col, row], acts, calls

    def config(self, world):
        return {"workload": f"configs[4]: sharded INT4 linear, M={self.M}",
                "column_parallel_KN": [8192, 65536], "row_parallel_KN": [65536, 8192],
                "weights": "INT4 symmetric RTN, fp16 scales (block 32); one seed, sliced per rank",
                "activations": "two-pass INT16 (hi_prec=1); N(0,1), 1% channels x20",
                "l2": "rotated weight copies; step working set > L2",
                "timing": "CUDA graph of one step (2 sharded calls incl. NCCL), CUDA events",
                "parallelism": (f"P={world}: column-parallel + NCCL all-gather, row-parallel + NCCL reduce-scatter"
                                if world > 1 else "P=1 (no collective)")}

    def host_acts(self):
        dev = _gen_device()
        return _to_host({(m, K): _outlier_acts(m, K, seed, dev) for m in {self.M, min(self.M, 128)}
                         for K, seed in ((8192, 31), (65536, 32))})

    def cpu_calls(self):
        m = min(self.M, 128)
        return [(8192, 65536, self.bits, [m], 5000), (65536, 8192, self.bits, [m], 5001)]

    def ref_calls(self):
        return [(8192, 65536, self.bits, [self.M], 5000), (65536, 8192, self.bits, [self.M], 5001)]

    @property
    def cpu_sample(self):
        return f"the two layers at M={min(self.M, 128)}"


class MlpFrontWorkload:
    """The front of a Qwen3.5-27B MLP block at decode batch sizes: the
    reference decoder's rmsnorm, then gate and up on the normalised rows
    (kernel/qwen35_decoder.cpp:405-407; H = 5120, intermediate 17408, INT4
    weights with fp16 scales).  Here: ql_quantize_act_rmsnorm_dev (row factors
    + quantizer with the norm fused in) and ONE decode launch over the
    concatenated [gate; up] weight (ql_weight_concat).  Every rank runs the
    same independent work (replicas)."""
    name = "mlp_front"
    metric = "fused RMSNorm + gate|up decode HBM throughput (INT4 weights, two-pass INT16 activations)"
    unit = "GB/s"
    H, INTER = 5120, 17408
    Ms = [1, 4, 8, 16]
    bits = 4
    eps = 1e-6
    copies = 3                    # 3 x 100 MB of [gate; up] rotated: each call streams from HBM
    kernel = "decode_kernel (ql_gemv.cu) on the concatenated gate|up weight"
    cpu_sample = "full sweeps (per M: the reference rmsnorm + gate and up i4_matmul)"

    def step_amount(self):
        """Algorithmic bytes of one step: per M the gate|up weights and fp16
        scales, the rows x, the norm weights and the outputs."""
        return sum(alg_bytes(M, self.H, 2 * self.INTER, self.bits) + 4 * self.H for M in self.Ms)

    def value(self, amount, seconds):
        return amount / seconds / 1e9

    def config(self, world):
        return {"workload": "MLP front of Qwen3.5-27B (rmsnorm -> gate, up) at decode batch sizes",
                "M": self.Ms, "H": self.H, "intermediate": self.INTER,
                "weights": "INT4 symmetric RTN, fp16 scales (gate and up concatenated along N)",
                "activations": "two-pass INT16 (hi_prec=1); rows N(0,1), 1% channels x20",
                "l2": f"{self.copies} rotated weight copies (300 MB); each call streams from HBM",
                "timing": "CUDA graph of one step (per M: norm factors, fused quantize, one matmul), CUDA events",
                "parallelism": "1 GPU" if world == 1 else f"replicas on {world} GPUs (no collective)"}


def run_mlp_front(args):
    import torch
    import torch.distributed as dist
    from breeze_engine_b200 import _lib as L
    from breeze_engine_b200 import backend

    wl = MlpFrontWorkload()
    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    lib = L.load()
    backend.set_hi_prec(True)
    H, I = wl.H, wl.INTER
    gate = Layer(lib, H, I, wl.bits, 1, 0, 2001, wl.copies)
    up = Layer(lib, H, I, wl.bits, 1, 0, 2002, wl.copies)
    both = [backend.concat_packed([g, u]) for g, u in zip(gate.handles, up.handles)]
    g = torch.Generator(device="cuda")
    g.manual_seed(2003)
    norm_w = (1.0 + 0.1 * torch.randn(H, generator=g, device="cuda")).float()
    xs = {M: _outlier_acts(M, H, 2100 + M) for M in wl.Ms}
    nws = {M: lib.ql_norm_act_workspace_bytes(M, H) for M in wl.Ms}
    wss = {M: torch.empty(nws[M], dtype=torch.uint8, device="cuda") for M in wl.Ms}
    outs = {M: torch.empty((M, 2 * I), dtype=torch.float32, device="cuda") for M in wl.Ms}
    outs_g = {M: torch.empty((M, I), dtype=torch.float32, device="cuda") for M in wl.Ms}
    outs_u = {M: torch.empty((M, I), dtype=torch.float32, device="cuda") for M in wl.Ms}
    stream = torch.cuda.current_stream()

    def ok(rc, what):
        if rc:
            raise RuntimeError(f"{what} failed: {lib.ql_error_string(rc)}")

    def quant_norm(M, s):
        ok(lib.ql_quantize_act_rmsnorm_dev(xs[M].data_ptr(), norm_w.data_ptr(), wl.eps, M, H, 1,
                                           wss[M].data_ptr(), nws[M], None, s), "quantize+norm")

    def fused(j, M, s):
        quant_norm(M, s)
        ok(lib.ql_matmul_quantized_dev(ctypes.c_void_p(both[j % wl.copies]), wss[M].data_ptr(), M, 1,
                                       outs[M].data_ptr(), s), "matmul")

    def separate(j, M, s):
        quant_norm(M, s)
        for hs, o in ((gate.handles, outs_g), (up.handles, outs_u)):
            ok(lib.ql_matmul_quantized_dev(ctypes.c_void_p(hs[j % wl.copies]), wss[M].data_ptr(), M, 1,
                                           o[M].data_ptr(), s), "matmul")

    def no_norm(j, M, s):
        ok(lib.ql_quantize_act_dev(xs[M].data_ptr(), M, H, 1, wss[M].data_ptr(), nws[M], s), "quantize")
        ok(lib.ql_matmul_quantized_dev(ctypes.c_void_p(both[j % wl.copies]), wss[M].data_ptr(), M, 1,
                                       outs[M].data_ptr(), s), "matmul")

    def matmul_only(j, M, s):
        ok(lib.ql_matmul_quantized_dev(ctypes.c_void_p(both[j % wl.copies]), wss[M].data_ptr(), M, 1,
                                       outs[M].data_ptr(), s), "matmul")

    def make_graph(body):
        for _ in range(2):
            for j, M in enumerate(wl.Ms):
                body(j, M, stream.cuda_stream)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            s = torch.cuda.current_stream().cuda_stream
            for j, M in enumerate(wl.Ms):
                body(j, M, s)
        return gr

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(t):
        if world > 1:
            tt = torch.tensor([t], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    def timed(gr, n, label="bench"):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(label)          # lets ncu --nvtx restrict a capture to it
        e0.record(stream)
        for _ in range(n):
            gr.replay()
        e1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / 1e3)

    graphs = {name: make_graph(body) for name, body in
              (("fused", fused), ("separate", separate), ("no_norm", no_norm))}
    # self-check: one launch over [gate; up] == the two separate launches, bit for bit
    graphs["fused"].replay()
    graphs["separate"].replay()
    torch.cuda.synchronize()
    for M in wl.Ms:
        if not (torch.equal(outs[M][:, :I].view(torch.int32), outs_g[M].view(torch.int32)) and
                torch.equal(outs[M][:, I:].view(torch.int32), outs_u[M].view(torch.int32))):
            raise RuntimeError(f"concatenated gate|up differs from separate launches at M={M}")

    for _ in range(args.warmup):
        graphs["fused"].replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    t_probe = timed(graphs["fused"], 3) / 3
    timed(graphs["fused"], max(1, int(1.0 / max(t_probe, 1e-6))))
    t = timed(graphs["fused"], args.steps, label="timed")
    clock_info = clocks.stop()
    clock_info["window"] = "sampled over ~1 s of back-to-back steps plus the timed region"
    parts = {"fused_us_per_step": round(t / args.steps * 1e6, 2)}
    for name in ("separate", "no_norm"):
        for _ in range(args.warmup):
            graphs[name].replay()
        parts[f"{name}_us_per_step"] = round(timed(graphs[name], args.steps) / args.steps * 1e6, 2)
    amount = wl.step_amount()
    value = world * wl.value(amount * args.steps, t)

    # the matmul kernel alone (its activations quantized above), for the roofline
    gk = make_graph(matmul_only)
    for _ in range(args.warmup):
        gk.replay()
    tk = timed(gk, args.steps) / args.steps
    kern_amount = sum(decode_kernel_bytes(M, H, 2 * I, wl.bits) for M in wl.Ms)
    achieved = kern_amount / tk / 1e9
    peak, kind = measured_peaks()
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "peak_kind": kind,
                "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                "kernel": wl.kernel, "us_per_launch": round(tk / len(wl.Ms) * 1e6, 2)}

    # end to end: x from pinned host memory, the fused calls, outputs back to pinned memory
    e2e = None
    if not args.no_e2e:
        hx = {M: xs[M].cpu().pin_memory() for M in wl.Ms}
        hc = {M: torch.empty((M, 2 * I), dtype=torch.float32).pin_memory() for M in wl.Ms}

        def e2e_step():
            for j, M in enumerate(wl.Ms):
                xs[M].copy_(hx[M], non_blocking=True)
                fused(j, M, stream.cuda_stream)
                hc[M].copy_(outs[M], non_blocking=True)
            stream.synchronize()

        for _ in range(args.warmup):
            e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        t_e2e = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": round(world * wl.value(amount * args.steps, t_e2e), 2), "unit": wl.unit,
               "h2d_bytes_per_step": int(sum(4 * M * H for M in wl.Ms)),
               "d2h_bytes_per_step": int(sum(4 * M * 2 * I for M in wl.Ms)),
               "api": "ql_quantize_act_rmsnorm_dev + ql_matmul_quantized_dev, pinned host buffers"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = mlp_front_cpu(wl, samples=2)
    if rank == 0:
        line = {"metric": wl.metric, "value": round(value, 2), "unit": wl.unit, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "s8xs8/u8->s32, f32 rescale; f64 row sums",
                "data": "synthetic (seeded N(0,0.02) weights, N(0,1) rows with outlier channels)",
                "config": wl.config(world), "roofline": roofline, "parts": parts,
                "gpu_launches": 3 * len(wl.Ms) * args.steps, "clocks": clock_info}
        if e2e:
            line["e2e"] = e2e
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del graphs, gk
    for h in both:
        backend.free(h)
    gate.free()
    up.free()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


WORKLOADS = {"decode": DecodeWorkload, "prefill": PrefillWorkload, "mlp_front": MlpFrontWorkload,
             "layer_m1": lambda: LayerSetWorkload(1), "layer_m512": lambda: LayerSetWorkload(512),
             "sharded_m1": lambda: ShardedWorkload(1), "sharded_m2048": lambda: ShardedWorkload(2048)}


# ------------------------------------------------------------------ our arm

def run_ours(args):
    import torch
    import torch.distributed as dist
    from breeze_engine_b200 import _lib as L
    from breeze_engine_b200 import backend

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    lib = L.load()
    backend.set_hi_prec(True)
    line = _measure(args, WORKLOADS[args.workload](), lib, rank, local_rank, world)
    # The headline metric names both halves of the path: the default decode
    # line also carries configs[2]'s prefill GEMM and configs[3]'s INT4 layer set
    # at one token (the 27B-class decode shapes), measured the same way; on
    # several GPUs also configs[4], the sharded layers at 1 and 2048 tokens.
    if args.workload == "decode" and not args.no_secondary:
        keep = ("metric", "value", "unit", "ms_per_step", "steps", "scaling", "config", "roofline", "e2e",
                "cpu_baseline", "gpu_launches", "clocks")
        extra = [("prefill", PrefillWorkload), ("layer_m1", lambda: LayerSetWorkload(1))]
        if world > 1:
            extra += [("sharded_m1", lambda: ShardedWorkload(1)), ("sharded_m2048", lambda: ShardedWorkload(2048))]
        for name, make in extra:
            sec = _measure(args, make(), lib, rank, local_rank, world)
            if rank == 0:
                line.setdefault("secondary", {})[name] = {k: sec[k] for k in keep if k in sec}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def _measure(args, wl, lib, rank, local_rank, world):
    """One workload on this rank: the timed step (value), the kernel-only
    pass (roofline), the host-pointer pass (e2e) and, on rank 0 at N = 1, the
    reference's CPU path (cpu_baseline).  Returns the JSON line on rank 0."""
    import torch
    import torch.distributed as dist
    from breeze_engine_b200.sharded import gather_columns, reduce_partials

    layers, acts, calls = wl.build(lib, world, rank)
    owners = getattr(wl, "owners", {})
    exchange = None
    if world > 1 and args.exchange == "peer" and any(layer.mode == "col" for layer, _, _ in calls):
        # one peer-memory exchange sized for the largest column-parallel output
        from breeze_engine_b200.sharded import PeerExchange
        cap = max([4 * M * layer.N for layer, _, M in calls if layer.mode == "col"] or [16])
        exchange = PeerExchange(cap)

    def mine(layer, M):
        """Whether this rank runs the call: every rank for sharded layers, the
        owner for whole layers dealt to one GPU."""
        return layer.mode != "whole" or owners.get((id(layer), M)) == rank

    outs, wss, local_a = {}, {}, {}
    for layer, h, M in calls:
        if not mine(layer, M):
            continue
        outs[(id(layer), M)] = torch.empty((M, layer.n_local), dtype=torch.float32, device="cuda")
        need = lib.ql_workspace_bytes(ctypes.c_void_p(h), M)
        if (layer.k_local, M) not in wss or wss[(layer.k_local, M)].numel() < need:
            wss[(layer.k_local, M)] = torch.empty(need, dtype=torch.uint8, device="cuda")
        # row-parallel: this rank's contiguous K slice of the activations
        local_a[(id(layer), M)] = (acts[(M, layer.K)] if layer.mode != "row" else
                                   torch.empty((M, layer.k_local), dtype=torch.float32, device="cuda"))

    # The calls of a step are independent units: with overlap, each call's
    # collective runs on a second stream while the next call's matmul runs,
    # and the step ends only when every collective has (the stream joins back).
    comm = torch.cuda.Stream() if world > 1 and not args.no_overlap else None

    def collective(layer, c):
        if layer.mode == "col":
            if exchange is not None:
                exchange.gather(c)
            else:
                gather_columns(c)
        elif layer.mode == "row":
            reduce_partials(c, "scatter")

    def step():
        main = torch.cuda.current_stream()
        s_ptr = main.cuda_stream
        forked = False
        for layer, h, M in calls:
            if not mine(layer, M):
                continue
            a, c, ws = local_a[(id(layer), M)], outs[(id(layer), M)], wss[(layer.k_local, M)]
            if layer.mode == "row":
                a.copy_(acts[(M, layer.K)][:, layer.k0:layer.k0 + layer.k_local])
            rc = lib.ql_matmul_dev_ws(ctypes.c_void_p(h), a.data_ptr(), M, c.data_ptr(),
                                      ws.data_ptr(), ws.numel(), s_ptr)
            if rc:
                raise RuntimeError(f"ql_matmul_dev_ws failed: {rc}")
            if world > 1 and layer.mode in ("col", "row"):
                if comm is None:
                    collective(layer, c)
                else:
                    done = torch.cuda.Event()
                    done.record(main)
                    comm.wait_event(done)
                    with torch.cuda.stream(comm):
                        collective(layer, c)
                    forked = True
        if forked:                            # join only a stream this step forked
            main.wait_stream(comm)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(t):
        if world > 1:
            tt = torch.tensor([t], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    # Eager warm-up (function attributes, NCCL communicators), then one CUDA
    # graph per step so host submission latency never shows in device time.
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream()

    def timed_replays(g, n, label="bench"):
        """Device time of n replays of graph g, max over ranks; a rank with no
        graph (a call another GPU owns) takes part in the barriers with 0."""
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(label)          # lets ncu --nvtx restrict a capture to it
        e0.record(stream)
        for _ in range(n if g is not None else 0):
            g.replay()
        e1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / 1e3 if g is not None else 0.0)

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    # Clock window: keep the same load running ~1 s while nvidia-smi samples,
    # then take the timed region right after it.
    clocks = ClockSampler(local_rank)
    clocks.start()
    t_probe = timed_replays(graph, 3) / 3
    n_window = max(1, int(1.0 / max(t_probe, 1e-6)))
    timed_replays(graph, n_window)
    t = timed_replays(graph, args.steps, label="timed")
    clock_info = clocks.stop()
    clock_info["window"] = "sampled over ~1 s of back-to-back steps plus the timed region"

    step_amount = wl.step_amount(calls)
    replicas = world > 1 and getattr(wl, "replicas", False)
    if replicas:
        step_amount *= world                  # every rank ran the whole step on its own inputs
    value = wl.value(step_amount * args.steps, t)

    # ---- per-launch pass (roofline): the matmul kernel alone, on activations
    # quantized once, REPS launches per call rotating over the layer's weight
    # copies, captured in a graph and timed with CUDA events.
    qws = {}
    for layer, h, M in calls:
        key = (id(layer), M)
        if key not in qws and mine(layer, M):
            a = local_a[key]
            if layer.mode == "row":
                a.copy_(acts[(M, layer.K)][:, layer.k0:layer.k0 + layer.k_local])
            n = lib.ql_act_workspace_bytes(M, layer.k_local)
            qws[key] = torch.empty(n, dtype=torch.uint8, device="cuda")
            rc = lib.ql_quantize_act_dev(a.data_ptr(), M, layer.k_local, 1, qws[key].data_ptr(), n,
                                         stream.cuda_stream)
            assert rc == 0
    torch.cuda.synchronize()
    REPS = 8 if wl.name == "decode" else 4
    kern_t, kern_amount, per_call = 0.0, 0, []
    for layer, h0, M in calls:
        gk = None
        if mine(layer, M):
            c, ws = outs[(id(layer), M)], qws[(id(layer), M)]
            # INT4 prefill takes the FP16-operand GEMM: prepare one workspace per
            # weight copy with a full call, then time the GEMM kernel alone on them
            prep = []
            if M > 64 and lib.ql_workspace_bytes(ctypes.c_void_p(h0), M) > lib.ql_act_workspace_bytes(M, layer.k_local):
                a = local_a[(id(layer), M)]
                for h in layer.handles:
                    n = lib.ql_workspace_bytes(ctypes.c_void_p(h), M)
                    w = torch.empty(n, dtype=torch.uint8, device="cuda")
                    assert lib.ql_matmul_dev_ws(ctypes.c_void_p(h), a.data_ptr(), M, c.data_ptr(), w.data_ptr(), n,
                                                stream.cuda_stream) == 0
                    prep.append((h, w, n))
                torch.cuda.synchronize()
                if lib.ql_prefill_gemm_dev(ctypes.c_void_p(prep[0][0]), prep[0][1].data_ptr(), prep[0][2], M, 1,
                                           c.data_ptr(), stream.cuda_stream) != 0:
                    prep = []
            gk = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gk):
                s_ptr = torch.cuda.current_stream().cuda_stream
                for r in range(REPS):
                    if prep:
                        h, w, n = prep[(layer.handles.index(h0) + r) % len(prep)]
                        rc = lib.ql_prefill_gemm_dev(ctypes.c_void_p(h), w.data_ptr(), n, M, 1, c.data_ptr(), s_ptr)
                    else:
                        h = layer.handles[(layer.handles.index(h0) + r) % len(layer.handles)]
                        rc = lib.ql_matmul_quantized_dev(ctypes.c_void_p(h), ws.data_ptr(), M, 1, c.data_ptr(),
                                                         s_ptr)
                    assert rc == 0
            gk.replay()
        nrep = max(2, args.steps // 2)
        dt = timed_replays(gk, nrep) / (nrep * REPS)
        amt = wl.kernel_amount(M, layer.k_local, layer.n_local, layer.bits)
        kern_t += dt
        kern_amount += amt
        per_call.append({"M": M, "K": layer.k_local, "N": layer.n_local, "us": round(dt * 1e6, 2),
                         wl.unit: round(wl.value(amt, dt), 1)})
        del gk
        prep = []
    achieved = wl.value(kern_amount, kern_t)
    roofline = wl.roofline(achieved, kern_amount / len(calls), calls, clock_info.get("sm_mhz"))
    roofline["kernel"] = wl.kernel
    roofline["per_call"] = per_call

    # ---- end to end through the reference-compatible host C ABI (i4_matmul)
    e2e = None
    if not args.no_e2e:
        host_a = {k: v.cpu().pin_memory() for k, v in local_a.items()}
        host_c = {k: torch.empty(tuple(v.shape), dtype=torch.float32).pin_memory() for k, v in outs.items()}

        def e2e_step():
            for layer, h, M in calls:
                if not mine(layer, M):
                    continue
                a = host_a[(id(layer), M)]
                c = host_c[(id(layer), M)]
                lib.i4_matmul(ctypes.c_void_p(h), ctypes.c_void_p(a.data_ptr()), M, ctypes.c_void_p(c.data_ptr()))
            return lib.ql_last_status()

        for _ in range(max(1, args.warmup)):
            assert e2e_step() == 0
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        t_e2e = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": round(wl.value(step_amount * args.steps, t_e2e), 2), "unit": wl.unit,
               "h2d_bytes_per_step": int(sum(4 * M * layer.k_local for layer, _, M in calls)),
               "d2h_bytes_per_step": int(sum(4 * M * layer.n_local for layer, _, M in calls)),
               "api": "i4_matmul (host pointers, pinned buffers, synchronous)"
                      + ("; outputs stay sharded per rank (no collective)" if world > 1 else "")}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl)

    line = None
    if rank == 0:
        cfg = wl.config(world)
        if world > 1 and any(layer.mode == "col" for layer, _, _ in calls):
            cfg["exchange"] = ("one-shot peer-memory all-gather (ql_peer_allgather_cols_dev)"
                               if exchange is not None else "NCCL all_gather_into_tensor")
            cfg["overlap"] = ("each call's collective on a second stream, overlapping the next call"
                              if comm is not None else "none")
            if exchange is not None and "parallelism" in cfg:
                cfg["parallelism"] = cfg["parallelism"].replace("NCCL all-gather", "peer-memory all-gather")
        line = {
            "metric": wl.metric, "value": round(value, 2), "unit": wl.unit, "impl": "ours", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "weak" if replicas else "strong", "vs_baseline": None,
            "dtype": "s8xs8/u8->s32, f32 rescale",
            "data": DATA,
            "config": cfg,
            "roofline": roofline,
            "gpu_launches": 2 * sum(1 for layer, _, M in calls if mine(layer, M)) * args.steps,
            "clocks": clock_info,
        }
        if e2e:
            line["e2e"] = e2e
        if cpu:
            line["cpu_baseline"] = cpu

    del graph
    for layer in layers:
        layer.free()
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
    if exchange is not None:
        exchange.close()
    return line


# ------------------------------------------------------------------ CPU reference

def cpu_has_vnni():
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        return False
    return "avx512_vnni" in flags and "avx512vbmi" in flags


def host_weights(K, N, bits, seed):
    """Random MatMulNBits codes + fp16 scales (CPU timing does not depend on values)."""
    rng = np.random.default_rng(seed)
    qw = rng.integers(0, 256, (N, K // 32, 4 * bits), dtype=np.uint8)
    sc = (rng.random(N * (K // 32), dtype=np.float32) * 0.02 + 0.001).astype(np.float16)
    return qw, sc


def _gen_device():
    import torch
    return "cuda" if torch.cuda.is_available() else "cpu"


def rtn_host_weights(K, N, bits, seed):
    """The GPU arm's layer weights (Layer: seeded N(0, 0.02), RTN-packed by
    quantize_matmul_nbits_torch), generated the same way and copied to host
    memory, so both arms multiply the same MatMulNBits arrays."""
    import torch
    from breeze_engine_b200.quant import quantize_matmul_nbits_torch
    dev = _gen_device()
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w = torch.randn((K, N), generator=g, device=dev, dtype=torch.float32).mul_(0.02)
    qw, sc, _ = quantize_matmul_nbits_torch(w, bits=bits, per_channel=(bits == 8))
    del w
    return qw.cpu().numpy(), sc.cpu().numpy()


def _reference_lib():
    from oracle.oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        return None, "oracle/_ref/libbreeze_ref.so not built (needs the reference checkout)"
    if not cpu_has_vnni():
        return None, "host CPU lacks AVX-512 VNNI/VBMI required by the reference kernel"
    return Reference(), None


class _RefCalls:
    """The reference's i4_matmul over the workload's calls, host buffers: the
    GPU arm's weights (rtn_host_weights with the layer's seed) and activations
    (the workload's own generator), copied to host memory."""

    def __init__(self, ref, wl, spec, threads):
        self.ref = ref
        self.handles = []
        for K, N, bits, Ms, seed in spec:
            qw, sc = rtn_host_weights(K, N, bits, seed)
            self.handles.append((K, N, bits, Ms, ref.prepack(qw, sc, None, K, N, bits)))
            del qw
        acts = wl.host_acts()
        self.acts = {(M, K): acts[(M, K)] for K, _, _, Ms, _ in spec for M in Ms}
        self.outs = {(M, N): np.empty((M, N), np.float32) for _, N, _, Ms, _ in spec for M in Ms}
        ref.lib.i4_set_threads(threads)
        ref.lib.i4_set_hi_prec(1)

    def step(self):
        for K, N, _, Ms, h in self.handles:
            for M in Ms:
                self.ref.lib.i4_matmul(ctypes.c_void_p(h), self.acts[(M, K)].ctypes.data, M,
                                       self.outs[(M, N)].ctypes.data)

    def amount(self, wl):
        if wl.unit == "GB/s":
            return sum(alg_bytes(M, K, N, bits) for K, N, bits, Ms, _ in self.handles for M in Ms)
        return sum(prefill_ops(M, K, N) for K, N, _, Ms, _ in self.handles for M in Ms)

    def free(self):
        for *_, h in self.handles:
            self.ref.free(h)


def _median_sample(step, samples, warmup=2):
    """Median wall time of `samples` calls of step() after `warmup` calls."""
    for _ in range(warmup):
        step()
    times = []
    for _ in range(samples):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    return statistics.median(times)


def _host_desc(threads):
    model = ""
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    numa = len([d for d in os.listdir("/sys/devices/system/node") if d.startswith("node")]) \
        if os.path.isdir("/sys/devices/system/node") else 1
    return f"{model or 'unknown CPU'}, {os.cpu_count()} logical CPUs, {numa} NUMA node(s), {threads} OpenMP threads"


def cpu_baseline(wl, samples=10):
    """The reference i4_matmul (OpenMP, all host threads) on a bounded sample:
    the median of `samples` timed steps after 2 warm-ups, on the GPU arm's
    weights and activations."""
    os.environ.setdefault("OMP_PROC_BIND", "spread")
    os.environ.setdefault("OMP_PLACES", "cores")
    ref, why = _reference_lib()
    if ref is None:
        return {"value": None, "unit": wl.unit, "cores": 0, "kind": "reference", "sample": why}
    threads = os.cpu_count() or 1
    rc = _RefCalls(ref, wl, wl.cpu_calls(), threads)
    dt = _median_sample(rc.step, samples)
    value = wl.value(rc.amount(wl), dt)
    rc.free()
    return {"value": round(value, 4 if wl.unit == "TOPS" else 2), "unit": wl.unit, "cores": threads,
            "kind": "reference", "ms_per_step": round(dt * 1e3, 2),
            "sample": f"median of {samples} x {wl.cpu_sample} after 2 warm-ups, set_hi_prec(1), "
                      f"OMP_PROC_BIND=spread; host: {_host_desc(threads)}"}


class _RefMlpFront:
    """The reference decoder's MLP front on the host: its own rmsnorm
    (kernel/qwen35_decoder.cpp:133-141, through oracle/ref_norm_probe.cpp) and
    i4_matmul for gate and up (:406-407), per M of the workload."""

    def __init__(self, ref, wl, threads):
        self.ref, self.wl = ref, wl
        H, I = wl.H, wl.INTER
        self.handles = []
        for i in range(2):
            qw, sc = host_weights(H, I, wl.bits, 300 + i)
            self.handles.append(ref.prepack(qw, sc, None, H, I, wl.bits))
            del qw
        rng = np.random.default_rng(9)
        self.norm_w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        self.xs = {M: rng.standard_normal((M, H)).astype(np.float32) for M in wl.Ms}
        self.hn = {M: np.empty((M, H), np.float32) for M in wl.Ms}
        self.outs = {M: np.empty((M, I), np.float32) for M in wl.Ms}
        ref.lib.i4_set_threads(threads)
        ref.lib.i4_set_hi_prec(1)

    def step(self):
        lib = self.ref.lib
        for M in self.wl.Ms:
            lib.refprobe_rmsnorm(self.hn[M].ctypes.data, self.xs[M].ctypes.data, self.norm_w.ctypes.data,
                                 M, self.wl.H, ctypes.c_float(self.wl.eps))
            for h in self.handles:
                lib.i4_matmul(ctypes.c_void_p(h), self.hn[M].ctypes.data, M, self.outs[M].ctypes.data)

    def amount(self, wl):
        return wl.step_amount()

    def free(self):
        for h in self.handles:
            self.ref.free(h)


def mlp_front_cpu(wl, samples=2):
    """cpu_baseline of the MLP-front workload (the reference's rmsnorm + two
    i4_matmul per M, OpenMP on all host threads)."""
    os.environ.setdefault("OMP_PROC_BIND", "spread")
    os.environ.setdefault("OMP_PLACES", "cores")
    ref, why = _reference_lib()
    if ref is None:
        return {"value": None, "unit": wl.unit, "cores": 0, "kind": "reference", "sample": why}
    threads = os.cpu_count() or 1
    rc = _RefMlpFront(ref, wl, threads)
    rc.step()
    t0 = time.perf_counter()
    for _ in range(samples):
        rc.step()
    dt = time.perf_counter() - t0
    rc.free()
    return {"value": round(wl.value(wl.step_amount() * samples, dt), 2), "unit": wl.unit, "cores": threads,
            "kind": "reference", "ms_per_step": round(dt / samples * 1e3, 2),
            "sample": f"{samples} x {wl.cpu_sample} after 1 warm-up, set_hi_prec(1), "
                      f"OpenMP {threads} threads, OMP_PROC_BIND=spread"}


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]()
    os.environ.setdefault("OMP_PROC_BIND", "spread")
    os.environ.setdefault("OMP_PLACES", "cores")
    ref, why = _reference_lib()
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    threads = os.cpu_count() or 1
    if wl.name == "mlp_front":
        rc = _RefMlpFront(ref, wl, threads)
    else:
        # the workload's full step (every call at its own M), on the GPU arm's data
        rc = _RefCalls(ref, wl, wl.ref_calls(), threads)
    for _ in range(args.warmup):
        rc.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        rc.step()
    dt = time.perf_counter() - t0
    value = wl.value(rc.amount(wl) * args.steps, dt)
    rc.free()
    # the same workload description as the GPU arm's line (world as launched)
    cfg = wl.config(world)
    line = {"metric": wl.metric, "value": round(value, 4), "unit": wl.unit, "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak" if wl.name == "mlp_front" else "strong", "vs_baseline": None,
            "dtype": "u8xs8->s32 (VPDPBUSD), f32 rescale",
            "data": DATA if wl.name != "mlp_front" else "synthetic (random MatMulNBits codes; N(0,1) rows)",
            "config": cfg,
            "cpu_baseline": {"value": round(value, 4), "unit": wl.unit, "cores": threads, "kind": "reference",
                             "sample": f"{args.steps} full steps after {args.warmup} warm-ups, rank 0 only; "
                                       f"host: {_host_desc(threads)}"},
            "e2e": {"value": round(value, 4), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ncu_case(K, N, bits, M, launches=4):
    """One layer (N(0, 0.02) weights, RTN-packed; INT8 per channel), activations
    quantized once (two-pass), then `launches` matmul-kernel launches (the decode
    kernel up to 64 tokens, the tensor-core GEMM above) rotating over enough
    weight copies that each launch streams its weights from HBM."""
    import torch
    from breeze_engine_b200 import _lib as L
    lib = L.load()
    torch.cuda.set_device(0)
    copies = int(max(1, min(4, -(-2 * L2_BYTES // (N * K * bits // 8)))))
    layer = Layer(lib, K, N, bits, 1, 0, 1234, copies)
    a = torch.randn((M, K), device="cuda", dtype=torch.float32)
    n = lib.ql_act_workspace_bytes(M, K)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    c = torch.empty((M, N), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.ql_quantize_act_dev(a.data_ptr(), M, K, 1, ws.data_ptr(), n, s) == 0
    full = lib.ql_workspace_bytes(ctypes.c_void_p(layer.handles[0]), M)
    if M > 64 and full > n:
        # INT4 prefill: full calls prepare one FP16-operand workspace per copy,
        # then the GEMM kernel alone (ql_prefill_gemm_dev) runs `launches` times
        prep = []
        for h in layer.handles:
            w = torch.empty(full, dtype=torch.uint8, device="cuda")
            assert lib.ql_matmul_dev_ws(ctypes.c_void_p(h), a.data_ptr(), M, c.data_ptr(), w.data_ptr(), full, s) == 0
            prep.append((h, w))
        for i in range(launches):
            h, w = prep[i % len(prep)]
            assert lib.ql_prefill_gemm_dev(ctypes.c_void_p(h), w.data_ptr(), full, M, 1, c.data_ptr(), s) == 0
    else:
        for i in range(launches):
            h = layer.handles[i % len(layer.handles)]
            assert lib.ql_matmul_quantized_dev(ctypes.c_void_p(h), ws.data_ptr(), M, 1, c.data_ptr(), s) == 0
    torch.cuda.synchronize()
    layer.free()
    print(json.dumps({"ncu_case": [K, N, bits, M], "launches": launches, "copies": copies,
                      "alg_bytes_per_launch": decode_kernel_bytes(M, K, N, bits),
                      "alg_ops_per_launch": prefill_ops(M, K, N)}))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="decode")
    ap.add_argument("--exchange", choices=["nccl", "peer"], default="peer",
                    help="column-parallel output exchange at N > 1: NCCL all-gather, or the one-shot "
                         "peer-memory all-gather of this library (ql_peer_allgather_cols_dev)")
    ap.add_argument("--no-overlap", action="store_true",
                    help="at N > 1, run each call's collective after it on the same stream instead of "
                         "overlapping it with the next (independent) call")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="decode workload: skip the configs[2] / configs[3] measurements in `secondary`")
    ap.add_argument("--ncu-case", metavar="K,N,BITS,M", default=None,
                    help="profiling driver: pack one layer, quantize once, run the matmul kernel "
                         "4 times and exit (for ncu captures of a single launch)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.ncu_case:
        run_ncu_case(*map(int, args.ncu_case.split(",")))
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "mlp_front":
        run_mlp_front(args)
    else:
        run_ours(args)
    return 0


if __name__ == "__main__":
    sys.exit(main())
