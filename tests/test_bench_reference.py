"""The reference arm of bench.py on the host (no GPU needed).

``bench.py --impl reference`` times the reference's own i4_matmul (built from
kernel/quantized_matmul.cpp into oracle/_ref) on the same workload as the GPU
arm and prints one JSON line.  The driver compares the two lines, so the
reference line must carry the GPU arm's metric, unit and config, say that it
is the reference, and describe its CPU run (cpu_baseline) and an e2e object
with no device copies.  Skipped where the reference build is absent.
"""
import json
import os
import subprocess
import sys

import pytest

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libbreeze_ref.so")


@pytest.mark.slow
@pytest.mark.skipif(not os.path.exists(REF_SO), reason="oracle/_ref/libbreeze_ref.so not built")
def test_reference_line_matches_the_gpu_arm():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    # the 27B-class layer set at one token: the smallest workload to build on the host; the
    # line's keys are the same for every workload
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                          "layer_m1", "--steps", "1", "--warmup", "1"], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=900)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    wl = bench.WORKLOADS["layer_m1"]()
    assert line["impl"] == "reference"
    assert line["metric"] == wl.metric and line["unit"] == wl.unit
    assert line["config"] == json.loads(json.dumps(wl.config(1)))          # as the GPU arm prints it
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["steps"] == 1 and line["warmup"] >= 3
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "reference" and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
