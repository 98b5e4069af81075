"""Generate ``tests/golden/golden.npz`` from the compiled reference.

Runs the reference's own ``i4_prepack_onnx`` / ``i4_matmul`` (built from
``kernel/quantized_matmul.cpp`` by ``oracle/Makefile`` into ``oracle/_ref``)
and its internal quantizer / per-block INT32 accumulators (``oracle/ref_probe.cpp``)
on every case of ``cases.py``, and stores:

  ``<case>/digest``            SHA-256 of the regenerated inputs
  ``<case>/C<i>``              reference FP32 output for activation set i
  ``<case>/cs<i>``             reference per-block INT32 accumulators (two-pass
                               sets with a small M*N*nblk only)
  ``<case>/hi<i>``, ``lo<i>``, ``as<i>``  reference quantizer planes (same subset)

It also runs the reference decoder's own ``rmsnorm``
(``kernel/qwen35_decoder.cpp:133-141``, exported by ``oracle/ref_norm_probe.cpp``)
on ``cases.norm_cases()`` and stores ``<case>/digest`` and ``<case>/hn`` in
``golden_norm.npz``, and its ``siluf(g) * u`` (``kernel/qwen35_decoder.cpp:129,
408``, the same probe file) on ``cases.silu_cases()``, storing ``<case>/digest``
and ``<case>/y`` in ``golden_silu.npz``.

Run from the repository root where the reference checkout exists:
``python tests/golden/make_golden.py [--norm-only]`` (``--norm-only`` writes the
norm and SiLU fixtures only).
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from cases import all_cases, input_digest, norm_cases, norm_digest, silu_cases, silu_digest  # noqa: E402
from oracle.oracle import Reference, build  # noqa: E402

CS_LIMIT = 10_000    # store INT32 accumulators when M*N*nblk is at most this


def make_norm(ref):
    out = {}
    for name, (x, w, eps) in norm_cases().items():
        out[f"{name}/digest"] = np.frombuffer(bytes.fromhex(norm_digest(x, w, eps)), np.uint8)
        out[f"{name}/hn"] = ref.rmsnorm(x, w, eps)
        print(f"norm {name}: {x.shape}")
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_norm.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def make_silu(ref):
    out = {}
    for name, (g, u) in silu_cases().items():
        out[f"{name}/digest"] = np.frombuffer(bytes.fromhex(silu_digest(g, u)), np.uint8)
        out[f"{name}/y"] = ref.silu_mul(g, u)
        print(f"silu {name}: {g.shape}")
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_silu.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def main():
    build()
    ref = Reference()
    make_norm(ref)
    make_silu(ref)
    if "--norm-only" in sys.argv[1:]:
        return
    out = {}
    for name, make in all_cases().items():
        case = make()
        out[f"{name}/digest"] = np.frombuffer(bytes.fromhex(input_digest(case)), np.uint8)
        h = ref.prepack(case["qweight"], case["scales"], case["qzeros"], case["K"], case["N"], case["bits"])
        try:
            for i, (hp, a) in enumerate(case["acts"]):
                c = ref.matmul(h, a, case["N"], hi_prec=hp, threads=2)
                out[f"{name}/C{i}"] = c
                if hp and a.shape[0] * case["N"] * (case["K"] // 32) <= CS_LIMIT:
                    hi, lo, asc = ref.quantize_i16(a)
                    cs = ref.block_sums(h, hi, lo, case["N"], case["K"])
                    replay = ref.replay(h, cs, asc, case["N"])
                    assert np.array_equal(replay.view(np.uint32), c.view(np.uint32)), name
                    out[f"{name}/cs{i}"] = cs
                    out[f"{name}/hi{i}"] = hi
                    out[f"{name}/lo{i}"] = lo
                    out[f"{name}/as{i}"] = asc
        finally:
            ref.free(h)
        print(f"{name}: {len(case['acts'])} activation sets")
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
