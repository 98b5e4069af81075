"""Golden-vector cases for the quantized-linear hot path.

Each case builds MatMulNBits inputs and FP32 activations deterministically.
``make_golden.py`` runs the compiled reference (``kernel/quantized_matmul.cpp``
via ``oracle/_ref``) on them and stores its outputs in ``golden.npz``; the
tests rebuild the inputs, check them against the stored SHA-256, and compare
the oracle and the CUDA library with the stored reference outputs.

Input recipes follow the reference's own tests:
  * ``pack_*``    -- ``tests/test_cpu_packing.py:33-96`` (fixture_weights:
    seed N+K+bits, edge bytes [0,1,7,15,127,128,254,255], uniform scales,
    explicit or default zero points; activations default_rng(5), rows 1 and 9,
    both activation modes).
  * ``width_*``   -- ``tests/test_qwen35_cpu.py:196-208`` (27B projection widths,
    default_rng(3), M=3, two-pass mode).
  * ``subnormal`` -- ``tests/test_cpu_packing.py:114-131`` (fp16 subnormal and
    signed-zero scales).
  * ``edge``      -- activations with zero, subnormal, huge, NaN/inf and
    outlier blocks (quantizer corner cases).
  * ``rtn_*``     -- this package's RTN packer on N(0, 0.02) weights with the
    BASELINE distributions (N(0,1) activations, 1% of channels x20), small sizes.

``norm_cases()`` are the RMSNorm prologue's inputs (rows x, weights w, eps);
``make_golden.py`` stores the reference decoder's own rmsnorm of each
(``kernel/qwen35_decoder.cpp:133-141``) in ``golden_norm.npz``.
"""
import hashlib

import numpy as np

EDGE_BYTES = [0, 1, 7, 15, 127, 128, 254, 255]


def fixture_weights(N, K, bits, dtype, explicit_zeros):
    rng = np.random.default_rng(N + K + bits)
    blocks = K // 32
    qw = rng.integers(0, 256, (N, blocks, 4 * bits), dtype=np.uint8)
    qw.reshape(-1)[:8] = EDGE_BYTES
    scales = rng.uniform(0.0001, 0.02, (N, blocks)).astype(dtype)
    zeros = None
    if explicit_zeros:
        zeros = (rng.integers(0, 256, (N, (blocks + 1) // 2), dtype=np.uint8)
                 if bits == 4 else np.full((N, blocks), 128, np.uint8))
    return qw, scales, zeros


def _pack_case(N, K, bits, dtype, zeros):
    qw, sc, qz = fixture_weights(N, K, bits, dtype, zeros)
    rng = np.random.default_rng(5)
    acts = []
    for hp in (False, True):
        for rows in (1, 9):
            acts.append((hp, rng.normal(size=(rows, K)).astype(np.float32)))
    return dict(N=N, K=K, bits=bits, qweight=qw, scales=sc, qzeros=qz, acts=acts)


def _width_case(K, N, bits):
    rng = np.random.default_rng(3)
    qw = rng.integers(0, 256, (N, K // 32, 32 * bits // 8), dtype=np.uint8)
    sc = rng.uniform(0.001, 0.005, (N, K // 32)).astype(np.float32)
    a = rng.normal(size=(3, K)).astype(np.float32)
    return dict(N=N, K=K, bits=bits, qweight=qw, scales=sc, qzeros=None,
                acts=[(True, a), (False, a)])


def _subnormal_case():
    qw, _, _ = fixture_weights(16, 32, 4, np.float16, False)
    sc = np.array([0, 0x8000, 1, 0x8001, 0x03FF, 0x0400, 0x3C00, 0x7BFF] * 2,
                  dtype=np.uint16).view(np.float16).reshape(16, 1)
    rng = np.random.default_rng(5)
    acts = [(hp, rng.normal(size=(rows, 32)).astype(np.float32)) for hp in (False, True) for rows in (1, 9)]
    return dict(N=16, K=32, bits=4, qweight=qw, scales=sc, qzeros=None, acts=acts)


def edge_activations(M, K, seed):
    rng = np.random.default_rng(seed)
    a = rng.normal(size=(M, K)).astype(np.float32)
    a[0, 0:32] = 0.0                                            # zero block: scale 0
    a[0, 32:64] = np.float32(1e-40)                             # subnormal block: inv = inf
    a[0, 64:96] = np.float32(3e38)                              # huge block
    a[0, 96:128] = np.float32(1e-36) * np.arange(32, dtype=np.float32)   # tiny ramp
    if M > 1:
        a[1, 5] = np.nan
        a[1, 40] = np.inf
        a[1, 70] = -np.inf
    if M > 2:
        a[2, 128:160] = -7.25                                   # constant block (all +-32767)
        a[2, 160:192] = np.float32(2.0) ** -126                 # smallest normal
    a[:, -1] *= 20.0                                            # outlier channel
    return a


def _edge_case(bits, zeros, dtype):
    N, K = 32, 256
    qw, sc, qz = fixture_weights(N, K, bits, dtype, zeros)
    a = edge_activations(5, K, 11)
    return dict(N=N, K=K, bits=bits, qweight=qw, scales=sc, qzeros=qz, acts=[(True, a), (False, a)])


def outlier_activations(M, K, seed, frac=0.01, factor=20.0):
    """N(0,1) activations with ``frac`` of the channels scaled by ``factor``."""
    rng = np.random.default_rng(seed)
    a = rng.normal(size=(M, K)).astype(np.float32)
    n_out = max(1, int(round(frac * K)))
    cols = rng.choice(K, size=n_out, replace=False)
    a[:, cols] *= np.float32(factor)
    return a


def _rtn_case(N, K, bits, M, symmetric, per_channel, outliers, seed):
    from breeze_engine_b200.quant import quantize_matmul_nbits
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, size=(K, N)).astype(np.float32)
    qw, sc, qz = quantize_matmul_nbits(w, bits=bits, symmetric=symmetric, per_channel=per_channel)
    a = outlier_activations(M, K, seed + 1) if outliers else \
        np.random.default_rng(seed + 1).normal(size=(M, K)).astype(np.float32)
    return dict(N=N, K=K, bits=bits, qweight=qw, scales=sc, qzeros=qz, acts=[(True, a)])


def all_cases():
    cases = {}
    for (N, K) in [(16, 32), (48, 96), (64, 512)]:
        for bits in (4, 8):
            for dtype in (np.float16, np.float32):
                for zeros in (False, True):
                    name = f"pack_{N}x{K}_b{bits}_{np.dtype(dtype).name}_{'zp' if zeros else 'nozp'}"
                    cases[name] = lambda N=N, K=K, bits=bits, dtype=dtype, zeros=zeros: \
                        _pack_case(N, K, bits, dtype, zeros)
    for (K, N, bits) in [(5120, 48, 8), (17408, 16, 4), (6144, 64, 8), (4096, 32, 4)]:
        cases[f"width_{K}x{N}_b{bits}"] = lambda K=K, N=N, bits=bits: _width_case(K, N, bits)
    cases["subnormal"] = _subnormal_case
    cases["edge_b4_zp"] = lambda: _edge_case(4, True, np.float16)
    cases["edge_b4_nozp"] = lambda: _edge_case(4, False, np.float32)
    cases["edge_b8"] = lambda: _edge_case(8, False, np.float16)
    cases["rtn_b4_m1"] = lambda: _rtn_case(64, 4096, 4, 1, True, False, False, 101)
    cases["rtn_b4_outliers"] = lambda: _rtn_case(32, 512, 4, 17, True, False, True, 103)
    cases["rtn_b4_asym"] = lambda: _rtn_case(48, 1024, 4, 5, False, False, True, 105)
    cases["rtn_b8_perchannel"] = lambda: _rtn_case(48, 1024, 8, 16, True, True, False, 107)
    return cases


def input_digest(case):
    h = hashlib.sha256()
    for key in ("qweight", "scales", "qzeros"):
        v = case[key]
        h.update(b"-" if v is None else np.ascontiguousarray(v).tobytes())
    for hp, a in case["acts"]:
        h.update(bytes([hp]))
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


# ------------------------------------------------------------------ RMSNorm prologue
def tie_rows(pairs=((3, 38), (4, 45), (5, 30), (6, 37), (7, 2), (10, 3), (2, 1), (1, 2)),
             exps=(0, -3, 5), K=64):
    """Rows whose reference mean of squares is decided by the serial order.

    x0 = 1 + a*2^-12 and x1 = b*2^-12 with a^2 + b^2 odd have squares summing
    exactly to B = 1 + a*2^-11 + (a^2 + b^2)*2^-24, and B / K (K = 64) lies
    exactly half way between two floats.  The other 62 entries are 2^-28,
    whose squares (2^-56) each fall below half an ulp of the running double
    sum and are dropped by the reference's serial loop, so its mean is the tie
    (rounded to even); any order that adds the small squares first gets a sum
    above the tie and the next float up.  For the first four pairs that one
    ulp of the mean also changes 1/sqrt(mean + 0), so hn differs.  Scaling a
    row by 2^e keeps all of this (squares scale by 4^e).
    """
    rows = []
    for e in exps:
        for a, b in pairs:
            r = np.full(K, np.float32(2.0 ** -28), np.float32)
            r[0] = np.float32(1.0 + a * 2.0 ** -12)
            r[1] = np.float32(b * 2.0 ** -12)
            rows.append(r * np.float32(2.0 ** e))
    return np.stack(rows)


def norm_cases():
    cases = {}
    rng = np.random.default_rng(21)
    x = (rng.normal(size=(6, 64)) * rng.uniform(0.01, 30.0, (6, 1))).astype(np.float32)
    cases["rand_k64"] = (x, rng.uniform(0.5, 2.0, 64).astype(np.float32), 1e-6)
    # Qwen3.5-27B hidden width, zero-centred norm weights near 1, outlier channels.
    w = (1.0 + 0.1 * np.random.default_rng(22).normal(size=5120)).astype(np.float32)
    cases["qwen_k5120"] = (outlier_activations(5, 5120, 23), w, 1e-6)
    cases["ties"] = (tie_rows(), np.ones(64, np.float32), 0.0)
    e = np.random.default_rng(24).normal(size=(6, 96)).astype(np.float32)
    e[0] = 0.0                                   # zero row: inv = 1/sqrt(eps)
    e[1, 7] = np.nan                             # NaN row
    e[2, 3] = np.inf                             # inf row: inv = 0
    e[3] = np.float32(1e-40)                     # subnormal row
    e[4] = np.float32(3e38)                      # huge row (squares ~1e77 in double)
    e[5, ::2] = -e[5, ::2]
    cases["edge_k96"] = (e, np.random.default_rng(25).uniform(-2, 2, 96).astype(np.float32), 1e-6)
    z = np.zeros((2, 32), np.float32)
    z[1, 0] = 1.0
    cases["zero_eps0_k32"] = (z, np.ones(32, np.float32), 0.0)   # 0 * inf = NaN in row 0
    return cases


def norm_digest(x, w, eps):
    h = hashlib.sha256()
    for v in (x, w, np.float32(eps)):
        h.update(np.ascontiguousarray(v).tobytes())
    return h.hexdigest()


def _neighbours(values, radius):
    """Every float within `radius` ulps of each value (by bit pattern)."""
    out = []
    for v in values:
        u = int(np.array([v], np.float32).view(np.uint32)[0])
        out.append(np.arange(u - radius, u + radius + 1, dtype=np.int64).astype(np.uint32).view(np.float32))
    return np.concatenate(out)


def silu_cases():
    """(gate, up) pairs for the SiLU * up prologue of the down projection
    (the reference decoder's ``g1 = siluf(g1) * g2``,
    ``kernel/qwen35_decoder.cpp:129, 408``): MLP-like values, the whole range of
    the exponential, and its edges -- overflow and underflow thresholds, the
    two inputs near float rounding midpoints where the C library's expf and a
    plain (unfused) evaluation of its method differ (32.5646324 and
    -63.0994606, reached as -g) with their neighbours, zeros, subnormals,
    infinities and NaN.  Every case is [M, K] with K % 32 == 0."""
    cases = {}
    rng = np.random.default_rng(31)
    cases["mlp_k4096"] = ((rng.normal(size=(8, 4096)) * 2.0).astype(np.float32),
                          (rng.normal(size=(8, 4096)) * 2.0).astype(np.float32))
    g = rng.uniform(-110.0, 110.0, size=(4, 2048)).astype(np.float32)
    cases["range_k2048"] = (g, rng.normal(size=(4, 2048)).astype(np.float32))
    special = np.array([-32.564632415771484, 63.09946060180664, 32.564632415771484, -63.09946060180664,
                        -88.72283935546875, -88.72284698486328, 88.0, -88.0, 103.97207641601562,
                        103.97208404541016, 87.3365478515625, -87.3365478515625, 0.0, -0.0, 1e-40, -1e-40,
                        np.inf, -np.inf, np.nan, 3e38, -3e38, 1e-30, -1e-30, 0.5, -0.5, 20.0, -20.0],
                       np.float32)
    edge = np.concatenate([special, _neighbours(special[:4], 200), _neighbours(special[4:12], 20)])
    k = ((edge.size + 31) // 32) * 32
    e = np.zeros(k, np.float32)
    e[: edge.size] = edge
    u = np.random.default_rng(32).normal(size=k).astype(np.float32)
    u[:32] = 1.0
    cases["edges"] = (e.reshape(1, k), u.reshape(1, k))
    return cases


def silu_digest(g, u):
    h = hashlib.sha256()
    for v in (g, u):
        h.update(np.ascontiguousarray(v).tobytes())
    return h.hexdigest()
