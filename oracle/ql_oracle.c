/*
 * ql_oracle.c -- CPU restatement of Breeze's quantized-linear hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in breeze_engine_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference leg may load it, and only as
 * the checker or the timed CPU baseline, never as a product code path.
 *
 * It restates the reference algorithm of kernel/quantized_matmul.cpp in
 * plain scalar C, working directly on the ONNX MatMulNBits layout (no VNNI
 * prepack), and is pinned against the compiled reference itself
 * (oracle/_ref, built by oracle/Makefile) and against the committed golden
 * fixtures in tests/golden.
 *
 * Semantics restated (reference file:line):
 *   - quantize_A_i16            kernel/quantized_matmul.cpp:237-258
 *       per (m, 32-block): amax = max|a| (NaN never wins the compare),
 *       scale = amax / 32767.f, inv = scale > 0 ? 1/scale : 0,
 *       q = clamp((int)lrint(a*inv), -32767, 32767), u = q + 32768,
 *       hi = u >> 8, lo = u & 255.
 *   - weight decode             breeze/quant.py:38-58 (INT4), :28-36 (INT8),
 *                               kernel/quantized_matmul.cpp:161-191
 *       INT4: low nibble = even k, zp from packed qzeros (low nibble = even
 *       block) or 8.  INT8: zp is 128.
 *   - per-block INT32 sum       kernel/quantized_matmul.cpp:298-312,262-268
 *       cs[m,n,b] = 256*(acc_hi - corr) + acc_lo == sum_k q16 * (w - zp).
 *   - FP32 rescale chain        kernel/quantized_matmul.cpp:311-315
 *       acc = 0; for b in order: f = (float)cs * bscale[n,b];
 *       acc = fmaf(ascale[m,b], f, acc).
 *   - INT8 single-pass mode     kernel/quantized_matmul.cpp:215-232,266-267
 *       (secondary; hi_prec = 0): q = clamp(lrint(a*inv), +-127),
 *       scale = amax / 127.f, cs = sum q8 * (w - zp).
 *   - RMSNorm prologue          kernel/qwen35_decoder.cpp:133-141
 *       ss = serial double sum of (double)x*x in j order,
 *       inv = 1.f / sqrtf((float)(ss / K) + eps), o = (x * inv) * w.
 *
 * Must be compiled with -ffp-contract=off and without -ffast-math so every
 * float operation rounds exactly once, as in the reference.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

/* (int)lrintf(x) as the reference evaluates it on x86-64: lrintf returns a
 * 64-bit long; NaN, +-inf and |x| >= 2^63 give LONG_MIN, whose low 32 bits
 * are 0.  For |x| < 2^63 the cast keeps the low 32 bits of the rounded
 * value.  The quantizer only reaches |x| >= 2^31 through inv == inf, so
 * the explicit form below is exact for every float input. */
static int lrint_low32(float x) {
    if (!(fabsf(x) < 9.2233720368547758e18f)) return 0;
    long long r = llrintf(x);
    return (int)(uint32_t)(uint64_t)r;
}

/* quantize_A_i16 restated.  A: [M,K] row-major fp32.  Outputs hi/lo planes
 * [M,K] u8 and ascale [M,K/32] fp32. */
void ql_oracle_quantize_i16(const float* A, int M, int K,
                            uint8_t* hi, uint8_t* lo, float* ascale) {
    const int nblk = K / 32;
    for (int m = 0; m < M; ++m) {
        for (int b = 0; b < nblk; ++b) {
            const float* a = A + (size_t)m * K + (size_t)b * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) {
                float v = fabsf(a[i]);
                if (v > amax) amax = v;
            }
            float scale = amax / 32767.0f;
            float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
            ascale[(size_t)m * nblk + b] = scale;
            for (int i = 0; i < 32; ++i) {
                int q = lrint_low32(a[i] * inv);
                q = q > 32767 ? 32767 : (q < -32767 ? -32767 : q);
                unsigned u = (unsigned)(q + 32768);
                hi[(size_t)m * K + (size_t)b * 32 + i] = (uint8_t)(u >> 8);
                lo[(size_t)m * K + (size_t)b * 32 + i] = (uint8_t)(u & 0xFF);
            }
        }
    }
}

/* quantize_A (INT8 single pass) restated.  q8 is written as the signed
 * value (the reference stores q + 128 as u8). */
void ql_oracle_quantize_i8(const float* A, int M, int K, int8_t* q8, float* ascale) {
    const int nblk = K / 32;
    for (int m = 0; m < M; ++m) {
        for (int b = 0; b < nblk; ++b) {
            const float* a = A + (size_t)m * K + (size_t)b * 32;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) {
                float v = fabsf(a[i]);
                if (v > amax) amax = v;
            }
            float scale = amax / 127.0f;
            float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
            ascale[(size_t)m * nblk + b] = scale;
            for (int i = 0; i < 32; ++i) {
                int q = lrint_low32(a[i] * inv);
                q = q > 127 ? 127 : (q < -127 ? -127 : q);
                q8[(size_t)m * K + (size_t)b * 32 + i] = (int8_t)q;
            }
        }
    }
}

/* Signed weight value w - zp for row n, input index k (MatMulNBits layout). */
static inline int weight_at(const uint8_t* qw, const uint8_t* qzeros, int K, int bits,
                            int n, int k) {
    const int nblk = K / 32, b = k / 32, j = k % 32;
    if (bits == 8) {
        return (int)qw[((size_t)n * nblk + b) * 32 + j] - 128;
    }
    const uint8_t byte = qw[((size_t)n * nblk + b) * 16 + j / 2];
    const int q = (j & 1) ? (byte >> 4) : (byte & 15);
    int zp = 8;
    if (qzeros) {
        const uint8_t z = qzeros[(size_t)n * ((nblk + 1) / 2) + b / 2];
        zp = (b & 1) ? (z >> 4) : (z & 15);
    }
    return q - zp;
}

/* Per-block INT32 accumulators from the hi/lo planes:
 * cs[m, n, b] = sum_k (256*(hi-128) + lo) * (w - zp).  Output [M, N, nblk]. */
void ql_oracle_block_sums(const uint8_t* qw, const uint8_t* qzeros, int N, int K, int bits,
                          const uint8_t* hi, const uint8_t* lo, int M, int32_t* cs) {
    const int nblk = K / 32;
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n)
            for (int b = 0; b < nblk; ++b) {
                int32_t s = 0;
                for (int j = 0; j < 32; ++j) {
                    const int k = b * 32 + j;
                    const int q16 = 256 * ((int)hi[(size_t)m * K + k] - 128) + (int)lo[(size_t)m * K + k];
                    s += q16 * weight_at(qw, qzeros, K, bits, n, k);
                }
                cs[((size_t)m * N + n) * nblk + b] = s;
            }
}

/* FP32 rescale chain over precomputed block sums.  bscale: [N, nblk] fp32. */
void ql_oracle_rescale(const int32_t* cs, const float* ascale, const float* bscale,
                       int M, int N, int K, float* C) {
    const int nblk = K / 32;
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int b = 0; b < nblk; ++b) {
                const float f = (float)cs[((size_t)m * N + n) * nblk + b] * bscale[(size_t)n * nblk + b];
                acc = fmaf(ascale[(size_t)m * nblk + b], f, acc);
            }
            C[(size_t)m * N + n] = acc;
        }
}

/* Whole hot path (two-pass INT16 mode): C[M,N] = i4_matmul(A).  Streams one
 * output at a time so it needs no [M,N,nblk] scratch.  hi/lo/ascale are
 * caller-provided scratch of sizes M*K, M*K and M*(K/32). */
void ql_oracle_matmul(const uint8_t* qw, const float* bscale, const uint8_t* qzeros,
                      int N, int K, int bits, const float* A, int M, float* C,
                      uint8_t* hi, uint8_t* lo, float* ascale) {
    const int nblk = K / 32;
    ql_oracle_quantize_i16(A, M, K, hi, lo, ascale);
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int b = 0; b < nblk; ++b) {
                int32_t s = 0;
                for (int j = 0; j < 32; ++j) {
                    const int k = b * 32 + j;
                    const int q16 = 256 * ((int)hi[(size_t)m * K + k] - 128) + (int)lo[(size_t)m * K + k];
                    s += q16 * weight_at(qw, qzeros, K, bits, n, k);
                }
                const float f = (float)s * bscale[(size_t)n * nblk + b];
                acc = fmaf(ascale[(size_t)m * nblk + b], f, acc);
            }
            C[(size_t)m * N + n] = acc;
        }
}

/* INT8 single-pass mode (hi_prec off) restated. */
void ql_oracle_matmul_i8(const uint8_t* qw, const float* bscale, const uint8_t* qzeros,
                         int N, int K, int bits, const float* A, int M, float* C,
                         int8_t* q8, float* ascale) {
    const int nblk = K / 32;
    ql_oracle_quantize_i8(A, M, K, q8, ascale);
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int b = 0; b < nblk; ++b) {
                int32_t s = 0;
                for (int j = 0; j < 32; ++j) {
                    const int k = b * 32 + j;
                    s += (int)q8[(size_t)m * K + k] * weight_at(qw, qzeros, K, bits, n, k);
                }
                const float f = (float)s * bscale[(size_t)n * nblk + b];
                acc = fmaf(ascale[(size_t)m * nblk + b], f, acc);
            }
            C[(size_t)m * N + n] = acc;
        }
}

/* The reference decoder's rmsnorm (kernel/qwen35_decoder.cpp:133-141): the
 * sum of squares in double, serially in j order (each (double)x*x is exact,
 * so contracting it into an fma, as -march builds of the reference may do,
 * rounds identically), then fp32 for the rest. */
void ql_oracle_rmsnorm(const float* X, const float* W, int M, int K, float eps, float* out) {
    for (int m = 0; m < M; ++m) {
        const float* x = X + (size_t)m * K;
        float* o = out + (size_t)m * K;
        double ss = 0.0;
        for (int j = 0; j < K; ++j) ss += (double)x[j] * (double)x[j];
        const float inv = 1.0f / sqrtf((float)(ss / K) + eps);
        for (int j = 0; j < K; ++j) o[j] = (x[j] * inv) * W[j];
    }
}
