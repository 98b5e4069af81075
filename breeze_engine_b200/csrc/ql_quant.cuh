// ql_quant.cuh -- per-(token, block) pieces of the activation quantizer shared
// by ql_quant.cu (the quantizer kernels) and ql_norm.cu (the fused RMSNorm +
// quantizer of the decode layout).  Arithmetic: the reference quantize_A_i16
// (kernel/quantized_matmul.cpp:237-258) and quantize_A (:215-232), as stated
// at the top of ql_quant.cu.
#pragma once
#include "ql_common.cuh"
#include "ql_internal.h"

namespace ql {

__device__ __forceinline__ int to_int_like_lrint(float x) {
    const float ax = fabsf(x);
    if (ax < 2147483648.0f) return __float2int_rn(x);
    if (ax < 9.2233720368547758e18f) return static_cast<int>(static_cast<uint32_t>(
                                                static_cast<unsigned long long>(__float2ll_rn(x))));
    return 0;   // NaN, +-inf, |x| >= 2^63
}

// The 32 values of (token m, block b): row m of A itself or, with the RMSNorm
// prologue (NORM), a = (x * row_inv[m]) * w[k] as the reference decoder's
// rmsnorm writes them (kernel/qwen35_decoder.cpp:139: x * inv * w, evaluated
// left to right, each product rounded to fp32), stored to hn when it is set.
// Row m's 32 values of block b.
__device__ __forceinline__ void load_raw_block(const float* __restrict__ A, int lda, int m, int b, float (&v)[32]) {
    const float4* src = reinterpret_cast<const float4*>(A + static_cast<size_t>(m) * lda + b * BLOCK_K);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = __ldg(src + i);
        v[4 * i + 0] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
}

// The RMSNorm prologue on one block: a = (x * r) * w[k] as the reference
// decoder's rmsnorm writes it (kernel/qwen35_decoder.cpp:139: x * inv * w,
// evaluated left to right, each product rounded to fp32), stored to hn when set.
__device__ __forceinline__ void norm_block(float (&v)[32], float r, const NormArgs& nrm, int m, int b) {
    const float4* w4 = reinterpret_cast<const float4*>(nrm.w + b * BLOCK_K);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 g = __ldg(w4 + i);
        v[4 * i + 0] = __fmul_rn(__fmul_rn(v[4 * i + 0], r), g.x);
        v[4 * i + 1] = __fmul_rn(__fmul_rn(v[4 * i + 1], r), g.y);
        v[4 * i + 2] = __fmul_rn(__fmul_rn(v[4 * i + 2], r), g.z);
        v[4 * i + 3] = __fmul_rn(__fmul_rn(v[4 * i + 3], r), g.w);
    }
    if (nrm.hn) {
        float4* dst = reinterpret_cast<float4*>(nrm.hn + static_cast<size_t>(m) * nrm.ldh + b * BLOCK_K);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
}

// ---------------------------------------------------------------- SiLU * up prologue
// The reference decoder's MLP input of the down projection is
//     g1 = siluf(g1) * g2,  siluf(x) = x / (1.0f + expf(-x))
// (kernel/qwen35_decoder.cpp:129, :408), with the host C library's expf.  That
// expf is not correctly rounded; it is the published table-driven method in
// double precision (k = round(x * 32/ln2) by adding and subtracting 1.5*2^52,
// 2^(k/32) from a 32-entry table, a degree-3 polynomial in the reduced
// argument, one rounding to float), built with fused multiply-adds on x86-64
// CPUs with FMA.  expf_host_method() evaluates the same method with the same
// fusions and roundings in explicit double operations, so it returns the
// library's bits: oracle/expf_ref.c restates it on the host, and its checker
// finds zero differences from the library over all 2^32 inputs.  The table
// entries are the correctly rounded doubles of 2^(i/32), minus i << 47.
static __device__ __constant__ unsigned long long EXP2_32_TAB[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

__device__ __forceinline__ float expf_host_method(float x) {
    const double invln2_32 = 0x1.71547652b82fep+0 * 32;     // 32 / ln 2
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;  // the method's minimax coefficients,
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;       // for the reduced argument in 1/32 units
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32;
    const uint32_t ux = __float_as_uint(x);
    const uint32_t top = (ux >> 20) & 0x7ffu;
    if (top >= ((0x42B00000u >> 20) & 0x7ffu)) {            // |x| >= 88 (0x42B00000 = 88.0f), NaN, inf
        if (ux == 0xFF800000u) return 0.0f;                 // -inf
        if (top >= 0x7f8u) return __fadd_rn(x, x);          // NaN, +inf
        if (x > 0x1.62e42ep6f) return __uint_as_float(0x7F800000u);   // above log(2^128): +inf
        if (x < -0x1.9fe368p6f) return 0.0f;                           // below log(2^-150)
    }
    const double xd = static_cast<double>(x);
    double kd = __fma_rn(invln2_32, xd, shift);             // x*32/ln2 rounded to an integer (+ shift)
    const unsigned long long ki = static_cast<unsigned long long>(__double_as_longlong(kd));
    kd = __dsub_rn(kd, shift);
    const double r = __fma_rn(invln2_32, xd, -kd);          // reduced argument, unrounded product
    const unsigned long long t = EXP2_32_TAB[ki & 31] + (ki << 47);
    const double s = __longlong_as_double(static_cast<long long>(t));
    const double z = __fma_rn(c0, r, c1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(c2, r, 1.0);
    y = __fma_rn(z, r2, y);
    y = __dmul_rn(y, s);
    return __double2float_rn(y);
}

// silu(g) * u as the reference evaluates it: x / (1 + expf(-x)), then * u,
// every operation one rounding.
__device__ __forceinline__ float silu_mul_ref(float g, float u) {
    const float e = expf_host_method(-g);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), u);
}

// Activation prologues of the quantizers: 0 = A as it is, 1 = the RMSNorm
// (NormArgs row_inv and w), 2 = silu(A) * up (NormArgs up / ldu: the gate
// projection's output in A, the up projection's in `up`).  With a prologue the
// values quantized can also be written out (NormArgs hn / ldh).
enum : int { PRO_NONE = 0, PRO_NORM = 1, PRO_SILU = 2 };

__device__ __forceinline__ void silu_block(float (&v)[32], const NormArgs& nrm, int m, int b) {
    const float4* u4 = reinterpret_cast<const float4*>(nrm.up + static_cast<size_t>(m) * nrm.ldu + b * BLOCK_K);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 u = __ldg(u4 + i);
        v[4 * i + 0] = silu_mul_ref(v[4 * i + 0], u.x);
        v[4 * i + 1] = silu_mul_ref(v[4 * i + 1], u.y);
        v[4 * i + 2] = silu_mul_ref(v[4 * i + 2], u.z);
        v[4 * i + 3] = silu_mul_ref(v[4 * i + 3], u.w);
    }
    if (nrm.hn) {
        float4* dst = reinterpret_cast<float4*>(nrm.hn + static_cast<size_t>(m) * nrm.ldh + b * BLOCK_K);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
}

// The 32 values of (token m, block b): row m of A itself, or with a prologue
// (PRO) normalised by the precomputed factor row_inv[m] or as silu(A) * up.
template <int PRO>
__device__ __forceinline__ void load_block(const float* __restrict__ A, int lda, int m, int b,
                                           const NormArgs& nrm, float (&v)[32]) {
    load_raw_block(A, lda, m, b, v);
    if (PRO == PRO_NORM) norm_block(v, __ldg(nrm.row_inv + m), nrm, m, b);
    if (PRO == PRO_SILU) silu_block(v, nrm, m, b);
}

// Decode-layout record of (token m, block b): the four fragment slots of
// token m (lanes 4*(m%8) + t) and its activation scale.
template <bool HP>
__device__ __forceinline__ void act_zero_block(const ActView& out, int m, int b) {
    constexpr int LB = HP ? 16 : 8;                                   // bytes per lane
    uint8_t* rec = out.q + static_cast<size_t>(b) * out.QREC;
    uint8_t* frag = rec + m * 4 * LB;
    if (m < out.TPB) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            if (HP) *reinterpret_cast<uint4*>(frag + t * LB) = make_uint4(0, 0, 0, 0);
            else *reinterpret_cast<uint2*>(frag + t * LB) = make_uint2(0, 0);
        }
    }
    reinterpret_cast<float*>(rec + out.TPB * 4 * LB)[m] = 0.0f;
    reinterpret_cast<int32_t*>(rec + out.TPB * 4 * LB + out.TPBA * 4)[m] = 0;
}

template <bool HP>
__device__ __forceinline__ void act_store_block(const float (&v)[32], const ActView& out, int m, int b) {
    constexpr int LB = HP ? 16 : 8;                                   // bytes per lane
    uint8_t* rec = out.q + static_cast<size_t>(b) * out.QREC;
    uint8_t* frag = rec + m * 4 * LB;
    float* scales = reinterpret_cast<float*>(rec + out.TPB * 4 * LB);
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float a = fabsf(v[i]);
        amax = (a > amax) ? a : amax;
    }
    constexpr float QMAX = HP ? 32767.0f : 127.0f;
    constexpr int IMAX = HP ? 32767 : 127;
    const float scale = __fdiv_rn(amax, QMAX);
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    scales[m] = scale;

    uint32_t hw[8], lw[8];
    int qsum = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        uint32_t hword = 0, lword = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int q = to_int_like_lrint(__fmul_rn(v[4 * w + j], inv));
            q = q > IMAX ? IMAX : (q < -IMAX ? -IMAX : q);
            qsum += q;
            if (HP) {
                const uint32_t u = static_cast<uint32_t>(q + 32768);
                hword |= ((u >> 8) ^ 0x80u) << (8 * j);      // hi - 128 as a signed byte
                lword |= (u & 0xFFu) << (8 * j);
            } else {
                lword |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * j);   // q8 as a signed byte
            }
        }
        hw[w] = hword;
        lw[w] = lword;
    }
    reinterpret_cast<int32_t*>(rec + out.TPB * 4 * LB + out.TPBA * 4)[m] = qsum;
    // lane t: k 4t..4t+3 (word t) and 16+4t..16+4t+3 (word 4+t) of each plane
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        if (HP) *reinterpret_cast<uint4*>(frag + t * LB) = make_uint4(hw[t], hw[4 + t], lw[t], lw[4 + t]);
        else *reinterpret_cast<uint2*>(frag + t * LB) = make_uint2(lw[t], lw[4 + t]);
    }
}

// ---------------------------------------------------------------- 8 lanes per block
// The decode-layout quantizer with one (token, block) pair per 8 consecutive
// lanes: lane c of the group holds values 4c..4c+3 of the block.  The block's
// amax (a maximum: exact in any order, NaN never wins the compare) and its sum
// of quantized values (integers) are combined with xor-shuffles inside the
// group; scale, inverse and every value's rounding are the same operations as
// act_store_block, so the record is bit-identical -- at an eighth of the
// serial latency per block, which is what a decode call waits for.  Every lane
// of the warp must call these (shuffles), valid or not.

// The 4 values (token m, block b, lane c) of the block, with the prologue.
template <int PRO>
__device__ __forceinline__ float4 load_quad(const float* __restrict__ A, int lda, int m, int b, int c,
                                            const NormArgs& nrm) {
    float4 v = __ldg(reinterpret_cast<const float4*>(A + static_cast<size_t>(m) * lda + b * BLOCK_K) + c);
    if (PRO == PRO_NORM) {
        const float r = __ldg(nrm.row_inv + m);
        const float4 g = __ldg(reinterpret_cast<const float4*>(nrm.w + b * BLOCK_K) + c);
        v.x = __fmul_rn(__fmul_rn(v.x, r), g.x);
        v.y = __fmul_rn(__fmul_rn(v.y, r), g.y);
        v.z = __fmul_rn(__fmul_rn(v.z, r), g.z);
        v.w = __fmul_rn(__fmul_rn(v.w, r), g.w);
    }
    if (PRO == PRO_SILU) {
        const float4 u = __ldg(reinterpret_cast<const float4*>(nrm.up + static_cast<size_t>(m) * nrm.ldu + b * BLOCK_K) + c);
        v.x = silu_mul_ref(v.x, u.x);
        v.y = silu_mul_ref(v.y, u.y);
        v.z = silu_mul_ref(v.z, u.z);
        v.w = silu_mul_ref(v.w, u.w);
    }
    if (PRO != PRO_NONE && nrm.hn)
        reinterpret_cast<float4*>(nrm.hn + static_cast<size_t>(m) * nrm.ldh + b * BLOCK_K)[c] = v;
    return v;
}

// Quantizes the group's block into its record; `store` false: take part in
// the shuffles only.  Padded token rows pass zeros and get the zero record.
template <bool HP>
__device__ __forceinline__ void act_store_quad(float4 v, const ActView& out, int m, int b, int c, bool store) {
    constexpr int LB = HP ? 16 : 8;
    constexpr float QMAX = HP ? 32767.0f : 127.0f;
    constexpr int IMAX = HP ? 32767 : 127;
    const float vv[4] = {v.x, v.y, v.z, v.w};
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float a = fabsf(vv[j]);
        amax = (a > amax) ? a : amax;
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        const float a = __shfl_xor_sync(0xffffffffu, amax, o);
        amax = (a > amax) ? a : amax;
    }
    const float scale = __fdiv_rn(amax, QMAX);
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    uint32_t hword = 0, lword = 0;
    int qsum = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        int q = to_int_like_lrint(__fmul_rn(vv[j], inv));
        q = q > IMAX ? IMAX : (q < -IMAX ? -IMAX : q);
        qsum += q;
        if (HP) {
            const uint32_t u = static_cast<uint32_t>(q + 32768);
            hword |= ((u >> 8) ^ 0x80u) << (8 * j);      // hi - 128 as a signed byte
            lword |= (u & 0xFFu) << (8 * j);
        } else {
            lword |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * j);   // q8 as a signed byte
        }
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
    if (!store) return;
    uint8_t* rec = out.q + static_cast<size_t>(b) * out.QREC;
    if (m < out.TPB) {
        // word c of each plane: slot t = c % 4, first (c < 4) or second half of the slot's words
        uint8_t* slot = rec + m * 4 * LB + (c & 3) * LB + (c < 4 ? 0 : 4);
        if (HP) {
            *reinterpret_cast<uint32_t*>(slot) = hword;
            *reinterpret_cast<uint32_t*>(slot + 8) = lword;
        } else {
            *reinterpret_cast<uint32_t*>(slot) = lword;
        }
    }
    if (c == 0) {
        reinterpret_cast<float*>(rec + out.TPB * 4 * LB)[m] = scale;
        reinterpret_cast<int32_t*>(rec + out.TPB * 4 * LB + out.TPBA * 4)[m] = qsum;
    }
}

}  // namespace ql
