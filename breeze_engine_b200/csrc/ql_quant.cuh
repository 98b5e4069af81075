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

// The 32 values of (token m, block b): row m of A itself or, with the RMSNorm
// prologue (NORM), normalised by the precomputed factor row_inv[m].
template <bool NORM>
__device__ __forceinline__ void load_block(const float* __restrict__ A, int lda, int m, int b,
                                           const NormArgs& nrm, float (&v)[32]) {
    load_raw_block(A, lda, m, b, v);
    if (NORM) norm_block(v, __ldg(nrm.row_inv + m), nrm, m, b);
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

}  // namespace ql
