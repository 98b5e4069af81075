// ql_quant.cu -- activation quantizer (FP32 -> per-32-block INT16 hi/lo planes).
//
// Bit-exact restatement on the GPU of the reference quantize_A_i16
// (kernel/quantized_matmul.cpp:237-258) and, for the single-pass mode,
// quantize_A (:215-232):
//   amax  = max |a| over the block (a NaN never wins the compare)
//   scale = amax / 32767.f            (__fdiv_rn: IEEE division, one rounding)
//   inv   = scale > 0 ? 1.f / scale : 0
//   q     = clamp((int)lrint(a * inv), -32767, 32767)
// lrint rounds to nearest-even and the reference truncates its 64-bit result
// to int: NaN / inf / |x| >= 2^63 give 0, |x| in [2^31, 2^63) keep the low
// 32 bits.  to_int_like_lrint() reproduces that for every float.
//
// Decode layout: 8 lanes own one (token, block) pair, each reading 16 bytes of
// A and writing one word of each plane (ql_quant.cuh, act_store_quad), so a
// decode call waits for one short pass.  GEMM layout: one thread per pair,
// 128 contiguous bytes of A in, 16-byte chunks of each plane out.  Both are a
// single HBM pass.
#include "ql_common.cuh"
#include "ql_internal.h"
#include "ql_quant.cuh"

namespace ql {

template <bool HP, int PRO>
__global__ void __launch_bounds__(256) quantize_act_kernel(const float* __restrict__ A, int lda,
                                                           int M, int K, ActView out, NormArgs nrm) {
    // Let a dependent (PDL) kernel start its weight streaming right away; it
    // still waits for this grid's completion before reading the planes.  This
    // grid itself may have started before its predecessor finished (it is
    // launched with PDL too): wait for it before reading A or writing planes.
    pdl_launch_dependents();
    pdl_wait();
    // 8 lanes per (token, block) pair (ql_quant.cuh, act_store_quad); padded
    // token rows quantize zeros into the zero record
    const int nblk = K / BLOCK_K;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long unit = idx >> 3;
    const int c = static_cast<int>(idx & 7);
    const bool valid = unit < static_cast<long long>(out.TPBA) * nblk;
    const int m = valid ? static_cast<int>(unit / nblk) : 0;
    const int b = valid ? static_cast<int>(unit % nblk) : 0;
    const float4 v = (valid && m < M) ? load_quad<PRO>(A, lda, m, b, c, nrm) : make_float4(0.f, 0.f, 0.f, 0.f);
    act_store_quad<HP>(v, out, m, b, c, valid);
}

// GEMM-layout variant (M > 64, ql_gemm16.cu / ql_gemm.cu): the token-half-major
// buffer of ql_internal.h -- per (64-token half, block) the hi plane (hi - 128,
// s8; q8 in single-pass mode) and the lo plane (u8) as canonical K-major
// tcgen05 B operands [2 K halves][8 groups of 8 tokens][8 tokens x 16 B], and
// per (128-token tile, block) 128 fp32 scales.  Tokens M..(tile end) are zeros.
template <bool HP, int PRO>
__global__ void __launch_bounds__(256) quantize_gemm_kernel(const float* __restrict__ A, int lda, int M, int K,
                                                            int m_tiles, uint8_t* __restrict__ out, NormArgs nrm) {
    pdl_launch_dependents();
    pdl_wait();                 // launched with PDL: the predecessor may still run
    const int nblk = K / BLOCK_K;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(m_tiles) * 128 * nblk) return;
    const int m = static_cast<int>(idx / nblk);
    const int b = static_cast<int>(idx % nblk);
    const int mt = m >> 7, mr = m & 127, tw = mr & 63;     // token within its 64-token half
    uint8_t* planes = out + gemm_planes_off(mt, mr >> 6, b, nblk);
    const int o = (tw >> 3) * 128 + (tw & 7) * 16;            // K half 0; K half 1 at +1024
    float* scale = reinterpret_cast<float*>(out + gemm_scales_off(mt, b, m_tiles, nblk)) + mr;
    if (m >= M) {
        const uint4 z = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(planes + o) = z;
        *reinterpret_cast<uint4*>(planes + o + 1024) = z;
        *reinterpret_cast<uint4*>(planes + 2048 + o) = z;
        *reinterpret_cast<uint4*>(planes + 2048 + o + 1024) = z;
        *scale = 0.0f;
        return;
    }
    float v[32];
    load_block<PRO>(A, lda, m, b, nrm, v);
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float a = fabsf(v[i]);
        amax = (a > amax) ? a : amax;
    }
    constexpr float QMAX = HP ? 32767.0f : 127.0f;
    constexpr int IMAX = HP ? 32767 : 127;
    const float scl = __fdiv_rn(amax, QMAX);
    const float inv = scl > 0.0f ? __fdiv_rn(1.0f, scl) : 0.0f;
    *scale = scl;
    uint32_t hw[8], lw[8];
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        uint32_t hword = 0, lword = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int q = to_int_like_lrint(__fmul_rn(v[4 * w + j], inv));
            q = q > IMAX ? IMAX : (q < -IMAX ? -IMAX : q);
            if (HP) {
                const uint32_t u = static_cast<uint32_t>(q + 32768);
                hword |= ((u >> 8) ^ 0x80u) << (8 * j);
                lword |= (u & 0xFFu) << (8 * j);
            } else {
                lword |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * j);
            }
        }
        hw[w] = hword;
        lw[w] = lword;
    }
    *reinterpret_cast<uint4*>(planes + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(planes + o + 1024) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    *reinterpret_cast<uint4*>(planes + 2048 + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    *reinterpret_cast<uint4*>(planes + 2048 + o + 1024) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
}

// Launches a quantizer with programmatic dependent launch: it may start while
// the previous kernel on the stream (a matmul of the previous layer) drains,
// and waits for it with griddepcontrol.wait before touching memory.
template <typename... Args>
static cudaError_t launch_pdl(void (*kern)(Args...), unsigned grid, unsigned threads, cudaStream_t stream,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

cudaError_t launch_quantize_gemm(const float* A, int lda, int M, int K, bool hi_prec, uint8_t* out,
                                 cudaStream_t stream, const NormArgs* norm) {
    const int m_tiles = (M + 127) / 128;
    const long long total = static_cast<long long>(m_tiles) * 128 * (K / BLOCK_K);
    const int threads = 256;
    const unsigned grid = static_cast<unsigned>((total + threads - 1) / threads);
    const NormArgs n = norm ? *norm : NormArgs{};
    if (norm) {
        if (hi_prec) return launch_pdl(quantize_gemm_kernel<true, PRO_NORM>, grid, threads, stream, A, lda, M, K, m_tiles, out, n);
        return launch_pdl(quantize_gemm_kernel<false, PRO_NORM>, grid, threads, stream, A, lda, M, K, m_tiles, out, n);
    }
    if (hi_prec) return launch_pdl(quantize_gemm_kernel<true, PRO_NONE>, grid, threads, stream, A, lda, M, K, m_tiles, out, n);
    return launch_pdl(quantize_gemm_kernel<false, PRO_NONE>, grid, threads, stream, A, lda, M, K, m_tiles, out, n);
}

// Reference-layout variant for parity checks: hi/lo unsigned [M][K] (the
// reference's au8_hi / au8_lo) and ascale [M][K/32].
__global__ void __launch_bounds__(256) quantize_ref_kernel(const float* __restrict__ A, int M, int K,
                                                           uint8_t* __restrict__ hi,
                                                           uint8_t* __restrict__ lo,
                                                           float* __restrict__ ascale) {
    const int nblk = K / BLOCK_K;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(M) * nblk) return;
    const int m = static_cast<int>(idx / nblk);
    const int b = static_cast<int>(idx % nblk);
    const float* a = A + static_cast<size_t>(m) * K + b * BLOCK_K;
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) {
        const float v = fabsf(a[i]);
        amax = (v > amax) ? v : amax;
    }
    const float scale = __fdiv_rn(amax, 32767.0f);
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    ascale[idx] = scale;
    for (int i = 0; i < 32; ++i) {
        int q = to_int_like_lrint(__fmul_rn(a[i], inv));
        q = q > 32767 ? 32767 : (q < -32767 ? -32767 : q);
        const uint32_t u = static_cast<uint32_t>(q + 32768);
        hi[static_cast<size_t>(m) * K + b * BLOCK_K + i] = static_cast<uint8_t>(u >> 8);
        lo[static_cast<size_t>(m) * K + b * BLOCK_K + i] = static_cast<uint8_t>(u & 0xFF);
    }
}

// Token groups of 8, rounded up to a power of two (the decode kernel is
// instantiated for 1, 2, 4 and 8 groups; padded tokens are zero rows).
static int act_groups(int M) {
    const int mt = (M + 7) / 8;
    return mt <= 1 ? 1 : mt <= 2 ? 2 : mt <= 4 ? 4 : 8;
}
static int act_tpb(int M) { return act_groups(M) == 1 ? M : 8 * act_groups(M); }
static int act_tpba(int M) { return (act_tpb(M) + 3) & ~3; }

// Sized for the two-pass layout (the larger one) whatever the mode.
size_t act_bytes(int M, int nblk) {
    const size_t rec = static_cast<size_t>(act_tpb(M)) * 64 + act_tpba(M) * 8;
    return (static_cast<size_t>(nblk) * rec + 255) & ~size_t(255);
}

ActView act_carve(void* ws, int M, int nblk, bool hi_prec) {
    ActView v;
    v.M = M;
    v.MT = act_groups(M);
    v.TPB = act_tpb(M);
    v.TPBA = act_tpba(M);
    v.nblk = nblk;
    v.hp = hi_prec ? 1 : 0;
    v.LB = hi_prec ? 16 : 8;
    v.QREC = v.TPB * 4 * v.LB + v.TPBA * 8;
    v.q = static_cast<uint8_t*>(ws);
    return v;
}

cudaError_t launch_quantize_act(const float* A, int lda, int M, int K, bool hi_prec,
                                const ActView& out, cudaStream_t stream, const NormArgs* norm) {
    const long long total = 8LL * out.TPBA * (K / BLOCK_K);          // 8 lanes per (token, block)
    const int threads = 256;
    const unsigned grid = static_cast<unsigned>((total + threads - 1) / threads);
    const NormArgs n = norm ? *norm : NormArgs{};
    if (norm) {
        if (hi_prec) return launch_pdl(quantize_act_kernel<true, PRO_NORM>, grid, threads, stream, A, lda, M, K, out, n);
        return launch_pdl(quantize_act_kernel<false, PRO_NORM>, grid, threads, stream, A, lda, M, K, out, n);
    }
    if (hi_prec) return launch_pdl(quantize_act_kernel<true, PRO_NONE>, grid, threads, stream, A, lda, M, K, out, n);
    return launch_pdl(quantize_act_kernel<false, PRO_NONE>, grid, threads, stream, A, lda, M, K, out, n);
}

// SiLU * up prologue (the down projection's input): G and U are the gate and
// up projections' outputs, ld floats per row; dOut (may be null, [M][K])
// receives the values quantized.
cudaError_t launch_quantize_act_silu(const float* G, const float* U, int ld, int M, int K, bool hi_prec,
                                     const ActView& out, float* dOut, cudaStream_t stream) {
    const long long total = 8LL * out.TPBA * (K / BLOCK_K);          // 8 lanes per (token, block)
    const int threads = 256;
    const unsigned grid = static_cast<unsigned>((total + threads - 1) / threads);
    const NormArgs n{nullptr, nullptr, dOut, K, U, ld};
    if (hi_prec) return launch_pdl(quantize_act_kernel<true, PRO_SILU>, grid, threads, stream, G, ld, M, K, out, n);
    return launch_pdl(quantize_act_kernel<false, PRO_SILU>, grid, threads, stream, G, ld, M, K, out, n);
}

cudaError_t launch_quantize_gemm_silu(const float* G, const float* U, int ld, int M, int K, bool hi_prec,
                                      uint8_t* out, float* dOut, cudaStream_t stream) {
    const int m_tiles = (M + 127) / 128;
    const long long total = static_cast<long long>(m_tiles) * 128 * (K / BLOCK_K);
    const int threads = 256;
    const unsigned grid = static_cast<unsigned>((total + threads - 1) / threads);
    const NormArgs n{nullptr, nullptr, dOut, K, U, ld};
    if (hi_prec)
        return launch_pdl(quantize_gemm_kernel<true, PRO_SILU>, grid, threads, stream, G, ld, M, K, m_tiles, out, n);
    return launch_pdl(quantize_gemm_kernel<false, PRO_SILU>, grid, threads, stream, G, ld, M, K, m_tiles, out, n);
}

cudaError_t launch_quantize_ref(const float* A, int M, int K, uint8_t* hi, uint8_t* lo,
                                float* ascale, cudaStream_t stream) {
    const long long total = static_cast<long long>(M) * (K / BLOCK_K);
    if (total == 0) return cudaSuccess;
    const int threads = 256;
    const unsigned grid = static_cast<unsigned>((total + threads - 1) / threads);
    quantize_ref_kernel<<<grid, threads, 0, stream>>>(A, M, K, hi, lo, ascale);
    return cudaGetLastError();
}

}  // namespace ql
