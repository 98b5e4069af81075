// ql_norm.cu -- RMSNorm row factors for the fused norm -> quantize prologue.
//
// The reference decoder normalises every row before its projections
// (kernel/qwen35_decoder.cpp:133-141):
//   double ss = 0; for j: ss += (double)x[j] * x[j];      // serial, in j order
//   float inv = 1.0f / std::sqrt((float)(ss / H) + eps);
//   o[j] = x[j] * inv * w[j];
// This file computes inv per row bit-exactly.  For the tensor-core GEMM layout
// (more than 64 tokens) rmsnorm_factor_kernel writes the factors and the GEMM
// quantizer applies the last line (ql_quant.cuh, load_block); for the decode
// layout quantize_act_norm_kernel does both in one launch, one CTA per row.
//
// Every square (double)x*x of a finite float is exact in double (24-bit
// significands give 48-bit products, and the exponent range of a float
// squared stays inside double's normal range), so the only roundings in ss
// are the serial additions.  A row is summed here in parallel (one CTA per
// row, any order) to P.  For n non-negative terms every summation order has a
// relative error of at most g = (n-1)u/(1-(n-1)u), u = 2^-53 (Higham,
// "Accuracy and Stability of Numerical Algorithms", 2nd ed., Sec. 4.2), so
// the reference's serial sum lies in [P(1-d), P(1+d)] for d = (8n+8)u, which
// covers both orders' errors and the rounding of the interval ends.  The map
// s -> (float)(s / H) is monotone, so when both ends of the interval round to
// the same float that float IS the reference's mean; otherwise (a mean within
// about 2^-45 relative of a float rounding boundary: ~1e-4 of rows at H =
// 5120) the CTA's first thread repeats the reference's serial loop.  Rows with
// an inf or NaN have a non-finite P and a non-finite serial sum of the same
// kind (NaN if any element is NaN, else +inf), and both give the same mean.
#include <cfloat>

#include "ql_common.cuh"
#include "ql_internal.h"
#include "ql_quant.cuh"

namespace ql {

namespace {

// The reference's serial loop and its conversion to the float mean.
__device__ __noinline__ float serial_mean(const float* __restrict__ x, int K) {
    double ss = 0.0;
    for (int j = 0; j < K; ++j) {
        const double v = static_cast<double>(x[j]);
        ss = __dadd_rn(ss, __dmul_rn(v, v));
    }
    return __double2float_rn(__ddiv_rn(ss, static_cast<double>(K)));
}

__device__ float certified_mean(const float* __restrict__ x, int K, double p) {
    const double H = static_cast<double>(K);
    if (!(p <= DBL_MAX)) return __double2float_rn(__ddiv_rn(p, H));   // NaN or +inf
    // d = (8K + 8) * 2^-53: 1 - d and 1 + d are exact doubles (an even multiple
    // of 2^-53 above 1, any multiple below it).
    const double d = static_cast<double>(8 * static_cast<long long>(K) + 8) * 0x1p-53;
    const float lo = __double2float_rn(__ddiv_rn(__dmul_rn(p, 1.0 - d), H));
    const float hi = __double2float_rn(__ddiv_rn(__dmul_rn(p, 1.0 + d), H));
    if (lo == hi) return lo;
    return serial_mean(x, K);
}

constexpr int NORM_THREADS = 256;

// inv = 1/sqrt(mean(x^2) + eps) of one row, computed by the whole CTA
// (NORM_THREADS threads, all of which must call it); every thread gets it.
__device__ float block_row_inv(const float* __restrict__ x, int K, float eps) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    double s = 0.0;
    for (int i = threadIdx.x; i < K / 4; i += NORM_THREADS) {
        const float4 f = __ldg(x4 + i);
        const double a = f.x, b = f.y, c = f.z, e = f.w;
        s += a * a + b * b + c * c + e * e;     // exact squares; sums in any order
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __shared__ double part[NORM_THREADS / 32];
    __shared__ float inv;
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double p = 0.0;
#pragma unroll
        for (int w = 0; w < NORM_THREADS / 32; ++w) p += part[w];
        const float mean = certified_mean(x, K, p);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    }
    __syncthreads();
    return inv;
}

// Row factors for the GEMM-layout quantizer (M > 64 tokens), one CTA per row.
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_factor_kernel(const float* __restrict__ X, int ldx,
                                                                      int M, int K, float eps,
                                                                      float* __restrict__ row_inv) {
    // Launched with PDL: the producer of X may still be draining.  The
    // quantizer that reads row_inv waits for this whole grid.
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x;
    if (m >= M) return;
    const float r = block_row_inv(X + static_cast<size_t>(m) * ldx, K, eps);
    if (threadIdx.x == 0) row_inv[m] = r;
}

// Decode layout (up to 64 tokens): one CTA per token row computes the row's
// factor and then quantizes the row's blocks with the norm applied, in one
// launch; CTAs of padded rows (M..TPBA-1) write their zero records.
template <bool HP>
__global__ void __launch_bounds__(NORM_THREADS) quantize_act_norm_kernel(const float* __restrict__ X, int ldx,
                                                                         int M, int K, float eps, ActView out,
                                                                         NormArgs nrm) {
    pdl_launch_dependents();   // the matmul may start streaming its weights
    pdl_wait();
    const int m = blockIdx.x;
    const int nblk = K / BLOCK_K;
    const bool real = m < M;                       // padded rows quantize zeros into zero records
    const float r = real ? block_row_inv(X + static_cast<size_t>(m) * ldx, K, eps) : 0.0f;
    // 8 lanes per block (ql_quant.cuh, act_store_quad); every lane runs every
    // round so the group shuffles stay converged
    const int c = threadIdx.x & 7;
    for (int b0 = 0; b0 < nblk; b0 += NORM_THREADS / 8) {
        const int b = b0 + (threadIdx.x >> 3);
        const bool valid = b < nblk;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid && real) {
            v = __ldg(reinterpret_cast<const float4*>(X + static_cast<size_t>(m) * ldx + b * BLOCK_K) + c);
            const float4 g = __ldg(reinterpret_cast<const float4*>(nrm.w + b * BLOCK_K) + c);
            v.x = __fmul_rn(__fmul_rn(v.x, r), g.x);    // (x * inv) * w, each product rounded
            v.y = __fmul_rn(__fmul_rn(v.y, r), g.y);
            v.z = __fmul_rn(__fmul_rn(v.z, r), g.z);
            v.w = __fmul_rn(__fmul_rn(v.w, r), g.w);
            if (nrm.hn) reinterpret_cast<float4*>(nrm.hn + static_cast<size_t>(m) * nrm.ldh + b * BLOCK_K)[c] = v;
        }
        act_store_quad<HP>(v, out, m, valid ? b : 0, c, valid);
    }
}

cudaError_t launch_norm(void (*kern)(const float*, int, int, int, float, ActView, NormArgs), unsigned grid,
                        cudaStream_t stream, const float* X, int ldx, int M, int K, float eps, const ActView& out,
                        const NormArgs& nrm) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NORM_THREADS);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, X, ldx, M, K, eps, out, nrm);
}

}  // namespace

cudaError_t launch_rmsnorm_factors(const float* X, int ldx, int M, int K, float eps, float* row_inv,
                                   cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(M));
    cfg.blockDim = dim3(NORM_THREADS);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rmsnorm_factor_kernel, X, ldx, M, K, eps, row_inv);
}

cudaError_t launch_quantize_act_norm(const float* X, int ldx, int M, int K, float eps, bool hi_prec,
                                     const ActView& out, const NormArgs& nrm, cudaStream_t stream) {
    if (M <= 0) return cudaSuccess;
    const unsigned grid = static_cast<unsigned>(out.TPBA);
    if (hi_prec) return launch_norm(quantize_act_norm_kernel<true>, grid, stream, X, ldx, M, K, eps, out, nrm);
    return launch_norm(quantize_act_norm_kernel<false>, grid, stream, X, ldx, M, K, eps, out, nrm);
}

}  // namespace ql
