// ql_internal.h -- host-side types shared by the CUDA translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace ql {

// Device-resident packed weight (the opaque handle behind void*).
//
// HBM layout: one record per (16-row group, 32-wide K block), records of a row
// group contiguous in K order, so a stage of any number of blocks of one row
// group is ONE contiguous bulk copy:
//   rec[G][nblk][REC]   REC = TB + SB + ZB bytes (a multiple of 16):
//     [0, TB)           16x32 tile in mma.sync m16n8k32 A-fragment order:
//                       lane L = 4g + t owns rows {g, g+8} x k {4t..4t+3, 16+4t..16+4t+3}.
//                       INT8: 16 bytes per lane, byte = q ^ 0x80 (= q - 128, signed).
//                       INT4: 8 bytes per lane, raw nibbles q; word 0 interleaves
//                       (row g, row g+8) for k 4t..4t+3, word 1 the same for k+16.
//                       TB = 512 (INT8) or 256 (INT4).
//     [TB, TB+SB)       16 block scales, entry 2g = row g, 2g+1 = row g+8; the
//                       caller's fp16 bits (SB = 32) or fp32 (SB = 64).
//     [TB+SB, REC)      INT4 explicit zero points only (ZB = 16): byte g =
//                       zp(g) | zp(g+8) << 4 for g < 8, then 8 padding bytes.
struct Weight {
    uint32_t magic;
    int N, K, nblk, bits;
    int scale_half;       // 1: fp16 scales, 0: fp32
    int has_zp;           // INT4 with explicit zero points
    int device;
    int G;                // N / 16 row groups
    int TB, SB, ZB, REC;  // record geometry (bytes)
    uint8_t* W;           // records
    size_t bytes;         // device bytes owned
};

constexpr uint32_t WEIGHT_MAGIC = 0x51574232u;   // "QWB2"

inline bool valid_weight(const void* h) {
    return h && static_cast<const Weight*>(h)->magic == WEIGHT_MAGIC;
}

inline void weight_geometry(int bits, bool scale_half, bool has_zp, int* TB, int* SB, int* ZB, int* REC) {
    *TB = bits == 8 ? 512 : 256;
    *SB = scale_half ? 32 : 64;
    *ZB = has_zp ? 16 : 0;
    *REC = *TB + *SB + *ZB;
}

// Quantized activations in the kernels' layout (scratch produced per call):
// one record per 32-wide K block, so a stage of blocks is one bulk copy.
//   rec[nblk][QREC]            QREC = TPB*4*LB + TPBA*8 bytes
//     [0, TPB*4*LB)            fragments of token m at m*4*LB: slot t holds what
//                              lane 4*(m%8)+t needs as its m16n8k32 B fragment --
//                              two-pass (LB = 16): hi-128 (signed) of k 4t..4t+3
//                              and 16+4t..16+4t+3, then lo (unsigned) of the same
//                              k; single-pass (LB = 8): q8 (signed) of those k.
//     [TPB*4*LB, +TPBA*4)      fp32 activation scales of tokens 0..TPBA-1;
//     [.., QREC)               int32 block sums of the quantized values (sum of
//                              q16, or of q8), for kernels that take the zero
//                              point out of the weights: sum q16*(q - zp) =
//                              sum q16*q - zp * sum q16.
// MT = token groups of 8 (1, 2, 4 or 8).  TPB = M when MT == 1 (only the real
// tokens are stored and copied) else 8*MT; TPBA = TPB rounded up to 4.
// Padded tokens (M..TPB-1, and scales up to TPBA) are written as zeros.
struct ActView {
    uint8_t* q;
    int M, MT, nblk;
    int TPB, TPBA;
    int LB;               // bytes per fragment slot (16 two-pass, 8 single-pass)
    int QREC;             // record bytes per block
    int hp;               // layout/mode the records were written in
};

size_t act_bytes(int M, int nblk);                       // one chunk of M <= 64 tokens
ActView act_carve(void* ws, int M, int nblk, bool hi_prec);

// Optional RMSNorm prologue of the activation quantizers (the reference
// decoder's rmsnorm before its projections, kernel/qwen35_decoder.cpp:133-141):
// the value quantized for (m, k) is (x[m][k] * row_inv[m]) * w[k], two rounded
// fp32 products in that order, and hn (if set) receives it.
struct NormArgs {
    const float* row_inv;   // [M] 1/sqrt(mean(x^2) + eps), from launch_rmsnorm_factors
    const float* w;         // [K] norm weights
    float* hn;              // [M][ldh] the values quantized (normalised rows, or silu * up), or nullptr
    int ldh;
    const float* up;        // SiLU prologue: [M][ldu] up-projection output multiplying silu(A)
    int ldu;
};
// row_inv[m] for M rows of X (ldx floats apart, K wide), ql_norm.cu.
cudaError_t launch_rmsnorm_factors(const float* X, int ldx, int M, int K, float eps, float* row_inv,
                                   cudaStream_t stream);
// Decode layout (M <= 64): the row factors and the quantizer with the norm
// applied in one launch (one CTA per token row), ql_norm.cu.
cudaError_t launch_quantize_act_norm(const float* X, int ldx, int M, int K, float eps, bool hi_prec,
                                     const ActView& out, const NormArgs& nrm, cudaStream_t stream);

constexpr int MAX_DECODE_TOKENS = 64;                    // MT <= 8 token groups

// Prefill (M > MAX_DECODE_TOKENS) runs the tcgen05 GEMMs (ql_gemm16.cu,
// ql_gemm.cu) on activations quantized into a token-half-major buffer:
//   planes  [m_tiles][2 halves][nblk][GEMM_HPLANES]: per 64-token half of a
//           128-token tile and 32-wide block, the hi plane (hi - 128, s8; q8 in
//           single-pass mode) then the lo plane (u8), each [2 K halves][8 token
//           groups][8 tokens x 16 B] -- the canonical K-major tcgen05 B operand
//           of 64 tokens (LBO 1024 B, SBO 128 B);
//   scales  [m_tiles][nblk][128] fp32 activation scales, after all planes.
// A half's planes are contiguous across blocks, so a stage of blocks of one
// half is one bulk copy; tokens M..(tile end) are zeros.
constexpr int GEMM_HPLANES = 4096;
constexpr int GEMM_SCALES = 128 * 4;
constexpr int GEMM_AREC = 2 * GEMM_HPLANES + GEMM_SCALES;   // bytes per (tile, block)
__host__ __device__ inline size_t gemm_planes_off(int mt, int h, int b, int nblk) {
    return ((static_cast<size_t>(mt) * 2 + h) * nblk + b) * GEMM_HPLANES;
}
__host__ __device__ inline size_t gemm_scales_off(int mt, int b, int m_tiles, int nblk) {
    return static_cast<size_t>(m_tiles) * 2 * nblk * GEMM_HPLANES +
           (static_cast<size_t>(mt) * nblk + b) * GEMM_SCALES;
}
size_t gemm_act_bytes(int M, int nblk);
cudaError_t launch_quantize_gemm(const float* A, int lda, int M, int K, bool hi_prec, uint8_t* out,
                                 cudaStream_t stream, const NormArgs* norm = nullptr);
cudaError_t launch_gemm(const Weight* w, const uint8_t* act, int M, bool hi_prec, float* C, int ldc,
                        int32_t* cs, cudaStream_t stream);

// INT4 weights with fp16 scales in two-pass mode also have a kind::f16 GEMM
// (ql_gemm16.cu) on the same activation records; launch_gemm picks it unless
// the prefill kernel selector (ql_set_prefill_kernel) asks for kind::i8.
bool gemm16_supports(const Weight* w, bool hi_prec);
cudaError_t launch_gemm16(const Weight* w, const uint8_t* act, int M, float* C, int ldc, int32_t* cs,
                          cudaStream_t stream);
enum : int { QL_PREFILL_AUTO = 0, QL_PREFILL_I8 = 1, QL_PREFILL_F16_PAIR = 2, QL_PREFILL_F16_STREAM = 3 };
int prefill_kernel();                                    // ql_api.cu

// INT4 prefill on pre-expanded FP16 operands (ql_gemmw.cu): the one-call
// entry points, given a workspace of ws_bytes_for_w() bytes, dequantize the
// weights once per call into [n_tiles][nblk][WREC16] (128 rows x 32 k FP16
// q - zp in the canonical tcgen05 A layout, then 128 fp32 weight scales) and
// quantize the activations into [m_tiles][nblk][AREC16_HP or _SP] (FP16 h and
// l/256 planes, or q8, in the B layout, then 128 fp32 activation scales).
constexpr int WREC16 = 128 * 32 * 2 + 128 * 4;           // 8704
constexpr int AREC16_HP = 2 * 128 * 32 * 2 + 128 * 4;    // 16896
constexpr int AREC16_SP = 128 * 32 * 2 + 128 * 4;        // 8704
bool gemmw_supports(const Weight* w);
size_t gemmw_act_bytes(int M, int nblk, bool hi_prec);
size_t gemmw_weight_bytes(const Weight* w);
cudaError_t launch_dequant_w16(const Weight* w, bool hi_prec, uint8_t* out, cudaStream_t stream);
cudaError_t launch_quantize_f16(const float* A, int lda, int M, int K, bool hi_prec, uint8_t* out,
                                cudaStream_t stream, const NormArgs* norm = nullptr);
cudaError_t launch_gemmw(const Weight* w, const uint8_t* wd, const uint8_t* ad, int M, bool hi_prec, float* C,
                         int ldc, int32_t* cs, cudaStream_t stream);

// Size of the fixed scratch behind ql_matmul_dev_noalloc (ql_api.cu); the
// public header states the same value as QL_NOALLOC_SCRATCH_BYTES.
constexpr size_t QL_NOALLOC_SCRATCH_BYTES = size_t(8) << 20;

// Launchers (return cudaError_t of the launch).
cudaError_t launch_quantize_act(const float* A, int lda, int M, int K, bool hi_prec,
                                const ActView& out, cudaStream_t stream, const NormArgs* norm = nullptr);
// The quantizers with the SiLU * up prologue (decode and GEMM layouts).
cudaError_t launch_quantize_act_silu(const float* G, const float* U, int ld, int M, int K, bool hi_prec,
                                     const ActView& out, float* dOut, cudaStream_t stream);
cudaError_t launch_quantize_gemm_silu(const float* G, const float* U, int ld, int M, int K, bool hi_prec,
                                      uint8_t* out, float* dOut, cudaStream_t stream);
cudaError_t launch_quantize_ref(const float* A, int M, int K, uint8_t* hi, uint8_t* lo,
                                float* ascale, cudaStream_t stream);
cudaError_t launch_decode(const Weight* w, const ActView& act, bool hi_prec, float* C,
                          int ldc, int32_t* cs, cudaStream_t stream, bool pdl);
// INT4 at one or two tokens: the dp4a decode kernel (ql_gemv4.cu), which
// launch_decode picks where it applies.
bool decode_dp4a_applies(const Weight* w, const ActView& act);
cudaError_t launch_decode_dp4a(const Weight* w, const ActView& act, bool hi_prec, float* C, int ldc, int32_t* cs,
                               cudaStream_t stream, bool pdl);

cudaError_t launch_prepack_onnx(Weight* w, const uint8_t* d_qw, const void* d_scales,
                                const uint8_t* d_qzeros, cudaStream_t stream);
cudaError_t launch_prepack_vnni(Weight* w, const uint8_t* d_B, const float* d_scales,
                                const int8_t* d_zp, cudaStream_t stream);

}  // namespace ql
