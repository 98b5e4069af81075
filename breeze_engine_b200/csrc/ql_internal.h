// ql_internal.h -- host-side types shared by the CUDA translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace ql {

// Device-resident packed weight (the opaque handle behind void*).
//
// HBM layout (all arrays 256-byte aligned, G = N/16 row groups):
//   W  [G][nblk][TB]    TB = 256 (INT4) or 512 (INT8).  One 16-row x 32-k tile
//                       per (group, block) in mma.sync m16n8k32 A-fragment order:
//                       lane L = 4g + t owns rows {g, g+8} x k {4t..4t+3, 16+4t..16+4t+3}.
//                       INT8: 16 bytes per lane, byte = q ^ 0x80 (= q - 128, signed).
//                       INT4: 8 bytes per lane, raw nibbles q; word 0 interleaves
//                       (row g, row g+8) for k 4t..4t+3, word 1 the same for k+16.
//   S  [G][nblk][16]    block scales, entry 2g = row g, 2g+1 = row g+8; kept as
//                       the caller's fp16 bits (exact widening on use) or fp32.
//   Z  [G][nblkZ][8]    INT4 explicit zero points only: byte g = zp(g) | zp(g+8) << 4;
//                       nblkZ = nblk rounded up to even (16-byte bulk copies).
struct Weight {
    uint32_t magic;
    int N, K, nblk, bits;
    int scale_half;       // 1: S holds fp16, 0: fp32
    int has_zp;           // INT4 with explicit zero points
    int device;
    int G, nblkZ;
    uint8_t* W;
    void* S;
    uint8_t* Z;
    size_t bytes;         // device bytes owned
};

constexpr uint32_t WEIGHT_MAGIC = 0x51574231u;   // "QWB1"

inline bool valid_weight(const void* h) {
    return h && static_cast<const Weight*>(h)->magic == WEIGHT_MAGIC;
}

// Quantized activations in the kernels' layout (scratch produced per call).
//   hs [nblk][MT][2][8][16]  hi plane as signed bytes (hi - 128); unused in
//                            INT8 single-pass mode.
//   lo [nblk][MT][2][8][16]  lo plane (unsigned) or, in single-pass mode, q8 (signed).
//   as [nblk][8*MT]          activation block scales (fp32).
// Token m lives in token group m/8, row m%8; [2] is the 16-byte K half.
// Padded tokens (M..8*MT-1) are written as zeros.
struct ActView {
    uint8_t* hs;
    uint8_t* lo;
    float* as;
    int M, MT, nblk;
};

size_t act_bytes(int M, int nblk);                       // one chunk of M <= 64 tokens
ActView act_carve(void* ws, int M, int nblk);

constexpr int MAX_DECODE_TOKENS = 64;                    // MT <= 8 token groups

// Launchers (return cudaError_t of the launch).
cudaError_t launch_quantize_act(const float* A, int lda, int M, int K, bool hi_prec,
                                const ActView& out, cudaStream_t stream);
cudaError_t launch_quantize_ref(const float* A, int M, int K, uint8_t* hi, uint8_t* lo,
                                float* ascale, cudaStream_t stream);
cudaError_t launch_decode(const Weight* w, const ActView& act, bool hi_prec, float* C,
                          int ldc, int32_t* cs, cudaStream_t stream, bool pdl);

cudaError_t launch_prepack_onnx(Weight* w, const uint8_t* d_qw, const void* d_scales,
                                const uint8_t* d_qzeros, cudaStream_t stream);
cudaError_t launch_prepack_vnni(Weight* w, const uint8_t* d_B, const float* d_scales,
                                const int8_t* d_zp, cudaStream_t stream);

}  // namespace ql
