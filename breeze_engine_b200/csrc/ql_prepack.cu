// ql_prepack.cu -- device-side weight prepack.
//
// Replaces the reference's CPU packers (kernel/quantized_matmul.cpp:140-194
// pack_onnx<Bits,HalfScales> and :480-499 i4_prepack) with GPU kernels that
// rearrange bytes already copied to HBM into the record layout documented on
// ql::Weight (ql_internal.h).  Like the reference they reorder without
// dequantizing: INT4 nibbles stay nibbles, INT8 bytes become q ^ 0x80, and
// fp16 scales keep their bits (widened exactly at use, as _cvtsh_ss does).
#include "ql_common.cuh"
#include "ql_internal.h"

namespace ql {

// Weights: one thread per (group, block, lane) writes that lane's fragment bytes.
template <int BITS>
__global__ void prepack_onnx_w_kernel(const uint8_t* __restrict__ qw, int G, int nblk, int REC,
                                      uint8_t* __restrict__ W) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblk * 32) return;
    const int lane = static_cast<int>(idx & 31);
    const long long tile = idx >> 5;                 // G * nblk + b
    const int b = static_cast<int>(tile % nblk);
    const int grp = static_cast<int>(tile / nblk);
    const int g = lane >> 2, t = lane & 3;
    const size_t row0 = static_cast<size_t>(grp) * 16 + g, row1 = row0 + 8;
    uint8_t* rec = W + tile * REC;
    if (BITS == 8) {
        const uint8_t* r0 = qw + (row0 * nblk + b) * 32;
        const uint8_t* r1 = qw + (row1 * nblk + b) * 32;
        auto word = [](const uint8_t* p) {
            return (static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
                    (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24)) ^
                   0x80808080u;
        };
        uint4 v;
        v.x = word(r0 + 4 * t);
        v.y = word(r1 + 4 * t);
        v.z = word(r0 + 16 + 4 * t);
        v.w = word(r1 + 16 + 4 * t);
        reinterpret_cast<uint4*>(rec)[lane] = v;
    } else {
        const uint8_t* r0 = qw + (row0 * nblk + b) * 16;
        const uint8_t* r1 = qw + (row1 * nblk + b) * 16;
        auto nib = [](const uint8_t* r, int k) { return (r[k >> 1] >> (4 * (k & 1))) & 15u; };
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w0 |= nib(r0, 4 * t + j) << (8 * j);
            w0 |= nib(r1, 4 * t + j) << (8 * j + 4);
            w1 |= nib(r0, 16 + 4 * t + j) << (8 * j);
            w1 |= nib(r1, 16 + 4 * t + j) << (8 * j + 4);
        }
        reinterpret_cast<uint2*>(rec)[lane] = make_uint2(w0, w1);
    }
}

// Scales: entry i of the record's scale field is row (i >> 1) + 8 * (i & 1)
// of the group, from the MatMulNBits scales [N][nblk].
template <typename T>
__global__ void prepack_scales_kernel(const T* __restrict__ in, int G, int nblk, int REC, int TB,
                                      uint8_t* __restrict__ W) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblk * 16) return;
    const int i = static_cast<int>(idx & 15);
    const long long tile = idx >> 4;
    const int b = static_cast<int>(tile % nblk);
    const int grp = static_cast<int>(tile / nblk);
    const size_t row = static_cast<size_t>(grp) * 16 + (i >> 1) + 8 * (i & 1);
    reinterpret_cast<T*>(W + tile * REC + TB)[i] = in[row * nblk + b];
}

// Zero points: byte g (< 8) of the record's zp field = zp(row g) | zp(row g+8) << 4,
// from the packed MatMulNBits qzeros [N][ceil(nblk/2)] (low nibble = even block);
// bytes 8..15 are padding.
__global__ void prepack_zp_kernel(const uint8_t* __restrict__ qz, int G, int nblk, int REC, int OFF,
                                  uint8_t* __restrict__ W) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblk * 16) return;
    const int g = static_cast<int>(idx & 15);
    const long long tile = idx >> 4;
    const int b = static_cast<int>(tile % nblk);
    const int grp = static_cast<int>(tile / nblk);
    uint8_t* dst = W + tile * REC + OFF;
    if (g >= 8) {
        dst[g] = 0;
        return;
    }
    const int packed = (nblk + 1) / 2;
    auto zp = [&](size_t row) { return (qz[row * packed + b / 2] >> (4 * (b & 1))) & 15; };
    const size_t row0 = static_cast<size_t>(grp) * 16 + g;
    dst[g] = static_cast<uint8_t>(zp(row0) | (zp(row0 + 8) << 4));
}

// Legacy VNNI layout (kernel/quantized_matmul.cpp:480-499): B [ntiles][nblk][8][32|64],
// scales fp32 [ntiles][nblk][16], zp s8 [ntiles][nblk][16].  The 16-column VNNI
// tile is one 16-row group here.  INT4 value (col, k) is nibble k%2 of byte
// g4*32 + col*2 + (k%4)/2 with g4 = (k%32)/4; INT8 byte (col, k) = B[g4*64 + col*4 + k%4].
template <int BITS>
__global__ void prepack_vnni_w_kernel(const uint8_t* __restrict__ B, int G, int nblk, int REC,
                                      uint8_t* __restrict__ W) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblk * 32) return;
    const int lane = static_cast<int>(idx & 31);
    const long long tile = idx >> 5;
    const int g = lane >> 2, t = lane & 3;
    constexpr int GB = BITS == 8 ? 64 : 32;
    const uint8_t* src = B + tile * 8 * GB;
    uint8_t* rec = W + tile * REC;
    auto val = [&](int col, int k) -> uint32_t {
        const int g4 = k >> 2, j = k & 3;
        if (BITS == 8) return src[g4 * 64 + col * 4 + j];                 // already q - 128
        return (src[g4 * 32 + col * 2 + (j >> 1)] >> (4 * (j & 1))) & 15u;
    };
    if (BITS == 8) {
        uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w[0] |= val(g, 4 * t + j) << (8 * j);
            w[1] |= val(g + 8, 4 * t + j) << (8 * j);
            w[2] |= val(g, 16 + 4 * t + j) << (8 * j);
            w[3] |= val(g + 8, 16 + 4 * t + j) << (8 * j);
        }
        reinterpret_cast<uint4*>(rec)[lane] = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w0 |= val(g, 4 * t + j) << (8 * j);
            w0 |= val(g + 8, 4 * t + j) << (8 * j + 4);
            w1 |= val(g, 16 + 4 * t + j) << (8 * j);
            w1 |= val(g + 8, 16 + 4 * t + j) << (8 * j + 4);
        }
        reinterpret_cast<uint2*>(rec)[lane] = make_uint2(w0, w1);
    }
}

__global__ void prepack_vnni_meta_kernel(const float* __restrict__ sc, const int8_t* __restrict__ zp,
                                         int G, int nblk, int REC, int TB, int ZOFF, int has_zp,
                                         uint8_t* __restrict__ W) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblk * 16) return;
    const int i = static_cast<int>(idx & 15);
    const long long tile = idx >> 4;               // grp * nblk + b
    const int col = (i >> 1) + 8 * (i & 1);
    const size_t src = tile * 16;                  // [ntiles][nblk][16] flattened
    uint8_t* rec = W + tile * REC;
    reinterpret_cast<float*>(rec + TB)[i] = sc[src + col];
    if (has_zp)
        rec[ZOFF + i] = i < 8 ? static_cast<uint8_t>((zp[src + i] & 15) | ((zp[src + i + 8] & 15) << 4)) : 0;
}

static unsigned grid_for(long long n, int threads) {
    return static_cast<unsigned>((n + threads - 1) / threads);
}

cudaError_t launch_prepack_onnx(Weight* w, const uint8_t* d_qw, const void* d_scales,
                                const uint8_t* d_qzeros, cudaStream_t stream) {
    const int T = 256;
    const long long lanes = static_cast<long long>(w->G) * w->nblk * 32;
    if (w->bits == 8)
        prepack_onnx_w_kernel<8><<<grid_for(lanes, T), T, 0, stream>>>(d_qw, w->G, w->nblk, w->REC, w->W);
    else
        prepack_onnx_w_kernel<4><<<grid_for(lanes, T), T, 0, stream>>>(d_qw, w->G, w->nblk, w->REC, w->W);
    const long long sn = static_cast<long long>(w->G) * w->nblk * 16;
    if (w->scale_half)
        prepack_scales_kernel<uint16_t><<<grid_for(sn, T), T, 0, stream>>>(
            static_cast<const uint16_t*>(d_scales), w->G, w->nblk, w->REC, w->TB, w->W);
    else
        prepack_scales_kernel<float><<<grid_for(sn, T), T, 0, stream>>>(
            static_cast<const float*>(d_scales), w->G, w->nblk, w->REC, w->TB, w->W);
    if (w->has_zp)
        prepack_zp_kernel<<<grid_for(sn, T), T, 0, stream>>>(d_qzeros, w->G, w->nblk, w->REC,
                                                             w->TB + w->SB, w->W);
    return cudaGetLastError();
}

cudaError_t launch_prepack_vnni(Weight* w, const uint8_t* d_B, const float* d_scales,
                                const int8_t* d_zp, cudaStream_t stream) {
    const int T = 256;
    const long long lanes = static_cast<long long>(w->G) * w->nblk * 32;
    if (w->bits == 8)
        prepack_vnni_w_kernel<8><<<grid_for(lanes, T), T, 0, stream>>>(d_B, w->G, w->nblk, w->REC, w->W);
    else
        prepack_vnni_w_kernel<4><<<grid_for(lanes, T), T, 0, stream>>>(d_B, w->G, w->nblk, w->REC, w->W);
    const long long mn = static_cast<long long>(w->G) * w->nblk * 16;
    prepack_vnni_meta_kernel<<<grid_for(mn, T), T, 0, stream>>>(d_scales, d_zp, w->G, w->nblk, w->REC,
                                                                w->TB, w->TB + w->SB, w->has_zp, w->W);
    return cudaGetLastError();
}

}  // namespace ql
