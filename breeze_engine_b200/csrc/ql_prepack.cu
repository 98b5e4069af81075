// ql_prepack.cu -- device-side weight prepack.
//
// Replaces the reference's CPU packers (kernel/quantized_matmul.cpp:140-194
// pack_onnx<Bits,HalfScales> and :480-499 i4_prepack) with GPU kernels that
// rearrange bytes already copied to HBM into the layout documented on
// ql::Weight (ql_internal.h).  Like the reference they reorder without
// dequantizing: INT4 nibbles stay nibbles, INT8 bytes become q ^ 0x80, and
// fp16 scales keep their bits (widened exactly at use, as _cvtsh_ss does).
#include "ql_common.cuh"
#include "ql_internal.h"

namespace ql {

// One thread per (group, block, lane): writes that lane's fragment bytes.
template <int BITS>
__global__ void prepack_onnx_w_kernel(const uint8_t* __restrict__ qw, int G, int nblk,
                                      uint8_t* __restrict__ W) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblk * 32) return;
    const int lane = static_cast<int>(idx & 31);
    const long long tile = idx >> 5;                 // G * nblk + b
    const int b = static_cast<int>(tile % nblk);
    const int grp = static_cast<int>(tile / nblk);
    const int g = lane >> 2, t = lane & 3;
    const size_t row0 = static_cast<size_t>(grp) * 16 + g, row1 = row0 + 8;
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
        reinterpret_cast<uint4*>(W)[tile * 32 + lane] = v;
    } else {
        const uint8_t* r0 = qw + (row0 * nblk + b) * 16;
        const uint8_t* r1 = qw + (row1 * nblk + b) * 16;
        auto nib = [](const uint8_t* r, int k) { return (r[k >> 1] >> (4 * (k & 1))) & 15u; };
        uint2 v;
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w0 |= nib(r0, 4 * t + j) << (8 * j);
            w0 |= nib(r1, 4 * t + j) << (8 * j + 4);
            w1 |= nib(r0, 16 + 4 * t + j) << (8 * j);
            w1 |= nib(r1, 16 + 4 * t + j) << (8 * j + 4);
        }
        v.x = w0;
        v.y = w1;
        reinterpret_cast<uint2*>(W)[tile * 32 + lane] = v;
    }
}

// Scales: out[(grp*nblk + b)*16 + 2g + h] = in[(16 grp + g + 8h) * nblk + b].
template <typename T>
__global__ void prepack_scales_kernel(const T* __restrict__ in, int G, int nblk, T* __restrict__ out) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblk * 16) return;
    const int i = static_cast<int>(idx & 15);
    const long long tile = idx >> 4;
    const int b = static_cast<int>(tile % nblk);
    const int grp = static_cast<int>(tile / nblk);
    const size_t row = static_cast<size_t>(grp) * 16 + (i >> 1) + 8 * (i & 1);
    out[idx] = in[row * nblk + b];
}

// Zero points: Z[(grp*nblkZ + b)*8 + g] = zp(row g) | zp(row g+8) << 4, read
// from the packed MatMulNBits qzeros [N][ceil(nblk/2)] (low nibble = even block).
__global__ void prepack_zp_kernel(const uint8_t* __restrict__ qz, int G, int nblk, int nblkZ,
                                  uint8_t* __restrict__ Z) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblkZ * 8) return;
    const int g = static_cast<int>(idx & 7);
    const long long tile = idx >> 3;
    const int b = static_cast<int>(tile % nblkZ);
    const int grp = static_cast<int>(tile / nblkZ);
    if (b >= nblk) {
        Z[idx] = 0x88;   // padding block, never used
        return;
    }
    const int packed = (nblk + 1) / 2;
    auto zp = [&](size_t row) { return (qz[row * packed + b / 2] >> (4 * (b & 1))) & 15; };
    const size_t row0 = static_cast<size_t>(grp) * 16 + g;
    Z[idx] = static_cast<uint8_t>(zp(row0) | (zp(row0 + 8) << 4));
}

// Legacy VNNI layout (kernel/quantized_matmul.cpp:480-499): B [ntiles][nblk][8][32|64],
// scales fp32 [ntiles][nblk][16], zp s8 [ntiles][nblk][16].  The 16-column VNNI
// tile is one 16-row group here.  INT4 value (col, k) is nibble k%2 of byte
// g4*32 + col*2 + (k%4)/2 with g4 = (k%32)/4; INT8 byte (col, k) = B[g4*64 + col*4 + k%4].
template <int BITS>
__global__ void prepack_vnni_w_kernel(const uint8_t* __restrict__ B, int G, int nblk,
                                      uint8_t* __restrict__ W) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblk * 32) return;
    const int lane = static_cast<int>(idx & 31);
    const long long tile = idx >> 5;
    const int g = lane >> 2, t = lane & 3;
    constexpr int GB = BITS == 8 ? 64 : 32;
    const uint8_t* src = B + tile * 8 * GB;
    auto val = [&](int col, int k) -> uint32_t {
        const int g4 = k >> 2, j = k & 3;
        if (BITS == 8) return src[g4 * 64 + col * 4 + j];                 // already q - 128
        return (src[g4 * 32 + col * 2 + (j >> 1)] >> (4 * (j & 1))) & 15u;
    };
    if (BITS == 8) {
        uint4 v;
        uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w[0] |= val(g, 4 * t + j) << (8 * j);
            w[1] |= val(g + 8, 4 * t + j) << (8 * j);
            w[2] |= val(g, 16 + 4 * t + j) << (8 * j);
            w[3] |= val(g + 8, 16 + 4 * t + j) << (8 * j);
        }
        v.x = w[0]; v.y = w[1]; v.z = w[2]; v.w = w[3];
        reinterpret_cast<uint4*>(W)[tile * 32 + lane] = v;
    } else {
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w0 |= val(g, 4 * t + j) << (8 * j);
            w0 |= val(g + 8, 4 * t + j) << (8 * j + 4);
            w1 |= val(g, 16 + 4 * t + j) << (8 * j);
            w1 |= val(g + 8, 16 + 4 * t + j) << (8 * j + 4);
        }
        reinterpret_cast<uint2*>(W)[tile * 32 + lane] = make_uint2(w0, w1);
    }
}

__global__ void prepack_vnni_meta_kernel(const float* __restrict__ sc, const int8_t* __restrict__ zp,
                                         int G, int nblk, int nblkZ, float* __restrict__ S,
                                         uint8_t* __restrict__ Z) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(G) * nblkZ * 16) return;
    const int i = static_cast<int>(idx & 15);
    const long long tile = idx >> 4;               // grp * nblkZ + b
    const int b = static_cast<int>(tile % nblkZ);
    const int grp = static_cast<int>(tile / nblkZ);
    const int col = (i >> 1) + 8 * (i & 1);
    if (b < nblk) {
        const size_t src = (static_cast<size_t>(grp) * nblk + b) * 16;
        S[src + i] = sc[src + col];
        if (Z && i < 8)
            Z[tile * 8 + i] = static_cast<uint8_t>((zp[src + i] & 15) | ((zp[src + i + 8] & 15) << 4));
    } else if (Z && i < 8) {
        Z[tile * 8 + i] = 0x88;
    }
}

static unsigned grid_for(long long n, int threads) {
    return static_cast<unsigned>((n + threads - 1) / threads);
}

cudaError_t launch_prepack_onnx(Weight* w, const uint8_t* d_qw, const void* d_scales,
                                const uint8_t* d_qzeros, cudaStream_t stream) {
    const int T = 256;
    const long long lanes = static_cast<long long>(w->G) * w->nblk * 32;
    if (w->bits == 8)
        prepack_onnx_w_kernel<8><<<grid_for(lanes, T), T, 0, stream>>>(d_qw, w->G, w->nblk, w->W);
    else
        prepack_onnx_w_kernel<4><<<grid_for(lanes, T), T, 0, stream>>>(d_qw, w->G, w->nblk, w->W);
    const long long sn = static_cast<long long>(w->G) * w->nblk * 16;
    if (w->scale_half)
        prepack_scales_kernel<uint16_t><<<grid_for(sn, T), T, 0, stream>>>(
            static_cast<const uint16_t*>(d_scales), w->G, w->nblk, static_cast<uint16_t*>(w->S));
    else
        prepack_scales_kernel<float><<<grid_for(sn, T), T, 0, stream>>>(
            static_cast<const float*>(d_scales), w->G, w->nblk, static_cast<float*>(w->S));
    if (w->has_zp) {
        const long long zn = static_cast<long long>(w->G) * w->nblkZ * 8;
        prepack_zp_kernel<<<grid_for(zn, T), T, 0, stream>>>(d_qzeros, w->G, w->nblk, w->nblkZ, w->Z);
    }
    return cudaGetLastError();
}

cudaError_t launch_prepack_vnni(Weight* w, const uint8_t* d_B, const float* d_scales,
                                const int8_t* d_zp, cudaStream_t stream) {
    const int T = 256;
    const long long lanes = static_cast<long long>(w->G) * w->nblk * 32;
    if (w->bits == 8)
        prepack_vnni_w_kernel<8><<<grid_for(lanes, T), T, 0, stream>>>(d_B, w->G, w->nblk, w->W);
    else
        prepack_vnni_w_kernel<4><<<grid_for(lanes, T), T, 0, stream>>>(d_B, w->G, w->nblk, w->W);
    const long long mn = static_cast<long long>(w->G) * w->nblkZ * 16;
    prepack_vnni_meta_kernel<<<grid_for(mn, T), T, 0, stream>>>(
        d_scales, d_zp, w->G, w->nblk, w->nblkZ, static_cast<float*>(w->S), w->has_zp ? w->Z : nullptr);
    return cudaGetLastError();
}

}  // namespace ql
