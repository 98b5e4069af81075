// ql_gemmw.cu -- INT4 prefill on pre-expanded FP16 operands: per call, the
// packed weights are dequantized once to FP16 (q - zp) tiles in the caller's
// workspace and the activations are quantized straight to FP16 planes; a
// tcgen05 kind::f16 GEMM then streams both with 1-D bulk copies and spends its
// CUDA cores only on the reference's per-block FP32 rescale.
//
// Computes C[m, n] = i4_matmul(A)[m, n] (kernel/quantized_matmul.cpp:270-318,
// the 8-row chunk loop :545-549) for INT4 weights with fp16 scales, bit-
// identical to the reference, with the numerics of ql_gemm16.cu:
//   two-pass:    q16 = 256*h + l, D = sum h*w + sum (l/256)*w = cs/256 (exact),
//                t = RN(D * (256*bscale)) = RN((float)cs * bscale)
//   single-pass: D = sum q8*w = cs (exact, |cs| < 2^16), t = RN(D * bscale)
//   acc = fma(ascale, t, acc) in ascending block order (:311-315).
// h in [-128, 127], l/256 (l in [0, 255]), q8 in [-127, 127] and w = q - zp in
// [-15, 15] are exact FP16 values, and every partial sum of D stays within the
// 24 significant bits of the tensor core's FP32 accumulator.
//
// Why a separate path.  ql_gemm16.cu unpacks the INT4 weights and converts the
// INT8 activation planes to FP16 inside the GEMM, once per 128x128 tile: at
// M = 2048 every weight tile is unpacked 16 times, and those CUDA-core roles
// bound the kernel.  Here the unpack happens once per call (an HBM pass of
// 2.25 bytes written per weight), the activation planes arrive in FP16, and
// the GEMM's only CUDA-core work is the epilogue.
//
// Operands in the workspace (all records in the canonical K-major SWIZZLE_NONE
// tcgen05 layout of ql_tcgen05.cuh, so a stage is a plain byte copy):
//   weights  [n_tiles][nblk][WREC]: 128 rows x 32 k FP16 (q - zp) as
//            [4 K columns of 8 k][16 groups of 8 rows][8 rows x 16 B] (8 KB),
//            then 128 fp32 scales 256*bscale (two-pass) or bscale; rows past
//            N are zero.
//   acts     [m_tiles][nblk][AREC]: per plane (h, then l/256; or q8) two
//            K halves of [2 K columns][16 groups of 8 tokens][8 tokens x 16 B]
//            (4 KB each), then 128 fp32 activation scales; tokens past M are zero.
//
// Kernel: persistent CTAs (one per SM) walk 128-row x 128-token tiles, token
// tile fastest (concurrent CTAs share a weight tile through L2).  Warps:
//   0     producer: per stage of BPS blocks one bulk copy of the weight records
//         and one of the activation records (no multicast)
//   1-2   MMA: two issuing warps take alternate stages; lane 0 issues per block
//         4 (two-pass) or 2 MMAs of 128x128x16 into one of 4 accumulator slots
//         of 128 columns (warp 1 owns the TMEM allocation).  Measured on B200:
//         an mbarrier wait (even on a completed phase) or a shared-memory
//         access in the issuing warp does not proceed until that warp's queued
//         MMAs have finished, so one issuer that waits once per block (the
//         per-block hand-off to the epilogue is the reference's per-block
//         rescale) drains the tensor pipe every block: 506 cycles per block
//         instead of 273.  With two issuers, each drains only its own previous
//         stage while the other's MMAs run (256 cycles per block).  Each issuer
//         does all of a stage's waits before issuing any of its MMAs.
//   3     scales: copies each block's 1 KB of scales from the stage into the
//         scale ring the epilogue reads, then fences its generic reads of the
//         stage against the stage's next bulk copy (off the issuing warps,
//         whose own proxy fence would stall them the same way).
//   4-11  epilogue: warp w reads TMEM lanes 32*(w%4).. (its 32 weight rows) and
//         64 token columns per block with two 32-column loads and one wait
//         (no shared-memory access between a load and its wait: a warp's
//         shared-memory accesses wait for its outstanding tcgen05.ld), releases
//         the slot, and runs the FP32 chain in registers, reading the block's
//         activation scales 16 columns at a time.  (Tried and slower on B200:
//         16 epilogue warps of 32 columns -- the 96-register cap spills --
//         and loading the next half while rescaling the current one, whose
//         scale reads then waited for that load.)
// Every wait is bounded (the device wait limit) and sets the device error
// word; on a failure all roles stop, bulk copies and MMAs in flight are
// drained (bounded) and TMEM is freed.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include "ql_common.cuh"
#include "ql_internal.h"
#include "ql_quant.cuh"
#include "ql_tcgen05.cuh"

namespace ql {

namespace {

constexpr int W_T = 128;                     // weight rows per tile (MMA M)
constexpr int A_T = 128;                     // tokens per tile (MMA N)
constexpr int W_TILE = W_T * 32 * 2;         // FP16 weight tile of one block (8 KB)
constexpr int N_EPI = 8;
constexpr int N_WARPS = 4 + N_EPI;
constexpr int W_SC = 3;                      // scale warp; warps 1 and 2 issue MMAs, 4.. are the epilogue
constexpr int E_COLS = 64;                   // token columns per epilogue thread
constexpr int N_ACC = 4;                     // TMEM accumulator slots of 128 columns
constexpr int N_SC = 8;                      // scale ring (1 KB per block)
constexpr int SC_BYTES = 1024;
constexpr uint32_t TMEM_NCOLS = 512;

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 8 INT4 weights of one record word (byte i = q(row g, k_i) | q(row g+8, k_i) << 4)
// -> exact FP16 (q - zp) of rows g and g+8, k_0..k_3 each as two half2 words.
// 0x6400 | q is the FP16 value 1024 + q; 0x6400 | 16q is 1024 + 16q, scaled by
// 1/16 in the FMA.  zg / zg8 are the half2 patterns of 1024 + zp and
// -(64 + zp) for rows g and g+8.
__device__ __forceinline__ void nib8_to_f16(uint32_t x, uint32_t zg, uint32_t zg8, uint2& rg, uint2& rg8) {
    const uint32_t y01 = __byte_perm(x, 0, 0x0100);
    const uint32_t y23 = __byte_perm(x, 0, 0x0302);
    constexpr uint32_t SIXTEENTH = 0x2C002C00u;
    rg = make_uint2(hsub2_bits((y01 & 0x000F000Fu) | 0x64006400u, zg),
                    hsub2_bits((y23 & 0x000F000Fu) | 0x64006400u, zg));
    rg8 = make_uint2(hfma2_bits((y01 & 0x00F000F0u) | 0x64006400u, SIXTEENTH, zg8),
                     hfma2_bits((y23 & 0x00F000F0u) | 0x64006400u, SIXTEENTH, zg8));
}

}  // namespace

// ---------------------------------------------------------------- weight dequant
// One warp per weight record (16 rows x 32 k): lane 4g + t holds rows g and
// g + 8 at k 4t..4t+3 and 16+4t..16+4t+3 (ql_internal.h), which land at
// (t/2)*2048 + (2gg)*128 + g*16 + (t%2)*8 in the tile (gg = the record's row
// group within its tile), row g + 8 one 8-row group (128 B) on, k + 16 two
// K columns (4096 B) on.  Row groups past the last one of the final tile are
// written as zeros.
template <bool ZP>
__global__ void __launch_bounds__(256) dequant_w16_kernel(const uint8_t* __restrict__ W, int G, int nblk,
                                                          int n_tiles, bool two_pass, uint8_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();                 // the workspace may still be read by the previous grid
    constexpr int TB = 256, SB = 32, ZB = ZP ? 16 : 0, REC = TB + SB + ZB;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int o_lane = (t >> 1) * 2048 + g * 16 + (t & 1) * 8;
    const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    const long long total = static_cast<long long>(n_tiles) * 8 * nblk;     // (tile row group, block)
    const float sfac = two_pass ? 256.0f : 1.0f;
    for (long long i = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); i < total;
         i += nwarps) {
        const int b = static_cast<int>(i % nblk);
        const long long rg = i / nblk;                  // row group over the padded tiles
        const int nt = static_cast<int>(rg >> 3), gg = static_cast<int>(rg & 7);
        uint8_t* tile = out + (static_cast<size_t>(nt) * nblk + b) * WREC16;
        uint8_t* o = tile + gg * 256 + o_lane;
        float* sc = reinterpret_cast<float*>(tile + W_TILE) + gg * 16;
        uint2 r0 = make_uint2(0, 0), r1 = r0, r2 = r0, r3 = r0;
        float s = 0.0f;
        if (rg < G) {
            const uint8_t* rec = W + (static_cast<size_t>(rg) * nblk + b) * REC;
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(rec + lane * 8));
            uint32_t zg = 0x64086408u, zg8 = 0xD480D480u;        // zp = 8
            if (ZP) {
                const uint32_t z = rec[TB + SB + g];
                zg = (0x6400u | (z & 15u)) * 0x00010001u;
                zg8 = (0xD400u | ((z >> 4) << 4)) * 0x00010001u;
            }
            nib8_to_f16(v.x, zg, zg8, r0, r1);
            nib8_to_f16(v.y, zg, zg8, r2, r3);
            if (lane < 16) {
                // row lane of the group: record entry 2*(lane%8) + lane/8 (2g = row g, 2g+1 = row g+8)
                const int e = 2 * (lane & 7) + (lane >> 3);
                s = __half2float(reinterpret_cast<const __half*>(rec + TB)[e]) * sfac;   // exact
            }
        }
        *reinterpret_cast<uint2*>(o) = r0;
        *reinterpret_cast<uint2*>(o + 128) = r1;
        *reinterpret_cast<uint2*>(o + 4096) = r2;
        *reinterpret_cast<uint2*>(o + 4096 + 128) = r3;
        if (lane < 16) sc[lane] = s;
    }
}

// ---------------------------------------------------------------- activation quantizer (FP16 planes)
// One thread per (token, block): the reference quantizer (ql_quant.cuh) and the
// planes written as FP16: h = hi - 128 and l/256 (two-pass) or q8 (single-pass),
// at plane p, K half kh, K column c (8 k each) and token tt of the tile:
//   p*8192 + kh*4096 + c*2048 + (tt/8)*128 + (tt%8)*16.
template <bool HP, int PRO>
__global__ void __launch_bounds__(256) quantize_f16_kernel(const float* __restrict__ A, int lda, int M, int K,
                                                           int m_tiles, uint8_t* __restrict__ out, NormArgs nrm) {
    pdl_launch_dependents();
    pdl_wait();
    const int nblk = K / BLOCK_K;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(m_tiles) * A_T * nblk) return;
    const int m = static_cast<int>(idx / nblk);
    const int b = static_cast<int>(idx % nblk);
    const int mt = m >> 7, tt = m & 127;
    constexpr int AREC = HP ? AREC16_HP : AREC16_SP;
    constexpr int PLANES = HP ? 2 : 1;
    uint8_t* rec = out + (static_cast<size_t>(mt) * nblk + b) * AREC;
    uint8_t* o = rec + (tt >> 3) * 128 + (tt & 7) * 16;
    float* scale = reinterpret_cast<float*>(rec + PLANES * 8192) + tt;
    if (m >= M) {
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int c = 0; c < 4 * PLANES; ++c) *reinterpret_cast<uint4*>(o + c * 2048) = z;
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
#pragma unroll
    for (int c = 0; c < 4; ++c) {                       // 8 k per 16-byte row: K column c of the block
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half hv[2], lv[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                int q = to_int_like_lrint(__fmul_rn(v[8 * c + 2 * j + e], inv));
                q = q > IMAX ? IMAX : (q < -IMAX ? -IMAX : q);
                if (HP) {
                    const int u = q + 32768;
                    hv[e] = __int2half_rn((u >> 8) - 128);                             // exact
                    lv[e] = __hmul(__int2half_rn(u & 0xFF), __float2half_rn(0.00390625f));   // l/256, exact
                } else {
                    lv[e] = __int2half_rn(q);                                          // exact
                }
            }
            hw[j] = static_cast<uint32_t>(__half_as_ushort(hv[0])) |
                    (static_cast<uint32_t>(__half_as_ushort(hv[1])) << 16);
            lw[j] = static_cast<uint32_t>(__half_as_ushort(lv[0])) |
                    (static_cast<uint32_t>(__half_as_ushort(lv[1])) << 16);
        }
        const int off = (c >> 1) * 4096 + (c & 1) * 2048;
        if (HP) {
            *reinterpret_cast<uint4*>(o + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(o + 8192 + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        } else {
            *reinterpret_cast<uint4*>(o + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
    }
}

// ---------------------------------------------------------------- GEMM
struct GemmWParams {
    const uint8_t* Wd;       // weight records [n_tiles][nblk][WREC16]
    const uint8_t* Ad;       // activation records [m_tiles][nblk][arec]
    float* C;
    int32_t* CS;
    int* err;
    int M, N, nblk, ldc;
    int m_tiles, n_tiles, tiles;
    int arec;                // activation record bytes (two- or single-pass)
    int BPS, STAGES;
    uint32_t stage_bytes, off_sc, off_stages;
};

template <bool HP, bool OUT_CS>
__global__ void __launch_bounds__(N_WARPS * 32, 1) gemmw_kernel(const GemmWParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    uint64_t* st_full = bars;
    uint64_t* st_empty = st_full + p.STAGES;
    uint64_t* acc_full = st_empty + p.STAGES;
    uint64_t* acc_empty = acc_full + N_ACC;
    uint64_t* sc_full = acc_empty + N_ACC;
    uint64_t* sc_empty = sc_full + N_SC;
    uint64_t* drain = sc_empty + N_SC;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
    uint8_t* sc_ring = smem + p.off_sc;          // per block: 128 f32 weight scales, then 128 f32 ascale
    uint8_t* stages = smem + p.off_stages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int spt = (p.nblk + p.BPS - 1) / p.BPS;        // stages per tile
    const uint32_t w_part = static_cast<uint32_t>(p.BPS) * WREC16;   // weight records inside a stage

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.STAGES; ++s) {
            mbar_init(smem_u32(&st_full[s]), 1);
            mbar_init(smem_u32(&st_empty[s]), 2);      // the MMAs' commit and the scale warp
        }
        for (int k = 0; k < N_ACC; ++k) {
            mbar_init(smem_u32(&acc_full[k]), 1);
            mbar_init(smem_u32(&acc_empty[k]), N_EPI);
        }
        for (int k = 0; k < N_SC; ++k) {
            mbar_init(smem_u32(&sc_full[k]), 1);
            mbar_init(smem_u32(&sc_empty[k]), N_EPI);
        }
        mbar_init(smem_u32(drain), 2);             // one commit per issuing warp
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(TMEM_NCOLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();   // the next kernel waits for this grid before touching its data

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        int si = 0;
        if (lane == 0) pdl_wait();                    // both operands come from the previous grids
        __syncwarp();
        for (int tile = blockIdx.x; tile < p.tiles && __shfl_sync(0xffffffffu, *abort_flag, 0) == 0;
             tile += gridDim.x) {
            const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
            for (int ks = 0; ks < spt; ++ks, ++si) {
                const int s = si % p.STAGES;
                if (si >= p.STAGES &&
                    !warp_wait(smem_u32(&st_empty[s]), ((si / p.STAGES) - 1) & 1, p.err, abort_flag))
                    break;
                if (lane == 0) {
                    const int b0 = ks * p.BPS;
                    const int nb = min(p.BPS, p.nblk - b0);
                    const uint32_t base = smem_u32(stages + static_cast<size_t>(s) * p.stage_bytes);
                    const uint32_t full = smem_u32(&st_full[s]);
                    mbar_arrive_expect_tx(full, static_cast<uint32_t>(nb) * (WREC16 + p.arec));
                    bulk_g2s(base, p.Wd + (static_cast<size_t>(nt) * p.nblk + b0) * WREC16, nb * WREC16, full);
                    bulk_g2s(base + w_part, p.Ad + (static_cast<size_t>(mt) * p.nblk + b0) * p.arec, nb * p.arec,
                             full);
                }
                __syncwarp();
            }
        }
        // drain: every stage this warp filled must have landed before exit
        const int issued = si;
        for (int k = std::max(0, issued - p.STAGES); k < issued; ++k)
            mbar_wait(smem_u32(&st_full[k % p.STAGES]), (k / p.STAGES) & 1, p.err);
    } else if (warp == 1 || warp == 2) {
        // ------------------------------------------------------------ MMA issuers
        // Warp 1 takes the even stages of the CTA's stage sequence, warp 2 the odd ones.
        constexpr uint32_t idesc = make_idesc_f16(W_T, A_T);
        const int parity = warp - 1;
        int si = 0, bi = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            for (int ks = 0; ks < spt && ok; ++ks, ++si) {
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                const int bi0 = bi;
                bi += nb;
                if ((si & 1) != parity) continue;
                const int s = si % p.STAGES;
                // every wait of the stage before its first MMA
                if (!(ok = warp_wait(smem_u32(&st_full[s]), (si / p.STAGES) & 1, p.err, abort_flag))) break;
                for (int j = 0; j < nb && ok; ++j) {
                    const int b = bi0 + j;
                    if (b >= N_ACC)
                        ok = warp_wait(smem_u32(&acc_empty[b % N_ACC]), ((b / N_ACC) - 1) & 1, p.err, abort_flag);
                }
                if (!ok) break;
                tc_fence_after();
                if (lane == 0) {
                    const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
                    for (int j = 0; j < nb; ++j) {
                        const uint32_t a0 = smem_u32(st + j * WREC16), b0 = smem_u32(st + w_part + j * p.arec);
                        const uint32_t d = tmem + ((bi0 + j) % N_ACC) * A_T;
                        const uint64_t da0 = make_smem_desc(a0, 2048, 128);
                        const uint64_t da1 = make_smem_desc(a0 + 4096, 2048, 128);
                        mma_f16(d, da0, make_smem_desc(b0, 2048, 128), idesc, 0);
                        mma_f16(d, da1, make_smem_desc(b0 + 4096, 2048, 128), idesc, 1);
                        if (HP) {
                            mma_f16(d, da0, make_smem_desc(b0 + 8192, 2048, 128), idesc, 1);
                            mma_f16(d, da1, make_smem_desc(b0 + 12288, 2048, 128), idesc, 1);
                        }
                        mma_commit(smem_u32(&acc_full[(bi0 + j) % N_ACC]));
                    }
                    mma_commit(smem_u32(&st_empty[s]));
                }
                __syncwarp();
            }
        }
        // drain: all MMAs issued by this warp's lane 0 complete before TMEM is freed
        if (lane == 0) mma_commit(smem_u32(drain));
        __syncwarp();
        mbar_wait(smem_u32(drain), 0, p.err);
    } else if (warp == W_SC) {
        // ------------------------------------------------------------ scales
        int si = 0, bi = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            for (int ks = 0; ks < spt && ok; ++ks, ++si) {
                const int s = si % p.STAGES;
                if (!(ok = warp_wait(smem_u32(&st_full[s]), (si / p.STAGES) & 1, p.err, abort_flag))) break;
                const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                for (int j = 0; j < nb; ++j, ++bi) {
                    const int sc = bi % N_SC;
                    if (bi >= N_SC &&
                        !(ok = warp_wait(smem_u32(&sc_empty[sc]), ((bi / N_SC) - 1) & 1, p.err, abort_flag)))
                        break;
                    // 16 B of the weight scales and 16 B of the activation scales per lane
                    uint4* dsc = reinterpret_cast<uint4*>(sc_ring + sc * SC_BYTES);
                    dsc[lane] = *reinterpret_cast<const uint4*>(st + j * WREC16 + W_TILE + lane * 16);
                    dsc[32 + lane] =
                        *reinterpret_cast<const uint4*>(st + w_part + j * p.arec + (HP ? 16384 : 8192) + lane * 16);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&sc_full[sc]));
                }
                if (!ok) break;
                fence_proxy_async_smem();            // this warp's reads of the stage before its next bulk copy
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&st_empty[s]));
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int e = warp - 4;
        const int q = warp & 3;                           // TMEM lane quarter (hardware rule: warp % 4)
        const int cq = e >> 2;                            // token columns E_COLS*cq ..
        const int row = q * 32 + lane;                    // weight row within the tile
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + cq * E_COLS;
        int bi = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
            const int n = nt * W_T + row;
            uint64_t acc[E_COLS / 2];                     // E_COLS token columns as f32x2 pairs
#pragma unroll
            for (int i = 0; i < E_COLS / 2; ++i) acc[i] = 0;
            for (int kb = 0; kb < p.nblk && ok; ++kb, ++bi) {
                const int ac = bi % N_ACC, sc = bi % N_SC;
                if (!(ok = warp_wait(smem_u32(&sc_full[sc]), (bi / N_SC) & 1, p.err, abort_flag))) break;
                if (!(ok = warp_wait(smem_u32(&acc_full[ac]), (bi / N_ACC) & 1, p.err, abort_flag))) break;
                tc_fence_after();
                const float* scs = reinterpret_cast<const float*>(sc_ring + sc * SC_BYTES);
                const uint32_t taddr = lane_base + ac * A_T;
                if constexpr (OUT_CS) {
                    // block sums [M][N][nblk] = 256 * D (two-pass) or D (exact): a checking output
#pragma unroll 1
                    for (int cc = 0; cc < E_COLS / 16; ++cc) {
                        uint32_t v[16];
                        tmem_ld16(taddr + cc * 16, v);
                        tmem_wait_ld();
                        const int m0 = mt * A_T + cq * E_COLS + cc * 16;
                        int32_t* dst = p.CS + (static_cast<size_t>(m0) * p.N + n) * p.nblk + kb;
#pragma unroll
                        for (int k = 0; k < 16; ++k) {
                            const int32_t cs = __float2int_rn(__uint_as_float(v[k]) * (HP ? 256.0f : 1.0f));
                            if (m0 + k < p.M && n < p.N) *dst = cs;
                            dst += static_cast<size_t>(p.N) * p.nblk;
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(smem_u32(&acc_empty[ac]));
                        mbar_arrive(smem_u32(&sc_empty[sc]));
                    }
                } else {
                    const float wsc = scs[row];                   // 256*bscale (two-pass) or bscale; 0 past N
                    const uint64_t ws2 = f2_pack(wsc, wsc);
                    const float* ascale = scs + 128 + cq * E_COLS;
                    // the whole slot in one wait (a warp's shared-memory accesses wait for
                    // its outstanding tcgen05.ld, so the scale reads come after it)
                    uint32_t v[E_COLS];
                    tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
                    tmem_ld32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&acc_empty[ac]));
                    // 16 columns at a time: their 4 scale loads issue back to back, so
                    // one shared-memory latency covers 16 outputs
#pragma unroll
                    for (int c0 = 0; c0 < E_COLS; c0 += 16) {
                        float4 a4[4];
#pragma unroll
                        for (int g = 0; g < 4; ++g) a4[g] = lds_f4(ascale + c0 + 4 * g);
#pragma unroll
                        for (int g = 0; g < 4; ++g) {
                            const int k = c0 + 4 * g;
                            const uint64_t d0 = i2_pack(static_cast<int32_t>(v[k]), static_cast<int32_t>(v[k + 1]));
                            const uint64_t d1 = i2_pack(static_cast<int32_t>(v[k + 2]), static_cast<int32_t>(v[k + 3]));
                            acc[k >> 1] = f2_fma(f2_pack(a4[g].x, a4[g].y), f2_mul(d0, ws2), acc[k >> 1]);
                            acc[(k >> 1) + 1] = f2_fma(f2_pack(a4[g].z, a4[g].w), f2_mul(d1, ws2), acc[(k >> 1) + 1]);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&sc_empty[sc]));
                }
            }
            if (!ok || OUT_CS) continue;
            // C[m, n] for this thread's token columns (lanes = consecutive n)
            if (n < p.N) {
#pragma unroll
                for (int i = 0; i < E_COLS / 2; ++i) {
                    const int m = mt * A_T + cq * E_COLS + 2 * i;
                    const float2 v = f2_unpack(acc[i]);
                    if (m < p.M) p.C[static_cast<size_t>(m) * p.ldc + n] = v.x;
                    if (m + 1 < p.M) p.C[static_cast<size_t>(m + 1) * p.ldc + n] = v.y;
                }
            }
        }
    }

    // every role is done (or aborted): free TMEM
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TMEM_NCOLS) : "memory");
}

// ------------------------------------------------------------------ host side

int* device_error_word();   // ql_api.cu

namespace {

template <typename... Args>
cudaError_t launch_pdl_ex(void (*kern)(Args...), unsigned grid, unsigned threads, size_t smem, cudaStream_t stream,
                          Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

int num_sms() {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (sms[dev] == 0) {
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (sms[dev] <= 0) sms[dev] = 148;
    }
    return sms[dev];
}

size_t align1k(size_t x) { return (x + 1023) & ~size_t(1023); }

template <bool HP, bool OUT_CS>
cudaError_t gemmw_launch(const GemmWParams& p0, cudaStream_t stream) {
    GemmWParams p = p0;
    p.BPS = 2;
    p.stage_bytes = static_cast<uint32_t>(align1k(static_cast<size_t>(p.BPS) * (WREC16 + p.arec)));
    const uint32_t bar_bytes = 1024;                        // barriers, abort flag, TMEM address
    p.off_sc = bar_bytes;
    p.off_stages = p.off_sc + N_SC * SC_BYTES;
    p.STAGES = 4;
    while (p.STAGES > 2 && p.off_stages + static_cast<size_t>(p.STAGES) * p.stage_bytes > 227 * 1024) --p.STAGES;
    const size_t smem = p.off_stages + static_cast<size_t>(p.STAGES) * p.stage_bytes;
    const size_t bars = (2 * p.STAGES + 2 * N_ACC + 2 * N_SC + 1) * 8 + 16;
    if (smem > 227 * 1024 || bars > bar_bytes || (p.arec % 16) || (WREC16 % 16) || (p.off_stages % 1024) ||
        (p.stage_bytes % 1024))
        return cudaErrorInvalidConfiguration;
    auto kern = gemmw_kernel<HP, OUT_CS>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    return launch_pdl_ex(kern, static_cast<unsigned>(std::min(p.tiles, num_sms())), N_WARPS * 32, smem, stream, p);
}

}  // namespace

bool gemmw_supports(const Weight* w) { return w->bits == 4 && w->scale_half; }

size_t gemmw_act_bytes(int M, int nblk, bool hi_prec) {
    const size_t m_tiles = (static_cast<size_t>(M) + A_T - 1) / A_T;
    return align1k(m_tiles * nblk * (hi_prec ? AREC16_HP : AREC16_SP));
}

size_t gemmw_weight_bytes(const Weight* w) {
    const size_t n_tiles = (static_cast<size_t>(w->N) + W_T - 1) / W_T;
    return align1k(n_tiles * w->nblk * WREC16);
}

cudaError_t launch_dequant_w16(const Weight* w, bool hi_prec, uint8_t* out, cudaStream_t stream) {
    const int n_tiles = (w->N + W_T - 1) / W_T;
    const long long warps = static_cast<long long>(n_tiles) * 8 * w->nblk;
    const unsigned grid = static_cast<unsigned>(std::min<long long>((warps + 7) / 8, 16LL * num_sms()));
    if (w->has_zp)
        return launch_pdl_ex(dequant_w16_kernel<true>, grid, 256, 0, stream, static_cast<const uint8_t*>(w->W), w->G,
                             w->nblk, n_tiles, hi_prec, out);
    return launch_pdl_ex(dequant_w16_kernel<false>, grid, 256, 0, stream, static_cast<const uint8_t*>(w->W), w->G,
                         w->nblk, n_tiles, hi_prec, out);
}

cudaError_t launch_quantize_f16(const float* A, int lda, int M, int K, bool hi_prec, uint8_t* out,
                                cudaStream_t stream, const NormArgs* norm) {
    const int m_tiles = (M + A_T - 1) / A_T;
    const long long total = static_cast<long long>(m_tiles) * A_T * (K / BLOCK_K);
    const unsigned grid = static_cast<unsigned>((total + 255) / 256);
    const NormArgs n = norm ? *norm : NormArgs{};
    if (norm) {
        if (hi_prec) return launch_pdl_ex(quantize_f16_kernel<true, PRO_NORM>, grid, 256, 0, stream, A, lda, M, K, m_tiles, out, n);
        return launch_pdl_ex(quantize_f16_kernel<false, PRO_NORM>, grid, 256, 0, stream, A, lda, M, K, m_tiles, out, n);
    }
    if (hi_prec) return launch_pdl_ex(quantize_f16_kernel<true, PRO_NONE>, grid, 256, 0, stream, A, lda, M, K, m_tiles, out, n);
    return launch_pdl_ex(quantize_f16_kernel<false, PRO_NONE>, grid, 256, 0, stream, A, lda, M, K, m_tiles, out, n);
}

cudaError_t launch_gemmw(const Weight* w, const uint8_t* wd, const uint8_t* ad, int M, bool hi_prec, float* C,
                         int ldc, int32_t* cs, cudaStream_t stream) {
    GemmWParams p = {};
    p.Wd = wd;
    p.Ad = ad;
    p.C = C;
    p.CS = cs;
    p.err = device_error_word();
    p.M = M;
    p.N = w->N;
    p.nblk = w->nblk;
    p.ldc = ldc;
    p.m_tiles = (M + A_T - 1) / A_T;
    p.n_tiles = (w->N + W_T - 1) / W_T;
    p.tiles = p.m_tiles * p.n_tiles;
    p.arec = hi_prec ? AREC16_HP : AREC16_SP;
    if (hi_prec) return cs ? gemmw_launch<true, true>(p, stream) : gemmw_launch<true, false>(p, stream);
    return cs ? gemmw_launch<false, true>(p, stream) : gemmw_launch<false, false>(p, stream);
}

}  // namespace ql
