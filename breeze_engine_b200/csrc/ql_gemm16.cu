// ql_gemm16.cu -- INT4 prefill GEMM (M > 64 tokens) on tcgen05 kind::f16 tensor
// cores with exact integer-valued operands.
//
// Computes C[m, n] = i4_matmul(A)[m, n] (kernel/quantized_matmul.cpp:270-318,
// the 8-row chunk loop :545-549) for INT4 weights with fp16 scales and
// two-pass INT16 activations, bit-identical to the reference.
//
// Numerics.  q16 = 256*h + l with h = hi - 128 in [-128, 127] and l in
// [0, 255]; w = q - zp in [-15, 15].  All of h, l/256 and w are exact FP16
// values, so per 32-wide block ONE accumulator
//     D = sum_k h_k*w_k + sum_k (l_k/256)*w_k = cs / 256
// is an exact multiple of 2^-8 with |D| < 2^16: every partial sum fits the 24
// significant bits of FP32, so the tensor core's FP32 accumulation (which keeps
// at least 24 bits aligned to the largest term -- checked on B200 against
// worst-case magnitudes, cancellation and both accumulation orders, and by the
// INT32 block-sum tests) adds without rounding.  The epilogue then needs no
// int->float conversion:
//     t   = RN(D * (256*bscale))  ==  RN((float)cs * bscale)   (256*bscale exact)
//     acc = fma(ascale, t, acc)                                 (ascending blocks)
// which is the reference's chain (kernel/quantized_matmul.cpp:311-315).
// |cs| <= 32*32767*15 < 2^24, so (float)cs is exact in the reference too.
//
// Compared with the kind::i8 kernel (ql_gemm.cu) this halves the TMEM
// footprint per block (one accumulator instead of hi|lo, so four slots are in
// flight), halves the TMEM reads, needs no re-seeding stores, and needs 2 FP32
// operations per output per block instead of 4.  The tensor core does the same
// number of MACs (K = 64 per block at FP16 rate instead of 2 x 32 at INT8 rate).
//
// Data path: the activation records in HBM/L2 stay the INT8 planes of
// ql_quant.cu (GEMM_AREC bytes per 128-token tile and block, shared with the
// kind::i8 kernel); converter warps expand them to FP16 in shared memory, and
// unpack warps expand the INT4 weight records to FP16 (q - zp).  L2 -> SM
// traffic per tile is therefore that of the INT8 kernel.
//
// Tile: 128 weight rows (MMA M) x 128 tokens (MMA N); persistent CTAs (one per
// SM, 512 TMEM columns = 4 accumulator slots of 128 columns) walk the tiles
// with the token tile fastest.
//
// Warp roles (16 warps):
//   0       producer: 1-D bulk copies (no multicast) of the 8 row groups'
//           weight records and the token tile's activation record per stage
//   1       MMA issuer (one thread) and TMEM owner
//   2-3     weight unpack: INT4 records -> FP16 (q - zp), canonical K-major
//           [4 core-matrix K columns][16 row groups of 8][8 rows x 16 B]
//   4-11    epilogue: warp w reads TMEM lanes 32*(w%4).. (its 32 weight rows)
//           and token half (w-4)/4 (64 columns)
//   12-15   activation convert: INT8 hi/lo planes -> FP16 h and l/256 tiles
// Every mbarrier is waited phase by phase in order by its consumers; every wait
// is bounded (1 s) and sets the device error word; on any failure all roles
// stop, in-flight bulk copies and MMAs are drained (bounded) and TMEM is freed.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include "ql_common.cuh"
#include "ql_internal.h"
#include "ql_tcgen05.cuh"

namespace ql {

namespace {

constexpr int T_N = 128;                 // weight rows per tile (MMA M)
constexpr int T_M = 128;                 // tokens per tile (MMA N)
constexpr int T_G = T_N / 16;            // 16-row weight groups per tile
constexpr int N_UNP = 2;                 // weight unpack warps (4 row groups each)
constexpr int N_EPI = 8;                 // epilogue warps
constexpr int N_CONV = 4;                // activation convert warps
constexpr int N_WARPS = 2 + N_UNP + N_EPI + N_CONV;
constexpr int E_COLS = 64;               // token columns per epilogue thread
constexpr int A_BYTES = T_N * 32 * 2;    // FP16 weight tile per block: 128 rows x 32 k (8 KB)
constexpr int B_BYTES = T_M * 64 * 2;    // FP16 activation tiles per block: h and l/256, 128 x 32 k each (16 KB)
constexpr int N_ASLOT = 4;               // weight tile ring
constexpr int N_BSLOT = 3;               // activation tile ring
constexpr int N_ACC = 4;                 // TMEM accumulator slots of 128 columns
constexpr int N_SC = 8;                  // scale ring: 256*bscale of 128 rows + ascale of 128 tokens per block
constexpr int SC_BYTES = 1024;
constexpr uint32_t TMEM_NCOLS = 512;
constexpr int AREC16 = GEMM_AREC;        // activation bytes per (tile, block) (ql_internal.h)

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// 8 INT4 weights of one record word (byte i = q(row g, k_i) | q(row g+8, k_i) << 4)
// -> exact FP16 (q - zp): rows g and g+8, k_0..k_3 each as two half2 words.
// The bytes are first spread to (b0, b1) and (b2, b3) in the two halves of a
// word; 0x6400 | q is the FP16 value 1024 + q (low nibble), 0x6400 | 16q is
// 1024 + 16q (high nibble, scaled back by 1/16 in the same FMA).  zg / zg8 are
// the half2 bit patterns of 1024 + zp and 64 + zp for rows g and g+8.
__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ void nib8_to_f16(uint32_t x, uint32_t zg, uint32_t zg8, uint2& rg, uint2& rg8) {
    const uint32_t y01 = __byte_perm(x, 0, 0x0100);            // bytes b0 and b1 in the two halves
    const uint32_t y23 = __byte_perm(x, 0, 0x0302);
    constexpr uint32_t SIXTEENTH = 0x2C002C00u;                // 1/16 in both halves
    rg = make_uint2(hsub2_bits((y01 & 0x000F000Fu) | 0x64006400u, zg),
                    hsub2_bits((y23 & 0x000F000Fu) | 0x64006400u, zg));
    rg8 = make_uint2(hfma2_bits((y01 & 0x00F000F0u) | 0x64006400u, SIXTEENTH, zg8),
                     hfma2_bits((y23 & 0x00F000F0u) | 0x64006400u, SIXTEENTH, zg8));
}

// 4 bytes of the hi plane (stored as hi ^ 0x80) -> FP16 h = hi - 128:
// 0x6400 | hi is 1024 + hi, minus 1152 (0x6480).
__device__ __forceinline__ uint2 hi4_to_f16(uint32_t w) {
    const uint32_t u = w ^ 0x80808080u;
    return make_uint2(hsub2_bits(__byte_perm(u, 0x64646464u, 0x4140), 0x64806480u),
                      hsub2_bits(__byte_perm(u, 0x64646464u, 0x4342), 0x64806480u));
}

// 4 bytes of the lo plane -> FP16 l/256: 0x4400 | l is 4 + l/256, minus 4 (0x4400).
__device__ __forceinline__ uint2 lo4_to_f16(uint32_t w) {
    return make_uint2(hsub2_bits(__byte_perm(w, 0x44444444u, 0x4140), 0x44004400u),
                      hsub2_bits(__byte_perm(w, 0x44444444u, 0x4342), 0x44004400u));
}

__device__ __forceinline__ void sts_v2(uint8_t* p, uint2 v) { *reinterpret_cast<uint2*>(p) = v; }
__device__ __forceinline__ void sts_v4(uint8_t* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

}  // namespace

struct Gemm16Params {
    const uint8_t* W;        // weight records [G][nblk][REC]
    const uint8_t* act;      // GEMM activation buffer (token-half major, ql_internal.h)
    float* C;
    int32_t* CS;
    int* err;
    int M, N, nblk, G, ldc;
    int m_tiles, n_tiles, tiles;
    int BPS, STAGES;
    uint32_t stage_bytes, off_act;   // inside a stage: weights of 8 groups, then activations
    uint32_t off_a, off_b, off_sc, off_stages;
};

template <bool ZP, bool OUT_CS>
__global__ void __launch_bounds__(N_WARPS * 32, 1) gemm16_kernel(const Gemm16Params p) {
    constexpr int TB = 256, SB = 32, ZB = ZP ? 16 : 0;
    constexpr int REC = TB + SB + ZB;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    uint64_t* stage_full = bars;
    uint64_t* stage_empty = stage_full + p.STAGES;
    uint64_t* a_full = stage_empty + p.STAGES;
    uint64_t* a_empty = a_full + N_ASLOT;
    uint64_t* b_full = a_empty + N_ASLOT;
    uint64_t* b_empty = b_full + N_BSLOT;
    uint64_t* acc_full = b_empty + N_BSLOT;
    uint64_t* acc_empty = acc_full + N_ACC;
    uint64_t* sc_full = acc_empty + N_ACC;
    uint64_t* sc_empty = sc_full + N_SC;
    uint64_t* drain = sc_empty + N_SC;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
    uint8_t* a_ring = smem + p.off_a;
    uint8_t* b_ring = smem + p.off_b;
    uint8_t* sc_ring = smem + p.off_sc;     // per block: 128 x f32 256*bscale, then 128 x f32 ascale
    uint8_t* stages = smem + p.off_stages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int spt = (p.nblk + p.BPS - 1) / p.BPS;        // stages per tile

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.STAGES; ++s) {
            mbar_init(smem_u32(&stage_full[s]), 1);
            mbar_init(smem_u32(&stage_empty[s]), N_UNP + N_CONV);
        }
        for (int a = 0; a < N_ASLOT; ++a) {
            mbar_init(smem_u32(&a_full[a]), N_UNP);
            mbar_init(smem_u32(&a_empty[a]), 1);
        }
        for (int b = 0; b < N_BSLOT; ++b) {
            mbar_init(smem_u32(&b_full[b]), N_CONV);
            mbar_init(smem_u32(&b_empty[b]), 1);
        }
        for (int k = 0; k < N_ACC; ++k) {
            mbar_init(smem_u32(&acc_full[k]), 1);
            mbar_init(smem_u32(&acc_empty[k]), N_EPI);
        }
        for (int k = 0; k < N_SC; ++k) {
            mbar_init(smem_u32(&sc_full[k]), N_CONV);
            mbar_init(smem_u32(&sc_empty[k]), N_EPI);
        }
        mbar_init(smem_u32(drain), 1);
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
        bool pdl_done = false;
        for (int tile = blockIdx.x; tile < p.tiles && __shfl_sync(0xffffffffu, *abort_flag, 0) == 0;
             tile += gridDim.x) {
            const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
            const int G0 = nt * T_G;
            const int groups = min(T_G, p.G - G0);
            for (int ks = 0; ks < spt; ++ks, ++si) {
                const int s = si % p.STAGES;
                if (si >= p.STAGES &&
                    !warp_wait(smem_u32(&stage_empty[s]), ((si / p.STAGES) - 1) & 1, p.err, abort_flag))
                    break;
                if (lane == 0) {
                    const int b0 = ks * p.BPS;
                    const int nb = min(p.BPS, p.nblk - b0);
                    const uint32_t base = smem_u32(stages + static_cast<size_t>(s) * p.stage_bytes);
                    const uint32_t full = smem_u32(&stage_full[s]);
                    mbar_arrive_expect_tx(full, (groups * REC + AREC16) * nb);
                    for (int g = 0; g < groups; ++g) {
                        const size_t rec0 = static_cast<size_t>(G0 + g) * p.nblk + b0;
                        bulk_g2s(base + g * p.BPS * REC, p.W + rec0 * REC, nb * REC, full);
                    }
                    if (!pdl_done) { pdl_wait(); pdl_done = true; }   // activations: previous grid
                    for (int h = 0; h < 2; ++h)
                        bulk_g2s(base + p.off_act + h * p.BPS * GEMM_HPLANES,
                                 p.act + gemm_planes_off(mt, h, b0, p.nblk), nb * GEMM_HPLANES, full);
                    bulk_g2s(base + p.off_act + 2 * p.BPS * GEMM_HPLANES,
                             p.act + gemm_scales_off(mt, b0, p.m_tiles, p.nblk), nb * GEMM_SCALES, full);
                }
                __syncwarp();
            }
        }
        // drain: every stage this warp filled must have landed before exit
        const int issued = si;
        for (int k = std::max(0, issued - p.STAGES); k < issued; ++k)
            mbar_wait(smem_u32(&stage_full[k % p.STAGES]), (k / p.STAGES) & 1, p.err);
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // Per block: D = A0*Bh0 + A1*Bh1 + A0*Bl0 + A1*Bl1 (K = 16 each; A = FP16
        // weights, Bh = h, Bl = l/256), first MMA overwriting the slot.
        constexpr uint32_t idesc = make_idesc_f16(T_N, T_M);
        int bi = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            for (int ks = 0; ks < spt && ok; ++ks) {
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                for (int j = 0; j < nb; ++j, ++bi) {
                    const int as = bi % N_ASLOT, bs = bi % N_BSLOT, ac = bi % N_ACC;
                    if (!(ok = warp_wait(smem_u32(&a_full[as]), (bi / N_ASLOT) & 1, p.err, abort_flag))) break;
                    if (!(ok = warp_wait(smem_u32(&b_full[bs]), (bi / N_BSLOT) & 1, p.err, abort_flag))) break;
                    if (bi >= N_ACC &&
                        !(ok = warp_wait(smem_u32(&acc_empty[ac]), ((bi / N_ACC) - 1) & 1, p.err, abort_flag)))
                        break;
                    tc_fence_after();
                    if (lane == 0) {
                        const uint32_t a0 = smem_u32(a_ring + as * A_BYTES);
                        const uint32_t b0 = smem_u32(b_ring + bs * B_BYTES);
                        const uint32_t d = tmem + ac * T_M;
                        const uint64_t da0 = make_smem_desc(a0, 2048, 128), da1 = make_smem_desc(a0 + 4096, 2048, 128);
                        mma_f16(d, da0, make_smem_desc(b0, 2048, 128), idesc, 0);
                        mma_f16(d, da1, make_smem_desc(b0 + 4096, 2048, 128), idesc, 1);
                        mma_f16(d, da0, make_smem_desc(b0 + 8192, 2048, 128), idesc, 1);
                        mma_f16(d, da1, make_smem_desc(b0 + 12288, 2048, 128), idesc, 1);
                        mma_commit(smem_u32(&acc_full[ac]));
                        mma_commit(smem_u32(&a_empty[as]));
                        mma_commit(smem_u32(&b_empty[bs]));
                    }
                    __syncwarp();
                }
            }
        }
        // drain: all MMAs issued by lane 0 complete before TMEM is freed
        if (lane == 0) mma_commit(smem_u32(drain));
        __syncwarp();
        mbar_wait(smem_u32(drain), 0, p.err);
    } else if (warp < 4) {
        // ------------------------------------------------------------ weight unpack
        // warp u = 2, 3 takes row groups u, u + N_UNP, ...
        const int u = warp - 2;
        const int g = lane >> 2, t = lane & 3;
        // canonical FP16 offset of (row g of group gg, k 4t..4t+3): core-matrix
        // K column t/2 (2048 B apart), 8-row group 2gg (128 B apart), row g (16 B),
        // element 4(t%2) (8 B); row g+8 is the next 8-row group, k+16 two K columns on
        const int o_lane = (t >> 1) * 2048 + g * 16 + (t & 1) * 8;
        int si = 0, bi = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            const int nt = tile / p.m_tiles;
            const int groups = min(T_G, p.G - nt * T_G);
            for (int ks = 0; ks < spt && ok; ++ks, ++si) {
                const int s = si % p.STAGES;
                if (!(ok = warp_wait(smem_u32(&stage_full[s]), (si / p.STAGES) & 1, p.err, abort_flag))) break;
                const uint8_t* wst = stages + static_cast<size_t>(s) * p.stage_bytes;
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                for (int j = 0; j < nb; ++j, ++bi) {
                    const int as = bi % N_ASLOT;
                    if (bi >= N_ASLOT &&
                        !(ok = warp_wait(smem_u32(&a_empty[as]), ((bi / N_ASLOT) - 1) & 1, p.err, abort_flag)))
                        break;
                    uint8_t* dst = a_ring + as * A_BYTES;
#pragma unroll
                    for (int k = 0; k < T_G / N_UNP; ++k) {
                        const int gg = u + k * N_UNP;
                        uint2 r0 = make_uint2(0, 0), r1 = r0, r2 = r0, r3 = r0;
                        if (gg < groups) {
                            const uint8_t* rec = wst + gg * p.BPS * REC + j * REC;
                            const uint2 v = *reinterpret_cast<const uint2*>(rec + lane * 8);
                            // 1024 + zp (row g) and -(64 + zp) (row g+8); zp = 8 by default
                            uint32_t zg = 0x64086408u, zg8 = 0xD480D480u;
                            if (ZP) {
                                const uint32_t z = rec[TB + SB + g];
                                zg = (0x6400u | (z & 15u)) * 0x00010001u;
                                zg8 = (0xD400u | ((z >> 4) << 4)) * 0x00010001u;
                            }
                            nib8_to_f16(v.x, zg, zg8, r0, r1);
                            nib8_to_f16(v.y, zg, zg8, r2, r3);
                        }
                        uint8_t* o = dst + gg * 256 + o_lane;
                        sts_v2(o, r0);                 // row g,   k 4t..
                        sts_v2(o + 128, r1);           // row g+8, k 4t..
                        sts_v2(o + 4096, r2);          // row g,   k 16+4t..
                        sts_v2(o + 4096 + 128, r3);    // row g+8, k 16+4t..
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor core
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&a_full[as]));
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(smem_u32(&stage_empty[s]));
            }
        }
    } else if (warp >= 4 + N_EPI) {
        // ------------------------------------------------------------ activation convert
        // Input (per block and 64-token half h): hi plane then lo plane, each
        // [2 K halves][8 token groups][8 tokens x 16 B] (16 k per row).  Output:
        // h chunks then l/256 chunks, each 4 KB [2 core-matrix K columns][16 token
        // groups][8 tokens x 16 B] (8 k per row): one 16-byte input row of K half
        // kh gives the two 16-byte output rows of chunk kh.
        const int ct = (warp - 4 - N_EPI) * 32 + lane;   // 0..127
        // the weight row whose scale this thread copies: group ct/16, entry
        // 2*(r%8) + r/8 of the record's scales (entry 2g = row g, 2g+1 = row g+8)
        const int cg = ct >> 4, cr = ct & 15, csidx = 2 * (cr & 7) + (cr >> 3);
        int si = 0, bi = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            const int nt = tile / p.m_tiles;
            const bool row_ok = cg < min(T_G, p.G - nt * T_G);
            for (int ks = 0; ks < spt && ok; ++ks, ++si) {
                const int s = si % p.STAGES;
                if (!(ok = warp_wait(smem_u32(&stage_full[s]), (si / p.STAGES) & 1, p.err, abort_flag))) break;
                const uint8_t* ast = stages + static_cast<size_t>(s) * p.stage_bytes + p.off_act;
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                for (int j = 0; j < nb; ++j, ++bi) {
                    const int bs = bi % N_BSLOT, sc = bi % N_SC;
                    if (bi >= N_BSLOT &&
                        !(ok = warp_wait(smem_u32(&b_empty[bs]), ((bi / N_BSLOT) - 1) & 1, p.err, abort_flag)))
                        break;
                    if (bi >= N_SC &&
                        !(ok = warp_wait(smem_u32(&sc_empty[sc]), ((bi / N_SC) - 1) & 1, p.err, abort_flag)))
                        break;
                    uint8_t* dst = b_ring + bs * B_BYTES;
                    // activation scale of token ct and 256*bscale of weight row ct
                    // (exact: an exponent shift of the FP16 scale); 0 past the last row group
                    float* scs = reinterpret_cast<float*>(sc_ring + sc * SC_BYTES);
                    scs[128 + ct] = reinterpret_cast<const float*>(ast + 2 * p.BPS * GEMM_HPLANES + j * GEMM_SCALES)[ct];
                    const uint8_t* wrec = stages + static_cast<size_t>(s) * p.stage_bytes + cg * p.BPS * REC + j * REC;
                    scs[ct] = row_ok ? __half2float(reinterpret_cast<const __half*>(wrec + TB)[csidx]) * 256.0f : 0.0f;
#pragma unroll
                    for (int rep = 0; rep < 2; ++rep) {
                        // input row w = kh*64 + tg*8 + r of token half rep (token 64*rep + 8*tg + r)
                        const int w = ct;
                        const int kh = w >> 6;
                        const int o = kh * 4096 + rep * 1024 + (w & 63) * 16;   // (8*rep + tg)*128 + r*16
                        const uint8_t* src = ast + (rep * p.BPS + j) * GEMM_HPLANES;
                        const uint4 vh = *reinterpret_cast<const uint4*>(src + w * 16);
                        const uint4 vl = *reinterpret_cast<const uint4*>(src + 2048 + w * 16);
                        const uint2 h0 = hi4_to_f16(vh.x), h1 = hi4_to_f16(vh.y);
                        const uint2 h2 = hi4_to_f16(vh.z), h3 = hi4_to_f16(vh.w);
                        const uint2 l0 = lo4_to_f16(vl.x), l1 = lo4_to_f16(vl.y);
                        const uint2 l2 = lo4_to_f16(vl.z), l3 = lo4_to_f16(vl.w);
                        sts_v4(dst + o, make_uint4(h0.x, h0.y, h1.x, h1.y));                // k 0..7
                        sts_v4(dst + o + 2048, make_uint4(h2.x, h2.y, h3.x, h3.y));         // k 8..15
                        sts_v4(dst + 8192 + o, make_uint4(l0.x, l0.y, l1.x, l1.y));
                        sts_v4(dst + 8192 + o + 2048, make_uint4(l2.x, l2.y, l3.x, l3.y));
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor core
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(smem_u32(&b_full[bs]));
                        mbar_arrive(smem_u32(&sc_full[sc]));
                    }
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(smem_u32(&stage_empty[s]));
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int e = warp - 4;
        const int q = warp & 3;                           // TMEM lane quarter (hardware rule: warp % 4)
        const int cq = e >> 2;                            // token columns E_COLS*cq ..
        const int row = q * 32 + lane;                    // weight row within the tile
        const int g16 = row >> 4;
        int bi = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
            const int n = nt * T_N + row;
            const int groups = min(T_G, p.G - nt * T_G);
            uint64_t acc[E_COLS / 2];                     // E_COLS token columns as f32x2 pairs
#pragma unroll
            for (int i = 0; i < E_COLS / 2; ++i) acc[i] = 0;
            for (int ks = 0; ks < spt && ok; ++ks) {
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                for (int j = 0; j < nb; ++j, ++bi) {
                    const int ac = bi % N_ACC, sc = bi % N_SC;
                    if (!(ok = warp_wait(smem_u32(&sc_full[sc]), (bi / N_SC) & 1, p.err, abort_flag))) break;
                    if (!(ok = warp_wait(smem_u32(&acc_full[ac]), (bi / N_ACC) & 1, p.err, abort_flag))) break;
                    tc_fence_after();
                    const float* scs = reinterpret_cast<const float*>(sc_ring + sc * SC_BYTES);
                    const float bs256 = scs[row];                 // 256 * bscale (0 past the last row group)
                    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + ac * T_M + cq * E_COLS;
                    if constexpr (OUT_CS) {
                        // block sums [M][N][nblk] = 256 * D (exact): a checking output
#pragma unroll 1
                        for (int cc = 0; cc < E_COLS / 16; ++cc) {
                            uint32_t v[16];
                            tmem_ld16(taddr + cc * 16, v);
                            tmem_wait_ld();
                            const int m0 = mt * T_M + cq * E_COLS + cc * 16;
                            int32_t* dst = p.CS + (static_cast<size_t>(m0) * p.N + n) * p.nblk + ks * p.BPS + j;
#pragma unroll
                            for (int k = 0; k < 16; ++k) {
                                const int32_t cs = __float2int_rn(__uint_as_float(v[k]) * 256.0f);
                                if (m0 + k < p.M && g16 < groups) *dst = cs;
                                dst += static_cast<size_t>(p.N) * p.nblk;
                            }
                        }
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(smem_u32(&acc_empty[ac]));
                            mbar_arrive(smem_u32(&sc_empty[sc]));
                        }
                        (void)bs256;
                    } else {
                        const uint64_t bs2 = f2_pack(bs256, bs256);
                        const float* ascale = scs + 128 + cq * E_COLS;
                        // 8-column chunks; the next chunk's TMEM load is in flight while
                        // this one is rescaled; the slot is released as soon as its last
                        // chunk has been read
                        constexpr int NCH = E_COLS / 8;
                        uint32_t v[2][8];
                        tmem_ld8(taddr, v[0]);
                        tmem_wait_ld();
#pragma unroll
                        for (int cc = 0; cc < NCH; ++cc) {
                            const int cur = cc & 1;
                            if (cc < NCH - 1) tmem_ld8(taddr + (cc + 1) * 8, v[cur ^ 1]);
#pragma unroll
                            for (int k = 0; k < 8; k += 4) {
                                const float4 a4 = lds_f4(ascale + cc * 8 + k);
                                const int i0 = (cc * 8 + k) >> 1;
                                const uint64_t d0 = i2_pack(static_cast<int32_t>(v[cur][k]),
                                                            static_cast<int32_t>(v[cur][k + 1]));
                                const uint64_t d1 = i2_pack(static_cast<int32_t>(v[cur][k + 2]),
                                                            static_cast<int32_t>(v[cur][k + 3]));
                                acc[i0] = f2_fma(f2_pack(a4.x, a4.y), f2_mul(d0, bs2), acc[i0]);
                                acc[i0 + 1] = f2_fma(f2_pack(a4.z, a4.w), f2_mul(d1, bs2), acc[i0 + 1]);
                            }
                            if (cc < NCH - 1) {
                                tmem_wait_ld();
                                if (cc == NCH - 2) {
                                    // every column of the slot is in registers: hand it back
                                    tc_fence_before();
                                    __syncwarp();
                                    if (lane == 0) mbar_arrive(smem_u32(&acc_empty[ac]));
                                }
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_u32(&sc_empty[sc]));
                    }
                }
            }
            if (!ok || OUT_CS) continue;
            // store C[m, n] for this thread's 64 token columns (lanes = consecutive n)
            if (g16 < groups) {
#pragma unroll
                for (int i = 0; i < E_COLS / 2; ++i) {
                    const int m = mt * T_M + cq * E_COLS + 2 * i;
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


// ======================================================================== CTA pair
// gemm16x2_kernel: the same numerics on tcgen05.mma.cta_group::2 (M = 256),
// selected with ql_set_prefill_kernel(2).  On B200 it runs at the speed of the
// single-CTA kernel (1855 vs 1861 us at M = 2048, K = 5120, N = 17408) with
// 40% less L2 -> SM traffic per SM: both are bound by pipeline latency in their
// CUDA-core roles, not by the copies the pair halves.
// A cluster of two CTAs on two SMs owns a tile of 256 weight rows x 128
// tokens: CTA r (cluster rank) holds weight rows 128r.. (the MMA's A rows) and
// the token half 64r.. (its half of the MMA's B columns) in its own shared
// memory, and receives all 128 token columns of its 128 rows in its own TMEM.
// Each CTA therefore loads and converts only half of the token tile: the
// activation L2 -> SM traffic and conversion work per SM halve, and the tensor
// core reads 6 KB instead of 8 KB of shared memory per 128x128x16 step.
//
// The leader (rank 0) issues the MMAs.  Operand readiness from both CTAs is
// counted on the leader's a_full / b_full barriers (the peer's unpack and
// convert warps arrive remotely, release at cluster scope after a
// fence.proxy.async); slot releases and accumulator-full signals are multicast
// commits to both CTAs; both CTAs' epilogues release an accumulator slot on the
// leader's acc_empty.  Waits are bounded (1 s) and a CTA that gives up raises
// the abort flag of both CTAs; the pair meets at a cluster barrier before exit.
//
// Warp roles (16 warps per CTA): 0 producer, 1 MMA (leader issues; both CTAs
// allocate TMEM), 2-3 and 14-15 weight unpack (2 row groups each), 4-11
// epilogue, 12-13 activation convert (64 tokens) -- so each SM sub-partition
// (warp % 4) runs two epilogue warps and one unpack or convert warp.
namespace {
constexpr int X_UNP = 4;                 // weight unpack warps
constexpr int X_CONV = 2;                // activation convert warps (64 tokens)
constexpr int X_B_BYTES = 64 * 64 * 2;   // FP16 B half per block: h, l/256 for 64 tokens (8 KB)
constexpr int X_ASLOT = 4, X_BSLOT = 4;

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
    return d;
}
// arrive on an mbarrier of either CTA of the pair (address from map_to_rank).
// Default (CTA-scope release) semantics, as the tensor-core pipelines use for
// peer signals: the data a peer signals about stays in the peer's own shared
// memory and is read by the peer's own tensor core.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity, uint32_t ns) {
    return mbar_try_wait_sleep(bar, parity, ns);
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// commit: arrive once on the barrier at this shared offset in both CTAs when
// all prior tcgen05 operations of this thread have completed
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 :: "r"(bar), "h"(static_cast<uint16_t>(3)) : "memory");
}

// Bounded wait for the pair: gives up after the wait limit, or when either CTA
// raised its abort flag; on giving up it raises both flags.
__device__ __forceinline__ bool pair_wait(uint32_t bar, uint32_t parity, int* err, volatile int* abort_flag,
                                          uint32_t peer_abort) {
    bool ok = mbar_try_wait_cluster(bar, parity, 0);
    if (!ok) {
        const uint64_t t0 = global_ns();
        uint64_t limit = WAIT_CHECK_NS;     // the device limit is read once this much has passed
        bool read = false;
        while (true) {
            if (mbar_try_wait_cluster(bar, parity, 10000)) { ok = true; break; }
            if (*abort_flag) break;
            if (global_ns() - t0 > limit && !read) {
                limit = wait_limit(err);
                read = true;
                continue;
            }
            if (global_ns() - t0 > limit) {
                record_error(err, QL_ETIMEOUT);
                *abort_flag = 1;
                asm volatile("st.shared::cluster.u32 [%0], %1;" :: "r"(peer_abort), "r"(1) : "memory");
                break;
            }
        }
    }
    return __all_sync(0xffffffffu, ok);
}
}  // namespace

template <bool ZP, bool OUT_CS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(N_WARPS * 32, 1) gemm16x2_kernel(const Gemm16Params p) {
    constexpr int TB = 256, SB = 32, ZB = ZP ? 16 : 0;
    constexpr int REC = TB + SB + ZB;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    uint64_t* stage_full = bars;
    uint64_t* stage_empty = stage_full + p.STAGES;
    uint64_t* a_full = stage_empty + p.STAGES;          // leader's counts both CTAs
    uint64_t* a_empty = a_full + X_ASLOT;               // multicast commit
    uint64_t* b_full = a_empty + X_ASLOT;               // leader's counts both CTAs
    uint64_t* b_empty = b_full + X_BSLOT;               // multicast commit
    uint64_t* acc_full = b_empty + X_BSLOT;             // multicast commit
    uint64_t* acc_empty = acc_full + N_ACC;             // leader's counts both CTAs
    uint64_t* sc_full = acc_empty + N_ACC;
    uint64_t* sc_empty = sc_full + N_SC;
    uint64_t* drain = sc_empty + N_SC;                  // multicast commit
    volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
    uint8_t* a_ring = smem + p.off_a;
    uint8_t* b_ring = smem + p.off_b;
    uint8_t* sc_ring = smem + p.off_sc;
    uint8_t* stages = smem + p.off_stages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const uint32_t peer_abort = map_to_rank(smem_u32(const_cast<int*>(abort_flag)), rank ^ 1u);
    const int spt = (p.nblk + p.BPS - 1) / p.BPS;
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    auto waitp = [&](uint64_t* bar, uint32_t parity) {
        return pair_wait(smem_u32(bar), parity, p.err, abort_flag, peer_abort);
    };
    // the leader's copy of a barrier (remote for rank 1)
    auto leader_bar = [&](uint64_t* bar) { return map_to_rank(smem_u32(bar), 0); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.STAGES; ++s) {
            mbar_init(smem_u32(&stage_full[s]), 1);
            mbar_init(smem_u32(&stage_empty[s]), X_UNP + X_CONV);
        }
        for (int a = 0; a < X_ASLOT; ++a) {
            mbar_init(smem_u32(&a_full[a]), 2 * X_UNP);
            mbar_init(smem_u32(&a_empty[a]), 1);
        }
        for (int b = 0; b < X_BSLOT; ++b) {
            mbar_init(smem_u32(&b_full[b]), 2 * X_CONV);
            mbar_init(smem_u32(&b_empty[b]), 1);
        }
        for (int k = 0; k < N_ACC; ++k) {
            mbar_init(smem_u32(&acc_full[k]), 1);
            mbar_init(smem_u32(&acc_empty[k]), 2 * N_EPI);
        }
        for (int k = 0; k < N_SC; ++k) {
            mbar_init(smem_u32(&sc_full[k]), X_CONV);
            mbar_init(smem_u32(&sc_empty[k]), N_EPI);
        }
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(TMEM_NCOLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync_all();        // both CTAs' barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        int si = 0;
        bool pdl_done = false;
        for (int tile = pair; tile < p.tiles && __shfl_sync(0xffffffffu, *abort_flag, 0) == 0; tile += pairs) {
            const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
            const int G0 = nt * 2 * T_G + static_cast<int>(rank) * T_G;
            const int groups = max(0, min(T_G, p.G - G0));
            for (int ks = 0; ks < spt; ++ks, ++si) {
                const int s = si % p.STAGES;
                if (si >= p.STAGES && !waitp(&stage_empty[s], ((si / p.STAGES) - 1) & 1)) break;
                if (lane == 0) {
                    const int b0 = ks * p.BPS;
                    const int nb = min(p.BPS, p.nblk - b0);
                    const uint32_t base = smem_u32(stages + static_cast<size_t>(s) * p.stage_bytes);
                    const uint32_t full = smem_u32(&stage_full[s]);
                    mbar_arrive_expect_tx(full, (groups * REC + GEMM_HPLANES + GEMM_SCALES) * nb);
                    for (int g = 0; g < groups; ++g) {
                        const size_t rec0 = static_cast<size_t>(G0 + g) * p.nblk + b0;
                        bulk_g2s(base + g * p.BPS * REC, p.W + rec0 * REC, nb * REC, full);
                    }
                    if (!pdl_done) { pdl_wait(); pdl_done = true; }   // activations: previous grid
                    bulk_g2s(base + p.off_act, p.act + gemm_planes_off(mt, static_cast<int>(rank), b0, p.nblk),
                             nb * GEMM_HPLANES, full);
                    bulk_g2s(base + p.off_act + p.BPS * GEMM_HPLANES,
                             p.act + gemm_scales_off(mt, b0, p.m_tiles, p.nblk), nb * GEMM_SCALES, full);
                }
                __syncwarp();
            }
        }
        const int issued = si;
        for (int k = std::max(0, issued - p.STAGES); k < issued; ++k)
            mbar_wait(smem_u32(&stage_full[k % p.STAGES]), (k / p.STAGES) & 1, p.err);
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader)
        if (leader) {
            constexpr uint32_t idesc = make_idesc_f16(2 * T_N, T_M);
            int bi = 0;
            bool ok = true;
            for (int tile = pair; tile < p.tiles && ok; tile += pairs) {
                for (int ks = 0; ks < spt && ok; ++ks) {
                    const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                    for (int j = 0; j < nb; ++j, ++bi) {
                        const int as = bi % X_ASLOT, bs = bi % X_BSLOT, ac = bi % N_ACC;
                        if (!(ok = waitp(&a_full[as], (bi / X_ASLOT) & 1))) break;
                        if (!(ok = waitp(&b_full[bs], (bi / X_BSLOT) & 1))) break;
                        if (bi >= N_ACC && !(ok = waitp(&acc_empty[ac], ((bi / N_ACC) - 1) & 1))) break;
                        tc_fence_after();
                        if (lane == 0) {
                            const uint32_t a0 = smem_u32(a_ring + as * A_BYTES);
                            const uint32_t b0 = smem_u32(b_ring + bs * X_B_BYTES);
                            const uint32_t d = tmem + ac * T_M;
                            const uint64_t da0 = make_smem_desc(a0, 2048, 128), da1 = make_smem_desc(a0 + 4096, 2048, 128);
                            mma_f16_pair(d, da0, make_smem_desc(b0, 1024, 128), idesc, 0);
                            mma_f16_pair(d, da1, make_smem_desc(b0 + 2048, 1024, 128), idesc, 1);
                            mma_f16_pair(d, da0, make_smem_desc(b0 + 4096, 1024, 128), idesc, 1);
                            mma_f16_pair(d, da1, make_smem_desc(b0 + 6144, 1024, 128), idesc, 1);
                            mma_commit_pair(smem_u32(&acc_full[ac]));
                            mma_commit_pair(smem_u32(&a_empty[as]));
                            mma_commit_pair(smem_u32(&b_empty[bs]));
                        }
                        __syncwarp();
                    }
                }
            }
            if (lane == 0) mma_commit_pair(smem_u32(drain));
            __syncwarp();
        }
        // both CTAs: every MMA that writes this CTA's TMEM has completed (the
        // leader commits once after its last MMA; the bound is far above any call)
        {
            const uint64_t t0 = global_ns();
            while (!mbar_try_wait_cluster(smem_u32(drain), 0, 20000)) {
                if (global_ns() - t0 > 60ull * wait_limit(p.err)) { record_error(p.err, QL_ETIMEOUT); break; }
            }
        }
    } else if (warp < 4 || warp >= 4 + N_EPI + X_CONV) {
        // ------------------------------------------------------------ weight unpack
        // warps 2, 3, 14, 15 -> u = 0..3; warp u takes row groups u and u + 4
        const int u = warp < 4 ? warp - 2 : warp - (4 + N_EPI + X_CONV) + 2;
        const int g = lane >> 2, t = lane & 3;
        const int o_lane = (t >> 1) * 2048 + g * 16 + (t & 1) * 8;
        int si = 0, bi = 0;
        bool ok = true;
        for (int tile = pair; tile < p.tiles && ok; tile += pairs) {
            const int nt = tile / p.m_tiles;
            const int groups = max(0, min(T_G, p.G - (nt * 2 * T_G + static_cast<int>(rank) * T_G)));
            for (int ks = 0; ks < spt && ok; ++ks, ++si) {
                const int s = si % p.STAGES;
                if (!(ok = waitp(&stage_full[s], (si / p.STAGES) & 1))) break;
                const uint8_t* wst = stages + static_cast<size_t>(s) * p.stage_bytes;
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                for (int j = 0; j < nb; ++j, ++bi) {
                    const int as = bi % X_ASLOT;
                    if (bi >= X_ASLOT && !(ok = waitp(&a_empty[as], ((bi / X_ASLOT) - 1) & 1))) break;
                    uint8_t* dst = a_ring + as * A_BYTES;
#pragma unroll
                    for (int k = 0; k < T_G / X_UNP; ++k) {
                        const int gg = u + k * X_UNP;
                        uint2 r0 = make_uint2(0, 0), r1 = r0, r2 = r0, r3 = r0;
                        if (gg < groups) {
                            const uint8_t* rec = wst + gg * p.BPS * REC + j * REC;
                            const uint2 v = *reinterpret_cast<const uint2*>(rec + lane * 8);
                            uint32_t zg = 0x64086408u, zg8 = 0xD480D480u;
                            if (ZP) {
                                const uint32_t z = rec[TB + SB + g];
                                zg = (0x6400u | (z & 15u)) * 0x00010001u;
                                zg8 = (0xD400u | ((z >> 4) << 4)) * 0x00010001u;
                            }
                            nib8_to_f16(v.x, zg, zg8, r0, r1);
                            nib8_to_f16(v.y, zg, zg8, r2, r3);
                        }
                        uint8_t* o = dst + gg * 256 + o_lane;
                        sts_v2(o, r0);
                        sts_v2(o + 128, r1);
                        sts_v2(o + 4096, r2);
                        sts_v2(o + 4096 + 128, r3);
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor cores
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(leader_bar(&a_full[as]));
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(smem_u32(&stage_empty[s]));
            }
        }
    } else if (warp >= 4 + N_EPI) {
        // ------------------------------------------------------------ activation convert (64 tokens)
        // Input per block: this CTA's half -- hi plane then lo plane, each [2 K
        // halves][8 token groups][8 tokens x 16 B].  Output B half: h chunks
        // (K 0-15, 16-31) then l/256 chunks, each 2 KB [2 core-matrix K columns]
        // [8 token groups][8 tokens x 16 B] (LBO 1024, SBO 128).
        const int ct = (warp - (4 + N_EPI)) * 32 + lane;   // warps 12, 13 -> 0..63
        int si = 0, bi = 0;
        bool ok = true;
        for (int tile = pair; tile < p.tiles && ok; tile += pairs) {
            const int nt = tile / p.m_tiles;
            const int G0 = nt * 2 * T_G + static_cast<int>(rank) * T_G;
            const int groups = max(0, min(T_G, p.G - G0));
            for (int ks = 0; ks < spt && ok; ++ks, ++si) {
                const int s = si % p.STAGES;
                if (!(ok = waitp(&stage_full[s], (si / p.STAGES) & 1))) break;
                const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
                const uint8_t* ast = st + p.off_act;
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                for (int j = 0; j < nb; ++j, ++bi) {
                    const int bs = bi % X_BSLOT, sc = bi % N_SC;
                    if (bi >= X_BSLOT && !(ok = waitp(&b_empty[bs], ((bi / X_BSLOT) - 1) & 1))) break;
                    if (bi >= N_SC && !(ok = waitp(&sc_empty[sc], ((bi / N_SC) - 1) & 1))) break;
                    uint8_t* dst = b_ring + bs * X_B_BYTES;
                    const uint8_t* src = ast + j * GEMM_HPLANES;
                    // scales: activation scales of all 128 tokens, 256*bscale of this CTA's 128 rows
                    float* scs = reinterpret_cast<float*>(sc_ring + sc * SC_BYTES);
                    const float* asrc = reinterpret_cast<const float*>(ast + p.BPS * GEMM_HPLANES + j * GEMM_SCALES);
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int r = ct + 64 * e;
                        scs[128 + r] = asrc[r];
                        const int cg = r >> 4, cr = r & 15;
                        const uint8_t* wrec = st + cg * p.BPS * REC + j * REC;
                        scs[r] = cg < groups
                                     ? __half2float(reinterpret_cast<const __half*>(wrec + TB)[2 * (cr & 7) + (cr >> 3)]) * 256.0f
                                     : 0.0f;
                    }
#pragma unroll
                    for (int rep = 0; rep < 2; ++rep) {
                        const int w = ct + 64 * rep;                      // input row kh*64 + tg*8 + r
                        const int o = (w >> 6) * 2048 + (w & 63) * 16;    // chunk kh: tg*128 + r*16
                        const uint4 vh = *reinterpret_cast<const uint4*>(src + w * 16);
                        const uint4 vl = *reinterpret_cast<const uint4*>(src + 2048 + w * 16);
                        const uint2 h0 = hi4_to_f16(vh.x), h1 = hi4_to_f16(vh.y);
                        const uint2 h2 = hi4_to_f16(vh.z), h3 = hi4_to_f16(vh.w);
                        const uint2 l0 = lo4_to_f16(vl.x), l1 = lo4_to_f16(vl.y);
                        const uint2 l2 = lo4_to_f16(vl.z), l3 = lo4_to_f16(vl.w);
                        sts_v4(dst + o, make_uint4(h0.x, h0.y, h1.x, h1.y));                // k 0..7
                        sts_v4(dst + o + 1024, make_uint4(h2.x, h2.y, h3.x, h3.y));         // k 8..15
                        sts_v4(dst + 4096 + o, make_uint4(l0.x, l0.y, l1.x, l1.y));
                        sts_v4(dst + 4096 + o + 1024, make_uint4(l2.x, l2.y, l3.x, l3.y));
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor cores
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive_cluster(leader_bar(&b_full[bs]));
                        mbar_arrive(smem_u32(&sc_full[sc]));
                    }
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(smem_u32(&stage_empty[s]));
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int e = warp - 4;
        const int q = warp & 3;
        const int cq = e >> 2;
        const int row = q * 32 + lane;
        const int g16 = row >> 4;
        int bi = 0;
        bool ok = true;
        for (int tile = pair; tile < p.tiles && ok; tile += pairs) {
            const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
            const int G0 = nt * 2 * T_G + static_cast<int>(rank) * T_G;
            const int n = G0 * 16 + row;
            const int groups = max(0, min(T_G, p.G - G0));
            uint64_t acc[E_COLS / 2];
#pragma unroll
            for (int i = 0; i < E_COLS / 2; ++i) acc[i] = 0;
            for (int ks = 0; ks < spt && ok; ++ks) {
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                for (int j = 0; j < nb; ++j, ++bi) {
                    const int ac = bi % N_ACC, sc = bi % N_SC;
                    if (!(ok = waitp(&sc_full[sc], (bi / N_SC) & 1))) break;
                    if (!(ok = waitp(&acc_full[ac], (bi / N_ACC) & 1))) break;
                    tc_fence_after();
                    const float* scs = reinterpret_cast<const float*>(sc_ring + sc * SC_BYTES);
                    const float bs256 = scs[row];
                    const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + ac * T_M + cq * E_COLS;
                    if constexpr (OUT_CS) {
#pragma unroll 1
                        for (int cc = 0; cc < E_COLS / 16; ++cc) {
                            uint32_t v[16];
                            tmem_ld16(taddr + cc * 16, v);
                            tmem_wait_ld();
                            const int m0 = mt * T_M + cq * E_COLS + cc * 16;
                            int32_t* dst = p.CS + (static_cast<size_t>(m0) * p.N + n) * p.nblk + ks * p.BPS + j;
#pragma unroll
                            for (int k = 0; k < 16; ++k) {
                                const int32_t cs = __float2int_rn(__uint_as_float(v[k]) * 256.0f);
                                if (m0 + k < p.M && g16 < groups) *dst = cs;
                                dst += static_cast<size_t>(p.N) * p.nblk;
                            }
                        }
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive_cluster(leader_bar(&acc_empty[ac]));
                            mbar_arrive(smem_u32(&sc_empty[sc]));
                        }
                        (void)bs256;
                    } else {
                        const uint64_t bs2 = f2_pack(bs256, bs256);
                        const float* ascale = scs + 128 + cq * E_COLS;
                        // 16-column chunks, the next chunk's TMEM load in flight while this
                        // one is rescaled; the slot is released once its last chunk is read
                        constexpr int NCH = E_COLS / 16;
                        uint32_t v[2][16];
                        tmem_ld16(taddr, v[0]);
                        tmem_wait_ld();
#pragma unroll
                        for (int cc = 0; cc < NCH; ++cc) {
                            const int cur = cc & 1;
                            if (cc < NCH - 1) tmem_ld16(taddr + (cc + 1) * 16, v[cur ^ 1]);
#pragma unroll
                            for (int k = 0; k < 16; k += 4) {
                                const float4 a4 = lds_f4(ascale + cc * 16 + k);
                                const int i0 = (cc * 16 + k) >> 1;
                                const uint64_t d0 = i2_pack(static_cast<int32_t>(v[cur][k]),
                                                            static_cast<int32_t>(v[cur][k + 1]));
                                const uint64_t d1 = i2_pack(static_cast<int32_t>(v[cur][k + 2]),
                                                            static_cast<int32_t>(v[cur][k + 3]));
                                acc[i0] = f2_fma(f2_pack(a4.x, a4.y), f2_mul(d0, bs2), acc[i0]);
                                acc[i0 + 1] = f2_fma(f2_pack(a4.z, a4.w), f2_mul(d1, bs2), acc[i0 + 1]);
                            }
                            if (cc < NCH - 1) {
                                tmem_wait_ld();
                                if (cc == NCH - 2) {
                                    tc_fence_before();
                                    __syncwarp();
                                    if (lane == 0) mbar_arrive_cluster(leader_bar(&acc_empty[ac]));
                                }
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_u32(&sc_empty[sc]));
                    }
                }
            }
            if (!ok || OUT_CS) continue;
            if (g16 < groups) {
#pragma unroll
                for (int i = 0; i < E_COLS / 2; ++i) {
                    const int m = mt * T_M + cq * E_COLS + 2 * i;
                    const float2 v = f2_unpack(acc[i]);
                    if (m < p.M) p.C[static_cast<size_t>(m) * p.ldc + n] = v.x;
                    if (m + 1 < p.M) p.C[static_cast<size_t>(m + 1) * p.ldc + n] = v.y;
                }
            }
        }
    }

    // every role is done (or aborted); the pair frees TMEM and meets before exit
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TMEM_NCOLS) : "memory");
    cluster_sync_all();
}

// ------------------------------------------------------------------ host side

int* device_error_word();   // ql_api.cu

template <bool ZP, bool OUT_CS>
static cudaError_t gemm16_launch(const Gemm16Params& p0, cudaStream_t stream) {
    constexpr int REC = 256 + 32 + (ZP ? 16 : 0);
    Gemm16Params p = p0;
    p.BPS = 4;
    p.off_act = T_G * p.BPS * REC;
    p.stage_bytes = (p.off_act + p.BPS * AREC16 + 1023) & ~1023u;
    const uint32_t bar_bytes = 1024;                       // barriers, abort flag, TMEM address
    p.off_a = bar_bytes;
    p.off_b = p.off_a + N_ASLOT * A_BYTES;
    p.off_sc = p.off_b + N_BSLOT * B_BYTES;
    p.off_stages = p.off_sc + N_SC * SC_BYTES;
    p.STAGES = 3;
    while (p.STAGES > 2 && p.off_stages + static_cast<size_t>(p.STAGES) * p.stage_bytes > 227 * 1024) --p.STAGES;
    const size_t smem = p.off_stages + static_cast<size_t>(p.STAGES) * p.stage_bytes;
    const size_t bars = (2 * p.STAGES + 2 * N_ASLOT + 2 * N_BSLOT + 2 * N_ACC + 2 * N_SC + 1) * 8 + 16;
    if (smem > 227 * 1024 || bars > bar_bytes || (p.off_act % 16) || (REC % 16) || (p.off_a % 1024) ||
        (p.off_b % 1024) || (p.off_stages % 1024))
        return cudaErrorInvalidConfiguration;
    auto kern = gemm16_kernel<ZP, OUT_CS>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    static int sms[64] = {0};
    if (sms[dev] == 0) {
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
        if (sms[dev] <= 0) sms[dev] = 148;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(p.tiles, sms[dev]));
    cfg.blockDim = dim3(N_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <bool ZP, bool OUT_CS>
static cudaError_t gemm16x2_launch(const Gemm16Params& p0, cudaStream_t stream) {
    constexpr int REC = 256 + 32 + (ZP ? 16 : 0);
    Gemm16Params p = p0;
    p.BPS = 4;
    p.off_act = T_G * p.BPS * REC;
    p.stage_bytes = (p.off_act + p.BPS * (GEMM_HPLANES + GEMM_SCALES) + 1023) & ~1023u;
    const uint32_t bar_bytes = 1024;
    p.off_a = bar_bytes;
    p.off_b = p.off_a + X_ASLOT * A_BYTES;
    p.off_sc = p.off_b + X_BSLOT * X_B_BYTES;
    p.off_stages = p.off_sc + N_SC * SC_BYTES;
    p.STAGES = 5;
    while (p.STAGES > 2 && p.off_stages + static_cast<size_t>(p.STAGES) * p.stage_bytes > 227 * 1024) --p.STAGES;
    const size_t smem = p.off_stages + static_cast<size_t>(p.STAGES) * p.stage_bytes;
    const size_t bars = (2 * p.STAGES + 2 * X_ASLOT + 2 * X_BSLOT + 2 * N_ACC + 2 * N_SC + 1) * 8 + 16;
    if (smem > 227 * 1024 || bars > bar_bytes || (p.off_act % 16) || (REC % 16) || (p.off_a % 1024) ||
        (p.off_b % 1024) || (p.off_sc % 1024) || (p.off_stages % 1024))
        return cudaErrorInvalidConfiguration;
    auto kern = gemm16x2_kernel<ZP, OUT_CS>;
    static int configured[64] = {0};
    static int max_pairs[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(N_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        // co-resident CTA pairs (one CTA per SM; pairs must share a GPC)
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaLaunchConfig_t q = cfg;
        q.gridDim = dim3(2 * std::max(1, sms / 2));
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kern, &q) != cudaSuccess || clusters <= 0) {
            cudaGetLastError();
            clusters = std::max(1, sms / 2);
        }
        max_pairs[dev] = clusters;
        configured[dev] = 1;
    }
    cfg.gridDim = dim3(2 * std::min(p.tiles, max_pairs[dev]));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

bool gemm16_supports(const Weight* w, bool hi_prec) {
    return w->bits == 4 && w->scale_half && hi_prec;
}

cudaError_t launch_gemm16(const Weight* w, const uint8_t* act, int M, float* C, int ldc, int32_t* cs,
                          cudaStream_t stream) {
    Gemm16Params p = {};
    p.W = w->W;
    p.act = act;
    p.C = C;
    p.CS = cs;
    p.err = device_error_word();
    p.M = M;
    p.N = w->N;
    p.nblk = w->nblk;
    p.G = w->G;
    p.ldc = ldc;
    p.m_tiles = (M + T_M - 1) / T_M;
    if (prefill_kernel() == QL_PREFILL_F16_PAIR) {
        // CTA pairs: tiles of 256 weight rows x 128 tokens
        p.n_tiles = (w->N + 2 * T_N - 1) / (2 * T_N);
        p.tiles = p.m_tiles * p.n_tiles;
        if (w->has_zp) return cs ? gemm16x2_launch<true, true>(p, stream) : gemm16x2_launch<true, false>(p, stream);
        return cs ? gemm16x2_launch<false, true>(p, stream) : gemm16x2_launch<false, false>(p, stream);
    }
    p.n_tiles = (w->N + T_N - 1) / T_N;
    p.tiles = p.m_tiles * p.n_tiles;
    if (w->has_zp) return cs ? gemm16_launch<true, true>(p, stream) : gemm16_launch<true, false>(p, stream);
    return cs ? gemm16_launch<false, true>(p, stream) : gemm16_launch<false, false>(p, stream);
}

}  // namespace ql
