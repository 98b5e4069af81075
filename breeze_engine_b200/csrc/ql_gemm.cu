// ql_gemm.cu -- prefill quantized GEMM (M > 64 tokens) on tcgen05 tensor cores.
//
// Computes C[m, n] = i4_matmul(A)[m, n] (kernel/quantized_matmul.cpp:270-365,
// the 8-row chunk loop :545-549) from activations quantized into the GEMM
// record layout (ql_quant.cu), bit-identical to the reference.
//
// Tile: 128 output features (weights are the MMA's M = 128 A operand) x 128
// tokens (the MMA's N = 128 B operand).  Persistent CTAs (one per SM, all 512
// TMEM columns) walk the tiles with the token tile fastest, so concurrent CTAs
// share weight tiles and activation tiles through L2.
//
// Per 32-wide K block two tcgen05.mma.cta_group::1.kind::i8 (128x128x32):
//   hi plane (hi - 128, s8) x weights (s8) and lo plane (u8) x weights (s8)
// into a TMEM slot of 256 columns (hi | lo); two slots alternate so the
// tensor core fills one while the epilogue drains the other.  Every block
// needs its own FP32 rescale (ascale[m,b] * bscale[n,b] differ per block), so
// the epilogue drains TMEM once per block: exact conversion of 256*S_hi + S_lo
// to float (the seeded-magic identity of ql_common.cuh) and the reference's
// chain acc = fma(ascale, RN(cs * bscale), acc) in ascending block order.
//
// Warp roles (12 warps):
//   0      producer: 1-D bulk copies (no multicast) of the 8 row groups' weight
//          records and the token tile's activation record per stage
//   1      MMA issuer (one thread) and TMEM owner (allocates/frees 512 columns)
//   2-3    unpack: weight records (mma.sync fragment order, INT4 nibbles or
//          INT8) -> s8 (q - zp) in the canonical K-major SWIZZLE_NONE layout
//          (core matrices of 8 rows x 16 B; LBO = 2048 B between the two
//          16-byte K halves, SBO = 128 B between 8-row groups)
//   4-11   epilogue: warp w reads TMEM lanes 32*(w%4).. (its 32 weight rows)
//          and token half (w-4)/4 (64 columns)
// Every mbarrier is waited by its consumers phase by phase in order; every wait
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

constexpr int TILE_N = 128;            // weight rows per tile (MMA M)
constexpr int TILE_M = 128;            // tokens per tile (MMA N)
constexpr int GROUPS = TILE_N / 16;    // 16-row weight groups per tile
constexpr int NUNPACK = 2;             // unpack warps
constexpr int NEPI = 8;                // epilogue warps: 4 TMEM lane quarters x 2 column halves
constexpr int NWARPS = 4 + NEPI;
constexpr int ECOLS = TILE_M / (NEPI / 4);   // token columns per epilogue thread (64)
constexpr int ECH = ECOLS / 8;               // 8-column TMEM chunks per block (block-sum path)
constexpr int A_SLOT = TILE_N * 32;    // canonical s8 weight tile per block (4 KB)
constexpr int NA = 4;                  // canonical weight slots
constexpr uint32_t TMEM_COLS = 512;    // two accumulator slots of hi|lo x 128 columns


}  // namespace

struct GemmParams {
    const uint8_t* W;        // weight records [G][nblk][REC]
    const uint8_t* act;      // GEMM activation buffer (token-half major, ql_internal.h)
    float* C;
    int32_t* CS;
    int* err;
    int M, N, nblk, G, ldc;
    int m_tiles, n_tiles, tiles;
    int BPS, STAGES;
    uint32_t stage_bytes, off_act;   // inside a stage: weights of 8 groups, then activations
    uint32_t off_a, off_stages;      // inside dynamic shared memory
};

// Activation stage layout (per stage of BPS blocks, after the weights):
// [half 0 planes: BPS x GEMM_HPLANES][half 1 planes][scales: BPS x 128 fp32];
// each half's hi / lo plane is the canonical K-major B operand of 64 tokens.
constexpr int AREC = GEMM_AREC;
static_assert(GEMM_AREC == 2 * GEMM_HPLANES + TILE_M * 4, "GEMM activation layout");

template <int BITS, bool HALF, bool ZP, bool HP, bool OUT_CS>
__global__ void __launch_bounds__(NWARPS * 32, 1) gemm_kernel(const GemmParams p) {
    constexpr int TB = BITS == 8 ? 512 : 256;
    constexpr int SB = HALF ? 32 : 64;
    constexpr int ZB = ZP ? 16 : 0;
    constexpr int REC = TB + SB + ZB;
    extern __shared__ __align__(1024) uint8_t smem[];
    // barriers: stage_full[S], stage_empty[S], a_full[NA], a_empty[NA], acc_full[2], acc_empty[2], drain
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    uint64_t* stage_full = bars;
    uint64_t* stage_empty = bars + p.STAGES;
    uint64_t* a_full = bars + 2 * p.STAGES;
    uint64_t* a_empty = a_full + NA;
    uint64_t* acc_full = a_empty + NA;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
    uint8_t* a_ring = smem + p.off_a;
    uint8_t* stages = smem + p.off_stages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int spt = (p.nblk + p.BPS - 1) / p.BPS;        // stages per tile

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.STAGES; ++s) {
            mbar_init(smem_u32(&stage_full[s]), 1);
            mbar_init(smem_u32(&stage_empty[s]), NUNPACK + 1 + NEPI);
        }
        for (int a = 0; a < NA; ++a) {
            mbar_init(smem_u32(&a_full[a]), NUNPACK);
            mbar_init(smem_u32(&a_empty[a]), 1);
        }
        for (int k = 0; k < 2; ++k) {
            mbar_init(smem_u32(&acc_full[k]), 1);
            mbar_init(smem_u32(&acc_empty[k]), NEPI);
        }
        mbar_init(smem_u32(drain), 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();   // the next kernel waits for this grid before touching its data
    // Seed both accumulator slots: the MMAs accumulate onto the bit patterns of
    // 1.5*2^31 (hi columns) and 1.5*2^23 (lo columns), so the sums come out of
    // TMEM already in the form the exact int->float conversion needs; the
    // epilogue re-seeds every column right after reading it.
    if (warp >= 4) {
        const uint32_t base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + ((warp - 4) >> 2) * ECOLS;
#pragma unroll
        for (int ac = 0; ac < 2; ++ac)
#pragma unroll
            for (int cc = 0; cc < ECH; ++cc) {
                if (HP) tmem_fill8(base + ac * 256 + cc * 8, static_cast<uint32_t>(HI_SEED));
                tmem_fill8(base + ac * 256 + 128 + cc * 8, static_cast<uint32_t>(LO_SEED));
            }
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp < 4) {
        if (warp == 0) {
            // ------------------------------------------------------------ producer
            // The whole warp runs the loop and waits (it stays converged); lane 0
            // issues the copies.
            int si = 0;        // stage sequence index
            bool pdl_done = false;
            for (int tile = blockIdx.x; tile < p.tiles && __shfl_sync(0xffffffffu, *abort_flag, 0) == 0;
                 tile += gridDim.x) {
                const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
                const int G0 = nt * GROUPS;
                const int groups = min(GROUPS, p.G - G0);
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
                        mbar_arrive_expect_tx(full, (groups * REC + AREC) * nb);
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
            // The whole warp waits (converged); lane 0 issues the MMAs and commits.
            // one MMA per 64-token half and plane (N = 64)
            const uint32_t idesc_hi = make_idesc_i8(TILE_N, TILE_M / 2, true, true);
            const uint32_t idesc_lo = make_idesc_i8(TILE_N, TILE_M / 2, true, !HP);
            int si = 0, bi = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
                for (int ks = 0; ks < spt && ok; ++ks, ++si) {
                    const int s = si % p.STAGES;
                    if (!(ok = warp_wait(smem_u32(&stage_full[s]), (si / p.STAGES) & 1, p.err, abort_flag))) break;
                    const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                    const uint32_t act_base = smem_u32(stages + static_cast<size_t>(s) * p.stage_bytes + p.off_act);
                    for (int j = 0; j < nb; ++j, ++bi) {
                        const int as = bi % NA, ac = bi & 1;
                        if (!(ok = warp_wait(smem_u32(&a_full[as]), (bi / NA) & 1, p.err, abort_flag))) break;
                        if (bi >= 2 &&
                            !(ok = warp_wait(smem_u32(&acc_empty[ac]), ((bi >> 1) - 1) & 1, p.err, abort_flag)))
                            break;
                        tc_fence_after();
                        if (lane == 0) {
                            const uint64_t da = make_smem_desc(smem_u32(a_ring + as * A_SLOT), 2048, 128);
                            const uint32_t d_hi = tmem + ac * 256, d_lo = d_hi + 128;
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const uint32_t pl = act_base + (h * p.BPS + j) * GEMM_HPLANES;
                                if (HP) mma_i8(d_hi + h * 64, da, make_smem_desc(pl, 1024, 128), idesc_hi, 1);   // onto the seeds
                                mma_i8(d_lo + h * 64, da, make_smem_desc(pl + 2048, 1024, 128), idesc_lo, 1);
                            }
                            mma_commit(smem_u32(&acc_full[ac]));
                            mma_commit(smem_u32(&a_empty[as]));
                        }
                        __syncwarp();
                    }
                    if (ok && lane == 0) mma_commit(smem_u32(&stage_empty[s]));
                    __syncwarp();
                }
            }
            // drain: all MMAs issued by lane 0 complete before TMEM is freed
            if (lane == 0) mma_commit(smem_u32(drain));
            __syncwarp();
            mbar_wait(smem_u32(drain), 0, p.err);
        } else {
            // ------------------------------------------------------------ unpack
            const int u = warp - 2;                           // row groups u, u+2, u+4, u+6
            const int g = lane >> 2, t = lane & 3;
            int si = 0, bi = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
                const int nt = tile / p.m_tiles;
                const int groups = min(GROUPS, p.G - nt * GROUPS);
                for (int ks = 0; ks < spt && ok; ++ks, ++si) {
                    const int s = si % p.STAGES;
                    if (!(ok = warp_wait(smem_u32(&stage_full[s]), (si / p.STAGES) & 1, p.err, abort_flag))) break;
                    const uint8_t* wst = stages + static_cast<size_t>(s) * p.stage_bytes;
                    const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                    for (int j = 0; j < nb; ++j, ++bi) {
                        const int as = bi % NA;
                        if (bi >= NA &&
                            !(ok = warp_wait(smem_u32(&a_empty[as]), ((bi / NA) - 1) & 1, p.err, abort_flag)))
                            break;
                        uint8_t* dst = a_ring + as * A_SLOT;
                        for (int gg = u; gg < GROUPS; gg += NUNPACK) {
                            uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
                            if (gg < groups) {
                                const uint8_t* rec = wst + gg * p.BPS * REC + j * REC;
                                if (BITS == 8) {
                                    const uint4 v = *reinterpret_cast<const uint4*>(rec + lane * 16);
                                    a0 = v.x; a1 = v.y; a2 = v.z; a3 = v.w;
                                } else {
                                    const uint2 v = *reinterpret_cast<const uint2*>(rec + lane * 8);
                                    uint32_t c0 = 0x78787878u, c1 = 0x78787878u;
                                    if (ZP) {
                                        const uint32_t z = rec[TB + SB + g];
                                        c0 = (0x80u - (z & 15u)) * 0x01010101u;
                                        c1 = (0x80u - (z >> 4)) * 0x01010101u;
                                    }
                                    a0 = nib_even_s8(v.x, c0);
                                    a1 = nib_odd_s8(v.x, c1);
                                    a2 = nib_even_s8(v.y, c0);
                                    a3 = nib_odd_s8(v.y, c1);
                                }
                            }
                            // canonical offset of (K half kc, 8-row group rg, row r, byte kb):
                            // kc*2048 + rg*128 + r*16 + kb;  rows g / g+8 of group gg are
                            // 8-row groups 2gg / 2gg+1, bytes 4t.. of K halves 0 and 1
                            const int o = (2 * gg) * 128 + g * 16 + 4 * t;
                            *reinterpret_cast<uint32_t*>(dst + o) = a0;
                            *reinterpret_cast<uint32_t*>(dst + o + 128) = a1;
                            *reinterpret_cast<uint32_t*>(dst + 2048 + o) = a2;
                            *reinterpret_cast<uint32_t*>(dst + 2048 + o + 128) = a3;
                        }
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the tensor core
                        __syncwarp();
                        if (lane == 0) mbar_arrive(smem_u32(&a_full[as]));
                    }
                    __syncwarp();
                    if (ok && lane == 0) mbar_arrive(smem_u32(&stage_empty[s]));
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int e = warp - 4;
        const int q = warp & 3;                           // TMEM lane quarter (hardware rule: warp % 4)
        const int cq = e >> 2;                            // token columns ECOLS*cq ..
        const int row = q * 32 + lane;                    // weight row within the tile
        const int g16 = row >> 4, r16 = row & 15;
        const int sidx = 2 * (r16 & 7) + (r16 >> 3);      // this row's entry in a record's scales
        int si = 0, bi = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            const int mt = tile % p.m_tiles, nt = tile / p.m_tiles;
            const int n = nt * TILE_N + row;
            const int groups = min(GROUPS, p.G - nt * GROUPS);
            uint64_t acc[ECOLS / 2];                      // ECOLS token columns as f32x2 pairs
#pragma unroll
            for (int i = 0; i < ECOLS / 2; ++i) acc[i] = 0;
            for (int ks = 0; ks < spt && ok; ++ks, ++si) {
                const int s = si % p.STAGES;
                if (!(ok = warp_wait(smem_u32(&stage_full[s]), (si / p.STAGES) & 1, p.err, abort_flag))) break;
                const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
                const int nb = min(p.BPS, p.nblk - ks * p.BPS);
                for (int j = 0; j < nb; ++j, ++bi) {
                    const int ac = bi & 1;
                    if (!(ok = warp_wait(smem_u32(&acc_full[ac]), (bi >> 1) & 1, p.err, abort_flag))) break;
                    tc_fence_after();
                    float bs = 0.0f;
                    if (g16 < groups) {
                        const uint8_t* rec = st + g16 * p.BPS * REC + j * REC;
                        bs = HALF ? __half2float(reinterpret_cast<const __half*>(rec + TB)[sidx])
                                  : reinterpret_cast<const float*>(rec + TB)[sidx];
                    }
                    const uint64_t bs2 = f2_pack(bs, bs);
                    const float* ascale = reinterpret_cast<const float*>(st + p.off_act + 2 * p.BPS * GEMM_HPLANES +
                                                                         j * GEMM_SCALES) + cq * ECOLS;
                    const uint32_t t_hi = tmem + (static_cast<uint32_t>(q * 32) << 16) + ac * 256 + cq * ECOLS;
                    if constexpr (OUT_CS) {
                        // block sums [M][N][nblk]: a checking output, not a fast path
#pragma unroll 1
                        for (int cc = 0; cc < ECH; ++cc) {
                            uint32_t h8[8], l8[8];
                            if (HP) tmem_ld8(t_hi + cc * 8, h8);
                            tmem_ld8(t_hi + 128 + cc * 8, l8);
                            tmem_wait_ld();
                            if (HP) tmem_fill8(t_hi + cc * 8, static_cast<uint32_t>(HI_SEED));
                            tmem_fill8(t_hi + 128 + cc * 8, static_cast<uint32_t>(LO_SEED));
                            const int m0 = mt * TILE_M + cq * ECOLS + cc * 8;
                            int32_t* dst = p.CS + (static_cast<size_t>(m0) * p.N + n) * p.nblk + ks * p.BPS + j;
#pragma unroll
                            for (int k = 0; k < 8; ++k) {
                                const int32_t lo = static_cast<int32_t>(l8[k]) - LO_SEED;
                                const int32_t cs = HP ? (static_cast<int32_t>(h8[k]) - HI_SEED) * 256 + lo : lo;
                                if (m0 + k < p.M && g16 < groups) *dst = cs;
                                dst += static_cast<size_t>(p.N) * p.nblk;
                            }
                        }
                    } else {
                    // 8-column chunks; the next chunk's TMEM loads are in flight while
                    // this chunk is converted and rescaled, and each chunk's columns
                    // are re-seeded for the slot's next block right after they are read
                    uint32_t hv[2][8], lv[2][8];
                    if (HP) tmem_ld8(t_hi, hv[0]);
                    tmem_ld8(t_hi + 128, lv[0]);
                    tmem_wait_ld();
#pragma unroll
                    for (int cc = 0; cc < ECH; ++cc) {
                        const int cur = cc & 1;
                        if (cc < ECH - 1) {
                            if (HP) tmem_ld8(t_hi + (cc + 1) * 8, hv[cur ^ 1]);
                            tmem_ld8(t_hi + 128 + (cc + 1) * 8, lv[cur ^ 1]);
                        }
                        if (HP) tmem_fill8(t_hi + cc * 8, static_cast<uint32_t>(HI_SEED));
                        tmem_fill8(t_hi + 128 + cc * 8, static_cast<uint32_t>(LO_SEED));
#pragma unroll
                        for (int k = 0; k < 8; k += 4) {
                            const float4 a4 = lds_f4(ascale + cc * 8 + k);
                            uint64_t y0, y1;
                            if (HP) {
                                y0 = cs_to_f2(static_cast<int32_t>(hv[cur][k]), static_cast<int32_t>(hv[cur][k + 1]),
                                              static_cast<int32_t>(lv[cur][k]), static_cast<int32_t>(lv[cur][k + 1]));
                                y1 = cs_to_f2(static_cast<int32_t>(hv[cur][k + 2]), static_cast<int32_t>(hv[cur][k + 3]),
                                              static_cast<int32_t>(lv[cur][k + 2]), static_cast<int32_t>(lv[cur][k + 3]));
                            } else {
                                const uint64_t neg = f2_pack(-12582912.0f, -12582912.0f);   // -1.5*2^23
                                y0 = f2_add(i2_pack(static_cast<int32_t>(lv[cur][k]), static_cast<int32_t>(lv[cur][k + 1])), neg);
                                y1 = f2_add(i2_pack(static_cast<int32_t>(lv[cur][k + 2]), static_cast<int32_t>(lv[cur][k + 3])), neg);
                            }
                            const int i0 = (cc * 8 + k) >> 1;
                            acc[i0] = f2_fma(f2_pack(a4.x, a4.y), f2_mul(y0, bs2), acc[i0]);
                            acc[i0 + 1] = f2_fma(f2_pack(a4.z, a4.w), f2_mul(y1, bs2), acc[i0 + 1]);
                        }
                        if (cc < ECH - 1) tmem_wait_ld();
                    }
                    }
                    // the slot is read and re-seeded: hand it back to the MMA warp
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&acc_empty[ac]));
                }
                fence_proxy_async_smem();      // scale reads of this stage before its refill
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(smem_u32(&stage_empty[s]));
            }
            if (!ok || OUT_CS) continue;
            // store C[m, n] for this thread's 64 token columns (lanes = consecutive n)
            if (g16 < groups) {
#pragma unroll
                for (int i = 0; i < ECOLS / 2; ++i) {
                    const int m = mt * TILE_M + cq * ECOLS + 2 * i;
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TMEM_COLS) : "memory");
}

// ------------------------------------------------------------------ host side

int* device_error_word();   // ql_api.cu

static int g_gemm_sms = 0;

template <int BITS, bool HALF, bool ZP, bool HP, bool OUT_CS>
static cudaError_t gemm_launch(const GemmParams& p0, cudaStream_t stream) {
    constexpr int REC = (BITS == 8 ? 512 : 256) + (HALF ? 32 : 64) + (ZP ? 16 : 0);
    GemmParams p = p0;
    p.BPS = 4;
    p.off_act = GROUPS * p.BPS * REC;
    p.stage_bytes = (p.off_act + p.BPS * AREC + 1023) & ~1023u;
    const uint32_t bar_bytes = 1024;                       // barriers, abort flag, TMEM address
    p.off_a = bar_bytes;
    p.off_stages = p.off_a + NA * A_SLOT;
    p.STAGES = 4;
    while (p.STAGES > 2 && p.off_stages + static_cast<size_t>(p.STAGES) * p.stage_bytes > 220 * 1024) --p.STAGES;
    const size_t smem = p.off_stages + static_cast<size_t>(p.STAGES) * p.stage_bytes;
    if (smem > 227 * 1024 || (p.off_act % 16) || (REC % 16)) return cudaErrorInvalidConfiguration;
    auto kern = gemm_kernel<BITS, HALF, ZP, HP, OUT_CS>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    if (g_gemm_sms == 0) {
        cudaDeviceGetAttribute(&g_gemm_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_gemm_sms <= 0) g_gemm_sms = 148;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(p.tiles, g_gemm_sms));
    cfg.blockDim = dim3(NWARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <bool HP, bool OUT_CS>
static cudaError_t gemm_dispatch(const Weight* w, const GemmParams& p, cudaStream_t stream) {
    if (w->bits == 8) {
        if (w->scale_half) return gemm_launch<8, true, false, HP, OUT_CS>(p, stream);
        return gemm_launch<8, false, false, HP, OUT_CS>(p, stream);
    }
    if (w->has_zp) {
        if (w->scale_half) return gemm_launch<4, true, true, HP, OUT_CS>(p, stream);
        return gemm_launch<4, false, true, HP, OUT_CS>(p, stream);
    }
    if (w->scale_half) return gemm_launch<4, true, false, HP, OUT_CS>(p, stream);
    return gemm_launch<4, false, false, HP, OUT_CS>(p, stream);
}

size_t gemm_act_bytes(int M, int nblk) {
    const size_t m_tiles = static_cast<size_t>((M + TILE_M - 1) / TILE_M);
    return m_tiles * static_cast<size_t>(nblk) * AREC;
}

cudaError_t launch_gemm(const Weight* w, const uint8_t* act, int M, bool hi_prec, float* C, int ldc,
                        int32_t* cs, cudaStream_t stream) {
    if (prefill_kernel() != QL_PREFILL_I8 && gemm16_supports(w, hi_prec))
        return launch_gemm16(w, act, M, C, ldc, cs, stream);
    GemmParams p = {};
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
    p.m_tiles = (M + TILE_M - 1) / TILE_M;
    p.n_tiles = (w->N + TILE_N - 1) / TILE_N;
    p.tiles = p.m_tiles * p.n_tiles;
    if (cs) return hi_prec ? gemm_dispatch<true, true>(w, p, stream) : gemm_dispatch<false, true>(w, p, stream);
    return hi_prec ? gemm_dispatch<true, false>(w, p, stream) : gemm_dispatch<false, false>(w, p, stream);
}

}  // namespace ql
