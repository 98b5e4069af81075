// ql_gemv4.cu -- decode kernel for INT4 weights at one or two tokens, on the
// CUDA cores' 4-way byte dot products (dp4a) instead of tensor-core MMAs.
//
// Computes C[m, n] = i4_matmul(A)[m, n] (kernel/quantized_matmul.cpp:270-318,
// tile_kernel) bit-identically to the reference, from the same packed records
// as ql_gemv.cu and the same quantized-activation records (ql_quant.cu).
//
// Why.  At M <= 2 the m16n8k32 MMA of ql_gemv.cu uses one or two of its eight
// token columns, yet every lane still unpacks its nibbles to signed bytes and
// converts and rescales four outputs per block: about 55 warp instructions per
// 16x32 record on B200, which leaves that kernel issue-bound at ~0.4 of HBM
// bandwidth.  Here a thread owns two rows of a record and works on the packed
// nibbles in place:
//   * a record's 32 bytes of rows g and g+8 hold b = q(g) + 16*q(g+8) per
//     byte; x & 0xF0F0F0F0 = 16*q(g+8) -- one mask per 8 weights, no
//     per-weight zero point;
//   * dp4a of the activation planes (hi - 128 signed, lo unsigned, or q8)
//     against b and against 16*q(g+8) gives, exactly in int32 (every partial
//     sum below 2^31 in magnitude),
//         sum q16*q(g+8) = (256*S_hi(16q') + S_lo(16q')) >> 4,
//         sum q16*q(g)   = 256*(S_hi(b) - S_hi(16q')) + (S_lo(b) - S_lo(16q'));
//   * the zero point comes out through the activation side:
//     cs = sum q16*(q - zp) = sum q16*q - zp * sum q16, where the quantizer
//     stores sum q16 per (token, block) in the record;
//   * (float)cs * bscale and acc = fma(ascale, f, acc) in ascending block order,
//     the reference's FP32 chain.
//
// Work split (as in ql_gemv.cu): a producer warp streams stages of BPS blocks
// (one bulk copy per row group and one for the activation records, no
// multicast); a consumer warp owns a quad of four row groups (lane = 8 *
// row group + g) and, with a K split, every SPLIT-th stage, handing the running
// accumulators to the warp of the next stage through a shared-memory relay
// slot guarded by an mbarrier.  Slots are used in phase order by one warp each;
// every wait is bounded (the device wait limit) and records QL_ETIMEOUT.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include "ql_common.cuh"
#include "ql_internal.h"

namespace ql {

namespace {

constexpr int D4_C = 8;                       // blocks whose f values are held before the chain

struct Dp4aParams {
    const uint8_t* W;        // weight records [G][nblk][REC]
    const uint8_t* q;        // activation records [nblk][QREC]
    float* C;
    int32_t* CS;
    int* err;
    int M, N, nblk, G, ldc;
    int TPB, TPBA, QREC;
    int Q4, SPLIT, BPS, STAGES;   // row-group quads per CTA, K split, blocks per stage, ring depth
    int PROD;                     // producer warps (producer p issues the stages p, p + PROD, ...)
    uint32_t stage_bytes, off_Q, off_relay, off_stages;
};

__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {     // signed a bytes x unsigned b bytes
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {     // unsigned x unsigned
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__host__ __device__ __forceinline__ int d4_relay_slots(int split) { return split < 2 ? 2 : split; }

// Block sums of rows g and g + 8 of one record for MTOK tokens:
//   cs[0][m] = sum_k q16[m][k] * (q[g][k] - zp[g]),   cs[1][m] likewise for row g + 8,
// and the two rows' block scales.  rec is the record (nibbles, scales, zero
// points), qrec the block's activation record, q_sum the offset of its block
// sums of q16 inside the record.  Exact in int32 (see the file comment).
template <bool HALF, bool ZP, int MTOK, bool HP>
__device__ __forceinline__ void d4_record(const uint8_t* rec, const uint8_t* qrec, int g, int q_sum,
                                          int (&cs)[2][MTOK], float& bs0, float& bs1) {
    constexpr int TB = 256, SB = HALF ? 32 : 64;
    const uint4 wa = *reinterpret_cast<const uint4*>(rec + 32 * g);
    const uint4 wb = *reinterpret_cast<const uint4*>(rec + 32 * g + 16);
    const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};   // q(g) + 16 q(g+8)
    uint32_t o[8];                                 // 16*q of row g+8
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = w[k] & 0xF0F0F0F0u;
    if (HALF) {
        const __half2 hs = *reinterpret_cast<const __half2*>(rec + TB + 4 * g);
        bs0 = __low2float(hs);
        bs1 = __high2float(hs);
    } else {
        const float2 fs = *reinterpret_cast<const float2*>(rec + TB + 8 * g);
        bs0 = fs.x;
        bs1 = fs.y;
    }
    int zg = 8, zg8 = 8;
    if (ZP) {
        const uint32_t z = rec[TB + SB + g];
        zg = static_cast<int>(z & 15u);
        zg8 = static_cast<int>(z >> 4);
    }
#pragma unroll
    for (int m = 0; m < MTOK; ++m) {
        // sums against the whole bytes (w) and against their high nibbles (o)
        int shw = 0, slw = 0, sho = 0, slo = 0;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            if (HP) {
                // slot t: hs of k 4t.. and 16+4t.., then lo of the same k
                const uint4 a = *reinterpret_cast<const uint4*>(qrec + (m * 4 + t) * 16);
                shw = dp4a_su(a.x, w[2 * t], shw);
                sho = dp4a_su(a.x, o[2 * t], sho);
                slw = dp4a_uu(a.z, w[2 * t], slw);
                slo = dp4a_uu(a.z, o[2 * t], slo);
                shw = dp4a_su(a.y, w[2 * t + 1], shw);
                sho = dp4a_su(a.y, o[2 * t + 1], sho);
                slw = dp4a_uu(a.w, w[2 * t + 1], slw);
                slo = dp4a_uu(a.w, o[2 * t + 1], slo);
            } else {
                const uint2 a = *reinterpret_cast<const uint2*>(qrec + (m * 4 + t) * 8);
                shw = dp4a_su(a.x, w[2 * t], shw);
                sho = dp4a_su(a.x, o[2 * t], sho);
                shw = dp4a_su(a.y, w[2 * t + 1], shw);
                sho = dp4a_su(a.y, o[2 * t + 1], sho);
            }
        }
        // row g: whole bytes minus high nibbles; row g+8: high nibbles / 16
        // (every term a multiple of 16); then the zero point
        const int sq = *reinterpret_cast<const int*>(qrec + q_sum + 4 * m);
        const int c0 = HP ? (shw - sho) * 256 + (slw - slo) : shw - sho;
        const int c1 = (HP ? (sho * 256 + slo) : sho) >> 4;
        cs[0][m] = c0 - zg * sq;
        cs[1][m] = c1 - zg8 * sq;
    }
}

}  // namespace

template <bool HALF, bool ZP, int MTOK, bool HP, bool OUT_CS>
__global__ void __launch_bounds__(384) decode_dp4a_kernel(const Dp4aParams p) {
    constexpr int TB = 256, SB = HALF ? 32 : 64, ZB = ZP ? 16 : 0, REC = TB + SB + ZB;
    constexpr int LB = HP ? 16 : 8;                 // activation bytes per fragment slot
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty_bar = full_bar + p.STAGES;
    uint64_t* relay_bar = empty_bar + p.STAGES;
    uint8_t* stages = smem + p.off_stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int consumers = p.Q4 * p.SPLIT;
    const int NS = d4_relay_slots(p.SPLIT);
    const int R = 4 * p.Q4;                         // row groups per CTA
    const int G0 = blockIdx.x * R;
    const int active = min(R, p.G - G0);
    const int active_q = (active + 3) / 4;          // quads holding at least one row group
    const int nst = (p.nblk + p.BPS - 1) / p.BPS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.STAGES; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), active_q);
        }
        for (int k = 0; k < p.Q4 * NS; ++k) mbar_init(smem_u32(&relay_bar[k]), 32);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp >= consumers) {
        // ----------------------------------------------------------- producers
        // producer pr issues the stages i = pr (mod PROD); STAGES is a multiple
        // of PROD, so it waits only on ring slots it filled itself
        if (lane != 0) return;
        const int pr = warp - consumers;
        auto issue = [&](int i, bool weights, bool acts) {
            const int s = i % p.STAGES;
            const uint32_t base = smem_u32(stages + static_cast<size_t>(s) * p.stage_bytes);
            const uint32_t full = smem_u32(&full_bar[s]);
            const int b0 = i * p.BPS;
            const int nb = min(p.BPS, p.nblk - b0);
            if (weights) {
                mbar_arrive_expect_tx(full, (active * REC + p.QREC) * nb);
                for (int w = 0; w < active; ++w) {
                    const size_t rec0 = static_cast<size_t>(G0 + w) * p.nblk + b0;
                    bulk_g2s(base + w * p.BPS * REC, p.W + rec0 * REC, nb * REC, full);
                }
            }
            if (acts) bulk_g2s(base + p.off_Q, p.q + static_cast<size_t>(b0) * p.QREC, nb * p.QREC, full);
        };
        const int first = min(p.STAGES, nst);
        for (int i = pr; i < first; i += p.PROD) issue(i, true, false);
        pdl_wait();                                   // activations come from the previous grid
        for (int i = pr; i < first; i += p.PROD) issue(i, false, true);
        for (int i = first + ((pr - first) % p.PROD + p.PROD) % p.PROD; i < nst; i += p.PROD) {
            const int s = i % p.STAGES;
            if (!mbar_wait(smem_u32(&empty_bar[s]), ((i / p.STAGES) - 1) & 1, p.err)) {
                for (int j = i - p.STAGES; j < i; j += p.PROD)       // let this producer's copies land
                    if (j >= 0 && !mbar_wait(smem_u32(&full_bar[j % p.STAGES]), (j / p.STAGES) & 1, p.err)) break;
                return;
            }
            issue(i, true, true);
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int qd = warp / p.SPLIT;                  // quad of row groups within the CTA
    const int split = warp % p.SPLIT;               // stages i = split, split + SPLIT, ...
    if (qd >= active_q) return;
    const int rr = lane >> 3, g = lane & 7;
    const int r = 4 * qd + rr;                      // row group within the CTA (< R)
    const bool row_ok = r < active;
    const int G = G0 + r;
    float* relay = reinterpret_cast<float*>(smem + p.off_relay) + static_cast<size_t>(qd) * NS * 32 * 4;
    const int q_scale = p.TPB * 4 * LB;             // activation scales inside a record
    const int q_sum = q_scale + p.TPBA * 4;         // block sums of the quantized values

    float acc[2][MTOK];                             // rows g, g+8
#pragma unroll
    for (int m = 0; m < MTOK; ++m) { acc[0][m] = 0.0f; acc[1][m] = 0.0f; }

    for (int i = split; i < nst; i += p.SPLIT) {
        const int s = i % p.STAGES;
        if (!mbar_wait(smem_u32(&full_bar[s]), (i / p.STAGES) & 1, p.err)) return;
        const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
        const uint8_t* Wst = st + r * p.BPS * REC;
        const uint8_t* Qst = st + p.off_Q;
        const int b0 = i * p.BPS;
        const int nb = min(p.BPS, p.nblk - b0);
        bool need_relay = !OUT_CS && p.SPLIT > 1 && i > 0;

        for (int j0 = 0; j0 < nb; j0 += D4_C) {
            float f[D4_C][2][MTOK], as[D4_C][MTOK];
#pragma unroll
            for (int u = 0; u < D4_C; ++u) {
                const int j = min(j0 + u, nb - 1);           // slots past nb are discarded
                const uint8_t* qrec = Qst + j * p.QREC;
                int cs[2][MTOK];
                float bs0, bs1;
                d4_record<HALF, ZP, MTOK, HP>(Wst + j * REC, qrec, g, q_sum, cs, bs0, bs1);
#pragma unroll
                for (int m = 0; m < MTOK; ++m) {
                    if (OUT_CS) {
                        if (j0 + u < nb && row_ok && m < p.M) {
                            const int n0 = G * 16 + g;
                            p.CS[(static_cast<size_t>(m) * p.N + n0) * p.nblk + b0 + j] = cs[0][m];
                            p.CS[(static_cast<size_t>(m) * p.N + n0 + 8) * p.nblk + b0 + j] = cs[1][m];
                        }
                        continue;
                    }
                    f[u][0][m] = __fmul_rn(__int2float_rn(cs[0][m]), bs0);     // (float)cs * bscale
                    f[u][1][m] = __fmul_rn(__int2float_rn(cs[1][m]), bs1);
                    as[u][m] = *reinterpret_cast<const float*>(qrec + q_scale + 4 * m);
                }
            }
            // the stage's last reads are done: hand it back before the serial chain
            if (j0 + D4_C >= nb) {
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
            }
            if (OUT_CS) continue;
            if (need_relay) {
                need_relay = false;
                const int slot = (i - 1) % NS;
                if (!mbar_wait(smem_u32(&relay_bar[qd * NS + slot]), ((i - 1) / NS) & 1, p.err)) return;
                const float4 v = *reinterpret_cast<const float4*>(relay + (slot * 32 + lane) * 4);
                acc[0][0] = v.x;
                acc[1][0] = v.y;
                if (MTOK > 1) { acc[0][MTOK - 1] = v.z; acc[1][MTOK - 1] = v.w; }
            }
#pragma unroll
            for (int u = 0; u < D4_C; ++u) {
                if (j0 + u >= nb) break;
#pragma unroll
                for (int m = 0; m < MTOK; ++m) {
                    acc[0][m] = __fmaf_rn(as[u][m], f[u][0][m], acc[0][m]);
                    acc[1][m] = __fmaf_rn(as[u][m], f[u][1][m], acc[1][m]);
                }
            }
        }
        if (OUT_CS) continue;
        if (p.SPLIT > 1 && i + 1 < nst) {
            // hand the accumulators to the warp of stage i + 1
            const int slot = i % NS;
            *reinterpret_cast<float4*>(relay + (slot * 32 + lane) * 4) =
                make_float4(acc[0][0], acc[1][0], acc[0][MTOK - 1], acc[1][MTOK - 1]);
            mbar_arrive(smem_u32(&relay_bar[qd * NS + slot]));
        }
        if (i + 1 >= nst && row_ok) {
            // this warp ran the last stage: store the outputs
            const int n0 = G * 16 + g;
#pragma unroll
            for (int m = 0; m < MTOK; ++m) {
                if (m < p.M) {
                    p.C[static_cast<size_t>(m) * p.ldc + n0] = acc[0][m];
                    p.C[static_cast<size_t>(m) * p.ldc + n0 + 8] = acc[1][m];
                }
            }
        }
    }
}

// Chain variant for layers with few row groups (N < 8192: the attention and
// down projections of a 27B-class layer).  A CTA owns R (1, 2 or 4) row groups
// over the whole K range, so the grid has G / R CTAs instead of G / 4, and the
// ordered FP32 chain leaves the consumers:
//   * PROD producer warps stream stages of BPS blocks as above, producer p
//     the stages p, p + PROD, ... (measured on B200: one issuing thread's
//     bulk copies stream at most ~16-19 GB/s however deep its ring, two
//     ~26 GB/s and four ~31 GB/s, so a CTA that owns one row group needs
//     several to keep HBM busy);
//   * consumer warp w takes stages w, w + CONS, ...; its lanes cover four
//     (row group, block) units per pass (lane = 8 * unit + g; a unit is one
//     record, 4 / R blocks of each of the R row groups per pass) and write the
//     rounded products f = (float)cs * bscale, and the blocks' activation
//     scales, into a ring of FS f-slots in shared memory;
//   * one chain warp walks the f-slots in stage order and runs
//     acc = fma(ascale, f, acc) in ascending block order, one lane per
//     (token, row) -- the reference's chain, with no hand-over between warps;
//     it stores the outputs at the end.
// f-slot layout: [MTOK][16 R][FSTR] floats (token, row of the CTA, block of
// the stage; FSTR = BPS rounded up to 16, plus 4, so that a chain lane reads
// sixteen blocks with four 16-byte loads inside its row and eight lanes hit
// distinct banks), then [MTOK][FSTR] activation scales.
struct ChainParams {
    const uint8_t* W;        // weight records [G][nblk][REC]
    const uint8_t* q;        // activation records [nblk][QREC]
    float* C;
    int* err;
    int M, N, nblk, G, ldc;
    int TPB, TPBA, QREC;
    int R, CONS, PROD, BPS, STAGES, FS;   // row groups per CTA, consumer and producer warps, blocks per
                                          // stage, ring depths
    uint32_t stage_bytes, off_Q, off_f, fslot_floats, fstr, off_stages;
};

template <bool HALF, bool ZP, int MTOK, bool HP>
__global__ void __launch_bounds__(416) decode_dp4a_chain_kernel(const ChainParams p) {
    constexpr int REC = 256 + (HALF ? 32 : 64) + (ZP ? 16 : 0);
    constexpr int LB = HP ? 16 : 8;
    constexpr int PU = 4;                           // passes held in registers before the stores
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty_bar = full_bar + p.STAGES;
    uint64_t* ffull_bar = empty_bar + p.STAGES;
    uint64_t* fempty_bar = ffull_bar + p.FS;
    float* fring = reinterpret_cast<float*>(smem + p.off_f);
    uint8_t* stages = smem + p.off_stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = p.R;
    const int rows = 16 * R;                        // row positions per token in an f-slot
    const int G0 = blockIdx.x * R;
    const int active = min(R, p.G - G0);
    const int nst = (p.nblk + p.BPS - 1) / p.BPS;
    const int FSTR = p.fstr;                        // floats per (token, row) in an f-slot
    const int as_off = MTOK * rows * FSTR;          // activation scales inside an f-slot

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.STAGES; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        for (int k = 0; k < p.FS; ++k) {
            mbar_init(smem_u32(&ffull_bar[k]), 32);
            mbar_init(smem_u32(&fempty_bar[k]), 32);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp > p.CONS) {
        // ----------------------------------------------------------- producers
        // producer pr issues the stages i = pr (mod PROD) and, as STAGES is a
        // multiple of PROD, waits only on ring slots it filled itself
        if (lane != 0) return;
        const int pr = warp - p.CONS - 1;
        auto issue = [&](int i, bool weights, bool acts) {
            const int s = i % p.STAGES;
            const uint32_t base = smem_u32(stages + static_cast<size_t>(s) * p.stage_bytes);
            const uint32_t full = smem_u32(&full_bar[s]);
            const int b0 = i * p.BPS;
            const int nb = min(p.BPS, p.nblk - b0);
            if (weights) {
                mbar_arrive_expect_tx(full, (active * REC + p.QREC) * nb);
                for (int w = 0; w < active; ++w) {
                    const size_t rec0 = static_cast<size_t>(G0 + w) * p.nblk + b0;
                    bulk_g2s(base + w * p.BPS * REC, p.W + rec0 * REC, nb * REC, full);
                }
            }
            if (acts) bulk_g2s(base + p.off_Q, p.q + static_cast<size_t>(b0) * p.QREC, nb * p.QREC, full);
        };
        const int first = min(p.STAGES, nst);
        for (int i = pr; i < first; i += p.PROD) issue(i, true, false);
        pdl_wait();                                   // activations come from the previous grid
        for (int i = pr; i < first; i += p.PROD) issue(i, false, true);
        for (int i = first + ((pr - first) % p.PROD + p.PROD) % p.PROD; i < nst; i += p.PROD) {
            const int s = i % p.STAGES;
            if (!mbar_wait(smem_u32(&empty_bar[s]), ((i / p.STAGES) - 1) & 1, p.err)) {
                for (int j = i - p.STAGES; j < i; j += p.PROD)       // let this producer's copies land
                    if (j >= 0 && !mbar_wait(smem_u32(&full_bar[j % p.STAGES]), (j / p.STAGES) & 1, p.err)) break;
                return;
            }
            issue(i, true, true);
        }
        return;
    }

    if (warp == p.CONS) {
        // --------------------------------------------------------------- chain
        // lane + 32 c = m * rows + row, c < 4 (rows * MTOK <= 128)
        const int chains = rows * MTOK;
        const int cpl = (chains + 31) / 32;
        int fo[4], ao[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int idx = min(lane + 32 * c, chains - 1);
            fo[c] = idx * FSTR;
            ao[c] = as_off + (idx / rows) * FSTR;
        }
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int i = 0; i < nst; ++i) {
            const int k = i % p.FS;
            if (!mbar_wait(smem_u32(&ffull_bar[k]), (i / p.FS) & 1, p.err)) return;
            const float* fs = fring + static_cast<size_t>(k) * p.fslot_floats;
            const int nb = min(p.BPS, p.nblk - i * p.BPS);
            // 16 blocks at a time: all loads first, then the dependent FMAs
            for (int j0 = 0; j0 < nb; j0 += 16) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (c >= cpl) break;
                    float4 fv[4], av[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        fv[q] = *reinterpret_cast<const float4*>(fs + fo[c] + j0 + 4 * q);
                        av[q] = *reinterpret_cast<const float4*>(fs + ao[c] + j0 + 4 * q);
                    }
                    if (j0 + 16 <= nb) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            acc[c] = __fmaf_rn(av[q].x, fv[q].x, acc[c]);
                            acc[c] = __fmaf_rn(av[q].y, fv[q].y, acc[c]);
                            acc[c] = __fmaf_rn(av[q].z, fv[q].z, acc[c]);
                            acc[c] = __fmaf_rn(av[q].w, fv[q].w, acc[c]);
                        }
                    } else {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int j = j0 + 4 * q;
                            if (j < nb) acc[c] = __fmaf_rn(av[q].x, fv[q].x, acc[c]);
                            if (j + 1 < nb) acc[c] = __fmaf_rn(av[q].y, fv[q].y, acc[c]);
                            if (j + 2 < nb) acc[c] = __fmaf_rn(av[q].z, fv[q].z, acc[c]);
                            if (j + 3 < nb) acc[c] = __fmaf_rn(av[q].w, fv[q].w, acc[c]);
                        }
                    }
                }
            }
            mbar_arrive(smem_u32(&fempty_bar[k]));
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int idx = lane + 32 * c;
            if (idx >= chains) break;
            const int m = idx / rows, row = idx % rows;
            const int rr = row >> 4;
            if (rr >= active || m >= p.M) continue;
            p.C[static_cast<size_t>(m) * p.ldc + (G0 + rr) * 16 + (row & 15)] = acc[c];
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    if (warp >= nst) return;                        // no stage for this warp
    const int upp = 4 / R;                          // blocks per pass
    const int x = lane >> 3, g = lane & 7;
    const int rr = x / upp, bb = x % upp;           // row group and block of this lane's unit
    const bool row_ok = rr < active;
    const int q_scale = p.TPB * 4 * LB;             // activation scales inside a record
    const int q_sum = q_scale + p.TPBA * 4;         // block sums of the quantized values
    for (int i = warp; i < nst; i += p.CONS) {
        const int s = i % p.STAGES, k = i % p.FS;
        if (!mbar_wait(smem_u32(&full_bar[s]), (i / p.STAGES) & 1, p.err)) return;
        if (i >= p.FS && !mbar_wait(smem_u32(&fempty_bar[k]), ((i / p.FS) - 1) & 1, p.err)) return;
        const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
        const uint8_t* Wst = st + rr * p.BPS * REC;
        const uint8_t* Qst = st + p.off_Q;
        float* fs = fring + static_cast<size_t>(k) * p.fslot_floats;
        const int nb = min(p.BPS, p.nblk - i * p.BPS);
        for (int j0 = 0; j0 < nb; j0 += PU * upp) {
            float f0[PU][MTOK], f1[PU][MTOK];
#pragma unroll
            for (int u = 0; u < PU; ++u) {
                const int j = min(j0 + u * upp + bb, nb - 1);      // slots past nb are discarded
                int cs[2][MTOK];
                float bs0, bs1;
                d4_record<HALF, ZP, MTOK, HP>(Wst + j * REC, Qst + j * p.QREC, g, q_sum, cs, bs0, bs1);
#pragma unroll
                for (int m = 0; m < MTOK; ++m) {
                    f0[u][m] = __fmul_rn(__int2float_rn(cs[0][m]), bs0);     // (float)cs * bscale
                    f1[u][m] = __fmul_rn(__int2float_rn(cs[1][m]), bs1);
                }
            }
#pragma unroll
            for (int u = 0; u < PU; ++u) {
                const int j = j0 + u * upp + bb;
                if (j >= nb) continue;
#pragma unroll
                for (int m = 0; m < MTOK; ++m) {
                    float* fr = fs + (m * rows + rr * 16 + g) * FSTR + j;
                    fr[0] = row_ok ? f0[u][m] : 0.0f;
                    fr[8 * FSTR] = row_ok ? f1[u][m] : 0.0f;
                }
                if (rr == 0 && g < MTOK)
                    fs[as_off + g * FSTR + j] = *reinterpret_cast<const float*>(Qst + j * p.QREC + q_scale + 4 * g);
            }
        }
        // the stage's reads are done: hand it back to the producer, the f-slot to the chain
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
        mbar_arrive(smem_u32(&ffull_bar[k]));
    }
}

// ------------------------------------------------------------------ host side

int* device_error_word();   // ql_api.cu

namespace {

struct D4Config {
    int Q4, SPLIT, BPS, STAGES, PROD;
};

int d4_sms() {
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

int d4_stage_bytes(int R, int BPS, int rec, int qrec) { return (R * BPS * rec + BPS * qrec + 127) & ~127; }

// Configuration from measurements on B200 (INT4, one and two tokens, K = 4096
// and 5120, 12288 to 151936 rows): one quad of row groups per CTA, the K
// range split over 4 consumer warps in stages of 8 blocks; 4 stages in the
// ring when every SM holds three or more quads' CTAs (about 4 CTAs resident per
// SM, 22 us for 34816 x 5120 and 62 us for 151936 x 4096 at one token), 8
// stages below that (13 us for 17408 x 5120).  Deeper stages (16 blocks),
// two-warp splits and 8-warp splits each measured slower.  Layers that give
// fewer than 128 quads take the chain variant (use_chain).
D4Config d4_plan(int G, int nblk, int rec, int qrec, int mtok) {
    const int sms = d4_sms();
    const long long quads = (G + 3) / 4;
    D4Config c;
    c.Q4 = 1;
    c.SPLIT = 4;
    c.BPS = D4_C;
    c.STAGES = quads >= 3LL * sms ? 4 : 8;
    // Two producer warps at one token, or when few quads share an SM (one
    // issuing thread's copies stream at most ~16-19 GB/s); measured on B200:
    // 17408 x 5120 14.6 -> 11.9 us (M = 1) and 16.2 -> 14.7 us (M = 2),
    // 34816 x 5120 20.9 -> 19.5 us and 151936 x 4096 66.5 -> 61.1 us at M = 1,
    // but 90 -> 101 us for 151936 x 4096 at M = 2; four producers were no better.
    c.PROD = (mtok == 1 || quads < 3LL * sms) ? 2 : 1;
    while (c.SPLIT > 1 && (nblk + c.BPS - 1) / c.BPS < 2 * c.SPLIT) c.SPLIT /= 2;
    if (c.STAGES % c.SPLIT) c.STAGES = ((c.STAGES + c.SPLIT - 1) / c.SPLIT) * c.SPLIT;
    if (c.STAGES < 2) c.STAGES = 2;
    (void)rec;
    (void)qrec;
    // Tuning override "Q4,SPLIT,BPS,STAGES[,PROD]" (0 keeps the planner's
    // value); the launch checks reject values that break the kernel's invariants.
    if (const char* env = std::getenv("BREEZE_QL_DP4A_CONFIG")) {
        int q = 0, sp = 0, b = 0, st = 0, pd = 0;
        if (std::sscanf(env, "%d,%d,%d,%d,%d", &q, &sp, &b, &st, &pd) >= 4) {
            if (q > 0) c.Q4 = q;
            if (sp > 0) c.SPLIT = sp;
            if (b > 0) c.BPS = b;
            if (st > 0) c.STAGES = st;
            if (pd > 0) c.PROD = pd;
        }
    }
    return c;
}

template <bool HALF, bool ZP, int MTOK, bool HP, bool OUT_CS>
cudaError_t d4_launch(const Dp4aParams& p0, cudaStream_t stream, bool pdl) {
    constexpr int REC = 256 + (HALF ? 32 : 64) + (ZP ? 16 : 0);
    Dp4aParams p = p0;
    const D4Config c = d4_plan(p.G, p.nblk, REC, p.QREC, MTOK);
    p.Q4 = c.Q4;
    p.SPLIT = c.SPLIT;
    p.BPS = c.BPS;
    p.STAGES = c.STAGES;
    p.PROD = c.PROD;
    const int R = 4 * c.Q4;
    p.off_Q = R * c.BPS * REC;
    p.stage_bytes = d4_stage_bytes(R, c.BPS, REC, p.QREC);
    const int NS = d4_relay_slots(c.SPLIT);
    const uint32_t bar_bytes = (2 * c.STAGES + c.Q4 * NS) * 8;
    p.off_relay = (bar_bytes + 127) & ~127u;
    const uint32_t relay_bytes = c.Q4 * NS * 32 * 16;
    p.off_stages = (p.off_relay + relay_bytes + 127) & ~127u;
    const size_t smem = p.off_stages + static_cast<size_t>(c.STAGES) * p.stage_bytes;
    const int consumers = c.Q4 * c.SPLIT;
    // the carve-up must fit the SM and keep the invariants the kernel relies on
    if (smem > 227 * 1024 || c.BPS < 1 || c.STAGES < 2 || c.Q4 < 1 || c.Q4 > 2 || c.SPLIT < 1 || c.SPLIT > 8 ||
        consumers > 8 || (c.STAGES % c.SPLIT) || c.PROD < 1 || c.PROD > 4 || (c.STAGES % c.PROD) ||
        (p.QREC % 16) || (REC % 16) || (p.off_Q % 16))
        return cudaErrorInvalidConfiguration;
    auto kern = decode_dp4a_kernel<HALF, ZP, MTOK, HP, OUT_CS>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.G + R - 1) / R);
    cfg.blockDim = dim3(32 * (consumers + c.PROD));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <bool HP, bool OUT_CS>
cudaError_t d4_dispatch(const Weight* w, const Dp4aParams& p, int M, cudaStream_t stream, bool pdl) {
#define QL_D4(HALF, ZP)                                                                     \
    return M == 1 ? d4_launch<HALF, ZP, 1, HP, OUT_CS>(p, stream, pdl)                      \
                  : d4_launch<HALF, ZP, 2, HP, OUT_CS>(p, stream, pdl)
    if (w->has_zp) {
        if (w->scale_half) QL_D4(true, true);
        QL_D4(false, true);
    }
    if (w->scale_half) QL_D4(true, false);
    QL_D4(false, false);
#undef QL_D4
}

// ---------------------------------------------------------------- chain variant

struct ChainConfig {
    int R, CONS, PROD, BPS, STAGES, FS;
};

int chain_fstr(int BPS) { return ((BPS + 15) & ~15) + 4; }
int chain_fslot_floats(int R, int BPS, int mtok) { return mtok * (16 * R + 1) * chain_fstr(BPS); }

// One row group per CTA, four consumer and four producer warps, stages of 32
// blocks; the ring as deep as the shared memory of the CTAs that share an SM
// allows (up to three per SM), at most 32 stages and no deeper than the K range
// needs.  Measured on B200 (INT4, one token, the 27B-class attention and down
// projections): stages of 32 blocks beat 16 and 8 on every layer; four
// producers took 3-6% off the 5120-row layers against one (three, which forces
// a 12-deep ring, was much slower); two or eight consumer warps, or two row
// groups per CTA, were no faster.
ChainConfig chain_plan(int G, int nblk, int rec, int qrec, int mtok) {
    const int sms = d4_sms();
    ChainConfig c;
    c.R = 1;
    c.CONS = 4;
    c.PROD = 4;
    c.BPS = 32;
    c.FS = 8;
    c.STAGES = 0;
    if (const char* env = std::getenv("BREEZE_QL_DP4A_CHAIN")) {   // "R,CONS,BPS,STAGES,FS[,PROD]", 0 = planner
        int r = 0, co = 0, b = 0, st = 0, fs = 0, pd = 0;
        if (std::sscanf(env, "%d,%d,%d,%d,%d,%d", &r, &co, &b, &st, &fs, &pd) >= 5) {
            if (r > 0) c.R = r;
            if (co > 0) c.CONS = co;
            if (b > 0) c.BPS = b;
            if (fs > 0) c.FS = fs;
            if (pd > 0) c.PROD = pd;
            c.STAGES = st;
        }
    }
    if (c.STAGES <= 0) {
        const long long ctas = (G + c.R - 1) / c.R;
        const int per_sm = static_cast<int>(std::min<long long>(3, std::max<long long>(1, (ctas + sms - 1) / sms)));
        const int budget = 227 * 1024 / per_sm - 2048;
        const int fslot = chain_fslot_floats(c.R, c.BPS, mtok);
        const int fixed = 256 + c.FS * fslot * 4 + 256;
        const int stage = d4_stage_bytes(c.R, c.BPS, rec, qrec);
        const int nst = (nblk + c.BPS - 1) / c.BPS;
        const int unit = std::max(c.CONS, c.PROD) % std::min(c.CONS, c.PROD) == 0 ? std::max(c.CONS, c.PROD)
                                                                                 : c.CONS * c.PROD;
        int st = (budget - fixed) / stage;
        st = std::min(st, 32);
        st = std::min(st, ((nst + unit - 1) / unit) * unit);
        st = (st / unit) * unit;
        c.STAGES = std::max(st, unit);
    }
    return c;
}

template <bool HALF, bool ZP, int MTOK, bool HP>
cudaError_t chain_launch(const Dp4aParams& p0, cudaStream_t stream, bool pdl) {
    constexpr int REC = 256 + (HALF ? 32 : 64) + (ZP ? 16 : 0);
    const ChainConfig c = chain_plan(p0.G, p0.nblk, REC, p0.QREC, MTOK);
    ChainParams p = {};
    p.W = p0.W;
    p.q = p0.q;
    p.C = p0.C;
    p.err = p0.err;
    p.M = p0.M;
    p.N = p0.N;
    p.nblk = p0.nblk;
    p.G = p0.G;
    p.ldc = p0.ldc;
    p.TPB = p0.TPB;
    p.TPBA = p0.TPBA;
    p.QREC = p0.QREC;
    p.R = c.R;
    p.CONS = c.CONS;
    p.PROD = c.PROD;
    p.BPS = c.BPS;
    p.STAGES = c.STAGES;
    p.FS = c.FS;
    p.off_Q = c.R * c.BPS * REC;
    p.stage_bytes = d4_stage_bytes(c.R, c.BPS, REC, p.QREC);
    p.fstr = chain_fstr(c.BPS);
    p.fslot_floats = chain_fslot_floats(c.R, c.BPS, MTOK);
    const uint32_t bar_bytes = (2 * c.STAGES + 2 * c.FS) * 8;
    p.off_f = (bar_bytes + 127) & ~127u;
    p.off_stages = (p.off_f + c.FS * p.fslot_floats * 4 + 127) & ~127u;
    const size_t smem = p.off_stages + static_cast<size_t>(c.STAGES) * p.stage_bytes;
    // the carve-up must fit the SM and keep the invariants the kernel relies on:
    // a stage and an f-slot return to the warp that used them last, and a warp
    // pass covers four (row group, block) units
    if (smem > 227 * 1024 || (c.R != 1 && c.R != 2 && c.R != 4) || c.CONS < 1 || c.CONS > 8 || c.PROD < 1 ||
        c.PROD > 4 || c.BPS < 1 || c.STAGES < 1 || c.FS < 1 || (c.STAGES % c.CONS) || (c.STAGES % c.PROD) ||
        (c.FS % c.CONS) || (p.QREC % 16) || (REC % 16))
        return cudaErrorInvalidConfiguration;
    auto kern = decode_dp4a_chain_kernel<HALF, ZP, MTOK, HP>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.G + c.R - 1) / c.R);
    cfg.blockDim = dim3(32 * (c.CONS + 1 + c.PROD));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <bool HP>
cudaError_t chain_dispatch(const Weight* w, const Dp4aParams& p, int M, cudaStream_t stream, bool pdl) {
#define QL_D4C(HALF, ZP)                                                                    \
    return M == 1 ? chain_launch<HALF, ZP, 1, HP>(p, stream, pdl)                           \
                  : chain_launch<HALF, ZP, 2, HP>(p, stream, pdl)
    if (w->has_zp) {
        if (w->scale_half) QL_D4C(true, true);
        QL_D4C(false, true);
    }
    if (w->scale_half) QL_D4C(true, false);
    QL_D4C(false, false);
#undef QL_D4C
}

// Which variant: BREEZE_QL_DP4A_KERNEL = "relay" or "chain" forces one;
// otherwise the relay kernel for layers of at least 128 quads of row groups
// (N >= 8192), the chain kernel below that.  Block sums (cs output) always
// take the relay kernel.
bool use_chain(const Weight* w) {
    const char* v = std::getenv("BREEZE_QL_DP4A_KERNEL");
    if (v && std::strcmp(v, "relay") == 0) return false;
    if (v && std::strcmp(v, "chain") == 0) return true;
    return (w->G + 3) / 4 < 128;
}

}  // namespace

// INT4 weights at one or two tokens run this file's kernels unless
// BREEZE_QL_DECODE_DP4A=0.
bool decode_dp4a_applies(const Weight* w, const ActView& act) {
    const char* v = std::getenv("BREEZE_QL_DECODE_DP4A");
    const bool off = v && v[0] == '0';
    return !off && w->bits == 4 && act.MT == 1 && act.TPB >= 1 && act.TPB <= 2;
}

cudaError_t launch_decode_dp4a(const Weight* w, const ActView& act, bool hi_prec, float* C, int ldc, int32_t* cs,
                               cudaStream_t stream, bool pdl) {
    if (act.hp != (hi_prec ? 1 : 0) || act.MT != 1 || act.TPB < 1 || act.TPB > 2 || act.M != act.TPB ||
        act.QREC != act.TPB * 4 * act.LB + act.TPBA * 8)
        return cudaErrorInvalidValue;
    Dp4aParams p = {};
    p.W = w->W;
    p.q = act.q;
    p.C = C;
    p.CS = cs;
    p.err = device_error_word();
    p.M = act.M;
    p.N = w->N;
    p.nblk = w->nblk;
    p.G = w->G;
    p.ldc = ldc;
    p.TPB = act.TPB;
    p.TPBA = act.TPBA;
    p.QREC = act.QREC;
    if (cs) return hi_prec ? d4_dispatch<true, true>(w, p, act.M, stream, pdl)
                           : d4_dispatch<false, true>(w, p, act.M, stream, pdl);
    if (use_chain(w)) return hi_prec ? chain_dispatch<true>(w, p, act.M, stream, pdl)
                                     : chain_dispatch<false>(w, p, act.M, stream, pdl);
    return hi_prec ? d4_dispatch<true, false>(w, p, act.M, stream, pdl)
                   : d4_dispatch<false, false>(w, p, act.M, stream, pdl);
}

}  // namespace ql
