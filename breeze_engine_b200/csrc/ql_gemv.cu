// ql_gemv.cu -- decode (skinny) quantized GEMV/GEMM for M = 1..64 tokens.
//
// Computes C[m, n] = i4_matmul(A)[m, n] (kernel/quantized_matmul.cpp:270-318
// tile_kernel, :320-365 tile_kernel8) from activations quantized by ql_quant.cu.
//
// Warp roles in a CTA that owns R row groups of 16 output features:
//   * producers (PROD warps, lane 0 each): producer p streams the stages
//     i = p (mod PROD) (BPS consecutive 32-wide blocks each) into a
//     STAGES-deep shared-memory ring with 1-D bulk copies (cp.async.bulk, no
//     multicast): ONE copy per row group (its weight records -- weights,
//     scales and zero points of BPS blocks are contiguous) plus ONE copy of the
//     activation records shared by the CTA.  Bulk copies cost a roughly fixed
//     number of cycles each, so stages are large and few; and one issuing
//     thread's copies stream at most ~16-19 GB/s on B200 however deep the ring
//     (measured), so CTAs that are few per SM use several producers.
//   * consumers (S per row group): warp (r, s) takes stages i = s, s+S, ...  Per
//     block: one 16x32 weight fragment (LDS.128 INT8; LDS.64 + 7 integer ops
//     per 8 nibbles INT4); per 8-token group one LDS.128 of both activation
//     planes and two m16n8k32 integer MMAs whose C operand is the constant
//     magic seed; then the exact f = RN((float)cs * bscale) with packed f32x2
//     ops (ql_common.cuh).  C blocks are computed together for ILP.
//   * exact FP32 chain: every output needs acc = fma(ascale_b, f_b, acc) in
//     ascending block order (kernel/quantized_matmul.cpp:311-315).  The warp of
//     stage i takes acc from the warp of stage i-1 through a shared-memory
//     relay slot guarded by an mbarrier (all 32 lanes arrive, so every lane's
//     store is released), applies its blocks in order and relays acc on; the
//     warp of the last stage stores C.  Only these FFMAs are serial; the MMAs
//     and conversions of the S warps overlap.
// Ring slots and relay slots are always used by the same warp in phase order
// (STAGES and the relay slot count are multiples of S), so no mbarrier waiter
// can run two phases ahead: mbarrier.try_wait.parity would report the previous
// phase's parity as complete.
//
// With PDL the producer issues the first weight stages before waiting on the
// quantizer grid (griddepcontrol.wait).
//
// Template parameters: BITS (4/8), HALF (fp16 scales), ZP (explicit INT4 zero
// points), MT (8-token groups: 1, 2, 4, 8), HP (two-pass INT16 / single-pass
// INT8), OUT_CS (write the per-block INT32 accumulators instead of C).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include "ql_common.cuh"
#include "ql_internal.h"

namespace ql {

struct DecodeParams {
    const uint8_t* W;        // weight records [G][nblk][REC]
    const uint8_t* q;        // activation records [nblk][QREC]
    float* C;
    int32_t* CS;
    int* err;
    int M, N, nblk, G, ldc;
    int TPB, TPBA, QREC;     // activation record geometry
    int R, SPLIT, BPS, STAGES, PROD;
    uint32_t stage_bytes;
    uint32_t off_Q;                        // activation records inside a stage
    uint32_t off_relay, off_stages;        // offsets inside dynamic shared memory
};

template <int BITS, bool HALF, bool ZP, bool HP>
struct Geom {
    static constexpr int TB = BITS == 8 ? 512 : 256;        // weight tile bytes
    static constexpr int SB = HALF ? 32 : 64;               // scale bytes per tile
    static constexpr int ZB = ZP ? 16 : 0;                  // zero-point bytes per tile
    static constexpr int REC = TB + SB + ZB;                // weight record bytes
    static constexpr int LB = HP ? 16 : 8;                  // activation bytes per lane
};

// Relay slots per row group: at least 2, and SPLIT when larger (see above).
__host__ __device__ __forceinline__ int relay_slots(int split) { return split < 2 ? 2 : split; }

// Blocks computed together per sub-chunk (registers hold their f and ascale).
// With a K split a stage is exactly one sub-chunk, so a warp computes all of
// its stage's f values before it waits for the relay: each relay hop then
// costs only the stage's FFMA chain and the hand-off.
template <int MT>
struct Chunk {
    static constexpr int C = MT == 1 ? 16 : (MT == 2 ? 8 : (MT == 4 ? 4 : 2));
};

template <int BITS, bool HALF, bool ZP, int MT, bool HP, bool OUT_CS>
__global__ void __launch_bounds__(384) decode_kernel(const DecodeParams p) {
    using Geo = Geom<BITS, HALF, ZP, HP>;
    constexpr int C = Chunk<MT>::C;
    extern __shared__ __align__(128) uint8_t smem[];
    // barriers: full[STAGES], empty[STAGES], relay[R][NS]
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty_bar = full_bar + p.STAGES;
    uint64_t* relay_bar = empty_bar + p.STAGES;
    uint8_t* stages = smem + p.off_stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int consumers = p.R * p.SPLIT;
    const int NS = relay_slots(p.SPLIT);
    const int G0 = blockIdx.x * p.R;
    const int active = min(p.R, p.G - G0);
    const int nst = (p.nblk + p.BPS - 1) / p.BPS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.STAGES; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), active);
        }
        for (int k = 0; k < p.R * NS; ++k) mbar_init(smem_u32(&relay_bar[k]), 32);
        fence_mbar_init();
    }
    __syncthreads();
    // The next kernel on the stream (the next layer's quantizer or matmul) may
    // be scheduled now: it waits for this grid's completion before it touches
    // anything this grid reads or writes, and meanwhile prefetches its weights.
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
                // all bytes this stage receives: each active row group's weight
                // records plus the shared activation records
                mbar_arrive_expect_tx(full, (active * Geo::REC + p.QREC) * nb);
                for (int w = 0; w < active; ++w) {
                    const size_t rec0 = static_cast<size_t>(G0 + w) * p.nblk + b0;
                    bulk_g2s(base + w * p.BPS * Geo::REC, p.W + rec0 * Geo::REC, nb * Geo::REC, full);
                }
            }
            if (acts)
                bulk_g2s(base + p.off_Q, p.q + static_cast<size_t>(b0) * p.QREC, nb * p.QREC, full);
        };
        const int first = min(p.STAGES, nst);
        for (int i = pr; i < first; i += p.PROD) issue(i, true, false);
        pdl_wait();                                   // activations come from the previous grid
        for (int i = pr; i < first; i += p.PROD) issue(i, false, true);
        for (int i = first + ((pr - first) % p.PROD + p.PROD) % p.PROD; i < nst; i += p.PROD) {
            const int s = i % p.STAGES;
            if (!mbar_wait(smem_u32(&empty_bar[s]), ((i / p.STAGES) - 1) & 1, p.err)) {
                // Giving up: let this producer's copies already issued land
                // before the CTA can exit (each slot's last issued phase;
                // bounded waits).
                for (int j = i - p.STAGES; j < i; j += p.PROD)
                    if (j >= 0 && !mbar_wait(smem_u32(&full_bar[j % p.STAGES]), (j / p.STAGES) & 1, p.err)) break;
                return;
            }
            issue(i, true, true);
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int r = warp / p.SPLIT;            // row group within the CTA
    const int split = warp % p.SPLIT;        // stages i = split, split + SPLIT, ...
    if (r >= active) return;
    const int G = G0 + r;
    const int g = lane >> 2, t = lane & 3;
    float* relay = reinterpret_cast<float*>(smem + p.off_relay) + static_cast<size_t>(r) * NS * 32 * 4 * MT;

    // Seeds as the MMA's C operand (constant registers, never overwritten).
    const int32_t seed_h[4] = {HI_SEED, HI_SEED, HI_SEED, HI_SEED};
    const int32_t seed_l[4] = {LO_SEED, LO_SEED, LO_SEED, LO_SEED};
    const uint64_t negc_lo = f2_pack(-12582912.0f, -12582912.0f);   // single-pass: -1.5*2^23
    const int qfrag = p.TPB * 4 * Geo::LB;   // scales start here inside an activation record

    uint64_t accA[MT], accB[MT];             // (row g | row g+8) x (tokens 2t, 2t+1)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) { accA[mt] = 0; accB[mt] = 0; }

    for (int i = split; i < nst; i += p.SPLIT) {
        const int s = i % p.STAGES;
        if (!mbar_wait(smem_u32(&full_bar[s]), (i / p.STAGES) & 1, p.err)) return;
        const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
        const uint8_t* Wst = st + r * p.BPS * Geo::REC;
        const uint8_t* Qst = st + p.off_Q;
        const int b0 = i * p.BPS;
        const int nb = min(p.BPS, p.nblk - b0);
        bool need_relay = !OUT_CS && p.SPLIT > 1 && i > 0;

        for (int j0 = 0; j0 < nb; j0 += C) {
            uint64_t fr[C][MT][2];           // f of C blocks (rows g, g+8)
            uint64_t ar[C][MT];              // their activation scale pairs
#pragma unroll
            for (int u = 0; u < C; ++u) {
                const int j = min(j0 + u, nb - 1);           // slots past nb are discarded
                const uint8_t* rec = Wst + j * Geo::REC;
                uint32_t a[4];
                if (BITS == 8) {
                    const uint4 v = *reinterpret_cast<const uint4*>(rec + lane * 16);
                    a[0] = v.x; a[1] = v.y; a[2] = v.z; a[3] = v.w;
                } else {
                    const uint2 v = *reinterpret_cast<const uint2*>(rec + lane * 8);
                    uint32_t c0 = 0x78787878u, c1 = 0x78787878u;          // zp = 8
                    if (ZP) {
                        const uint32_t z = rec[Geo::TB + Geo::SB + g];
                        c0 = (0x80u - (z & 15u)) * 0x01010101u;
                        c1 = (0x80u - (z >> 4)) * 0x01010101u;
                    }
                    a[0] = nib_even_s8(v.x, c0);
                    a[1] = nib_odd_s8(v.x, c1);
                    a[2] = nib_even_s8(v.y, c0);
                    a[3] = nib_odd_s8(v.y, c1);
                }
                float bs0, bs1;
                if (HALF) {
                    const __half2 hs = *reinterpret_cast<const __half2*>(rec + Geo::TB + g * 4);
                    bs0 = __low2float(hs);
                    bs1 = __high2float(hs);
                } else {
                    const float2 f = *reinterpret_cast<const float2*>(rec + Geo::TB + g * 8);
                    bs0 = f.x;
                    bs1 = f.y;
                }
                const uint64_t bsA = f2_pack(bs0, bs0), bsB = f2_pack(bs1, bs1);
                const uint8_t* qrec = Qst + j * p.QREC;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const int tok = mt * 8 + g;               // this lane's B-fragment token
                    int32_t h[4], l[4];
                    if (HP) {
                        uint4 qv = make_uint4(0, 0, 0, 0);
                        if (MT > 1 || tok < p.TPB)
                            qv = *reinterpret_cast<const uint4*>(qrec + (tok * 4 + t) * 16);
                        mma_s8s8_c(h, a, qv.x, qv.y, seed_h);    // hi - 128 plane
                        mma_s8u8_c(l, a, qv.z, qv.w, seed_l);    // lo plane
                    } else {
                        uint2 qv = make_uint2(0, 0);
                        if (MT > 1 || tok < p.TPB)
                            qv = *reinterpret_cast<const uint2*>(qrec + (tok * 4 + t) * 8);
                        mma_s8s8_c(l, a, qv.x, qv.y, seed_l);
                    }
                    if (OUT_CS) {
                        if (j0 + u < nb) {
                            const int tok0 = mt * 8 + 2 * t;
                            const int n0 = G * 16 + g;
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int tk = tok0 + (e & 1);
                                const int n = n0 + 8 * (e >> 1);
                                const int32_t cs = HP ? (h[e] - HI_SEED) * 256 + (l[e] - LO_SEED)
                                                      : l[e] - LO_SEED;
                                if (tk < p.M)
                                    p.CS[(static_cast<size_t>(tk) * p.N + n) * p.nblk + b0 + j] = cs;
                            }
                        }
                        continue;
                    }
                    uint64_t yA, yB;
                    if (HP) {
                        yA = cs_to_f2(h[0], h[1], l[0], l[1]);
                        yB = cs_to_f2(h[2], h[3], l[2], l[3]);
                    } else {
                        yA = f2_add(i2_pack(l[0], l[1]), negc_lo);   // exact (|cs| < 2^22)
                        yB = f2_add(i2_pack(l[2], l[3]), negc_lo);
                    }
                    fr[u][mt][0] = f2_mul(yA, bsA);
                    fr[u][mt][1] = f2_mul(yB, bsB);
                    // activation scales of tokens 2t, 2t+1 (TPBA is a multiple of
                    // 4, so both or neither exist; padded scales are zero)
                    const int tk = mt * 8 + 2 * t;
                    ar[u][mt] = tk < p.TPBA ? *reinterpret_cast<const uint64_t*>(qrec + qfrag + tk * 4) : 0;
                }
            }
            if (OUT_CS) continue;
            // Every read of this stage's shared memory is done once the last
            // sub-chunk's f values are in registers: hand the stage back to the
            // producer before the (serial) relay wait and FFMA chain, so the
            // ring refills while the chain runs.
            if (j0 + C >= nb) {
                fence_proxy_async_smem();      // this warp's reads before the refill's bulk copy
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
            }
            // ---- take the running accumulator of stage i-1 (once per stage)
            if (need_relay) {
                need_relay = false;
                const int slot = (i - 1) % NS;
                if (!mbar_wait(smem_u32(&relay_bar[r * NS + slot]), ((i - 1) / NS) & 1, p.err)) return;
                const float* src = relay + (slot * 32 + lane) * 4 * MT;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const float4 v = *reinterpret_cast<const float4*>(src + 4 * mt);
                    accA[mt] = f2_pack(v.x, v.y);
                    accB[mt] = f2_pack(v.z, v.w);
                }
            }
            // ---- the FP32 chain over these C blocks, ascending order
#pragma unroll
            for (int u = 0; u < C; ++u) {
                if (j0 + u >= nb) break;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    accA[mt] = f2_fma(ar[u][mt], fr[u][mt][0], accA[mt]);
                    accB[mt] = f2_fma(ar[u][mt], fr[u][mt][1], accB[mt]);
                }
            }
        }
        // release the stage to the producer (the FP32 path released it above)
        if (OUT_CS) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
            continue;
        }
        if (p.SPLIT > 1 && i + 1 < nst) {
            // hand the accumulator to the warp of stage i + 1
            const int slot = i % NS;
            float* dst = relay + (slot * 32 + lane) * 4 * MT;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const float2 A2 = f2_unpack(accA[mt]);
                const float2 B2 = f2_unpack(accB[mt]);
                *reinterpret_cast<float4*>(dst + 4 * mt) = make_float4(A2.x, A2.y, B2.x, B2.y);
            }
            mbar_arrive(smem_u32(&relay_bar[r * NS + slot]));
        }
        if (i + 1 >= nst) {
            // this warp ran the last stage: store the outputs
            const int n0 = G * 16 + g;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int tok0 = mt * 8 + 2 * t;
                const float2 A2 = f2_unpack(accA[mt]);
                const float2 B2 = f2_unpack(accB[mt]);
                if (tok0 < p.M) {
                    p.C[static_cast<size_t>(tok0) * p.ldc + n0] = A2.x;
                    p.C[static_cast<size_t>(tok0) * p.ldc + n0 + 8] = B2.x;
                }
                if (tok0 + 1 < p.M) {
                    p.C[static_cast<size_t>(tok0 + 1) * p.ldc + n0] = A2.y;
                    p.C[static_cast<size_t>(tok0 + 1) * p.ldc + n0 + 8] = B2.y;
                }
            }
        }
    }
}

// ------------------------------------------------------------------ host side

struct DecodeConfig {
    int R, SPLIT, BPS, STAGES, PROD;
};

static int g_num_sms = 0;
constexpr int SMEM_BUDGET = 110 * 1024;   // dynamic shared memory per CTA: >= 2 CTAs per SM

static int stage_bytes_for(int R, int BPS, int rec, int qrec) {
    return (R * BPS * rec + BPS * qrec + 127) & ~127;
}

static DecodeConfig choose_config(int G, int nblk, int C, int rec, int qrec, int bits) {
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    DecodeConfig c;
    // ~12 consumer warps per SM in total: row groups first, then K splits.
    const long long target = 12LL * g_num_sms;
    // (Measured on B200: 4 row groups per CTA without a split win from ~600
    // row groups up; below that, split K across 4 warps per row group.)
    // INT4 records are half the size of INT8 ones, so a split stage of C
    // blocks is a small copy and every relay hop (one per stage) costs as much
    // as for INT8: INT4 uses at most 4 consumer warps per CTA and, where the
    // row has enough blocks, stages of 2C blocks.  (Measured on B200 at M = 1:
    // 23-41% faster on 5120x6144, 6144x5120 and 17408x5120 layers.)
    const int max_warps = bits == 4 ? 4 : 8;
    // Tuning override "R,SPLIT,BPS,STAGES[,PROD]" (each 0 = keep the planner's
    // choice), applied where the planner makes that choice.  Values that break
    // the planner's invariants are rejected by launch_t.
    int ov_r = 0, ov_sp = 0, ov_b = 0, ov_s = 0, ov_p = 0;
    if (const char* env = std::getenv("BREEZE_QL_DECODE_CONFIG"))
        if (std::sscanf(env, "%d,%d,%d,%d,%d", &ov_r, &ov_sp, &ov_b, &ov_s, &ov_p) < 4)
            ov_r = ov_sp = ov_b = ov_s = ov_p = 0;
    c.R = 1;
    c.SPLIT = 1;
    if (G >= 4 * g_num_sms) c.R = 4;
    else if (G >= 2 * g_num_sms) c.R = 2;
    if (ov_r > 0) c.R = ov_r;
    while (c.R <= 2 && c.SPLIT < 8 && c.R * c.SPLIT < max_warps &&
           static_cast<long long>(G) * c.SPLIT * 2 <= target)
        c.SPLIT *= 2;
    const int nblk_even = (nblk + 1) & ~1;
    // A split stage is one or two sub-chunks (C blocks); at least two stages per split.
    while (c.SPLIT > 1 && (nblk_even + C - 1) / C < 2 * c.SPLIT) c.SPLIT /= 2;
    if (ov_sp > 0) c.SPLIT = ov_sp;
    if (c.SPLIT > 1) {
        c.BPS = C;
        if (bits == 4 && (nblk_even + 2 * C - 1) / (2 * C) >= 2 * c.SPLIT) c.BPS = 2 * C;
    } else {
        // Stages of >= 32 KB (bulk copies have a fixed cost each), two of
        // which must fit the shared-memory budget.
        c.BPS = C;
        while (c.BPS < 32 && stage_bytes_for(c.R, c.BPS, rec, qrec) < 32768 &&
               2 * stage_bytes_for(c.R, c.BPS + C, rec, qrec) <= SMEM_BUDGET)
            c.BPS += C;
    }
    if (c.BPS > nblk_even) c.BPS = std::max(2, ((nblk_even + C - 1) / C) * C);
    if (ov_b > 0) c.BPS = ov_b;
    // One producer: on the INT8 decode sweep (B200, M = 1..16) two producers
    // were within 1% and four 26% slower (their ring rounds up to a multiple
    // of four stages); this kernel's 50 MB layers are not producer-bound.
    c.PROD = 1;
    if (ov_p > 0) c.PROD = ov_p;
    // Ring slots go back to the warp (consumer and producer) that used them
    // last: STAGES is a multiple of SPLIT and of PROD.
    const int unit = std::max(c.SPLIT, c.PROD) % std::min(c.SPLIT, c.PROD) == 0 ? std::max(c.SPLIT, c.PROD)
                                                                               : c.SPLIT * c.PROD;
    const int st = stage_bytes_for(c.R, c.BPS, rec, qrec);
    // ~48 KB in flight per CTA, >= 2 stages per split.
    c.STAGES = std::max(2 * c.SPLIT, (49152 + st - 1) / st);
    c.STAGES = std::min(c.STAGES, std::max(2 * c.SPLIT, 8));
    c.STAGES = ((c.STAGES + unit - 1) / unit) * unit;
    if (c.STAGES < 2) c.STAGES = 2;
    while (c.STAGES - unit >= std::max(2, c.SPLIT) && c.STAGES * st > SMEM_BUDGET) c.STAGES -= unit;
    if (ov_s > 0) c.STAGES = ov_s;
    return c;
}

template <int BITS, bool HALF, bool ZP, int MT, bool HP, bool OUT_CS>
static cudaError_t launch_t(const DecodeParams& p0, const DecodeConfig& c, cudaStream_t stream, bool pdl) {
    using Geo = Geom<BITS, HALF, ZP, HP>;
    constexpr int C = Chunk<MT>::C;
    DecodeParams p = p0;
    p.R = c.R;
    p.SPLIT = c.SPLIT;
    p.BPS = c.BPS;
    p.STAGES = c.STAGES;
    p.PROD = c.PROD;
    p.off_Q = c.R * c.BPS * Geo::REC;
    p.stage_bytes = stage_bytes_for(c.R, c.BPS, Geo::REC, p.QREC);
    const int NS = relay_slots(c.SPLIT);
    const uint32_t bar_bytes = (2 * c.STAGES + c.R * NS) * 8;
    p.off_relay = (bar_bytes + 127) & ~127u;
    const uint32_t relay_bytes = c.R * NS * 32 * 4 * MT * 4;
    p.off_stages = (p.off_relay + relay_bytes + 127) & ~127u;
    const size_t smem = p.off_stages + static_cast<size_t>(c.STAGES) * p.stage_bytes;
    // Host-side guards: the carve-up must fit the SM and keep the invariants
    // the kernel relies on (16-byte copies, slots owned by one warp).
    const int consumers = c.R * c.SPLIT;
    if (smem > 227 * 1024 || c.BPS < 2 || (c.BPS % C) || c.STAGES < 2 || c.R < 1 || c.R > 8 ||
        c.SPLIT < 1 || c.SPLIT > 8 || consumers > 8 || (c.STAGES % c.SPLIT) || c.PROD < 1 || c.PROD > 4 ||
        (c.STAGES % c.PROD) || (p.QREC % 16) ||
        (Geo::REC % 16) || (p.off_Q % 16))
        return cudaErrorInvalidConfiguration;
    auto kern = decode_kernel<BITS, HALF, ZP, MT, HP, OUT_CS>;
    // Raise the dynamic shared-memory limit once per instantiation and device,
    // so launches captured into a CUDA graph make no attribute calls.
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (configured[dev] < static_cast<int>(smem)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = 227 * 1024;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.G + c.R - 1) / c.R);
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

template <int BITS, bool HALF, bool ZP, bool HP, bool OUT_CS>
static cudaError_t dispatch_mt(const DecodeParams& p, int MT, cudaStream_t stream, bool pdl) {
    using Geo = Geom<BITS, HALF, ZP, HP>;
    auto cfg = [&](int C) { return choose_config(p.G, p.nblk, C, Geo::REC, p.QREC, BITS); };
    switch (MT) {
        case 1: return launch_t<BITS, HALF, ZP, 1, HP, OUT_CS>(p, cfg(Chunk<1>::C), stream, pdl);
        case 2: return launch_t<BITS, HALF, ZP, 2, HP, OUT_CS>(p, cfg(Chunk<2>::C), stream, pdl);
        case 4: return launch_t<BITS, HALF, ZP, 4, HP, OUT_CS>(p, cfg(Chunk<4>::C), stream, pdl);
        default: return launch_t<BITS, HALF, ZP, 8, HP, OUT_CS>(p, cfg(Chunk<8>::C), stream, pdl);
    }
}

template <bool HP, bool OUT_CS>
static cudaError_t dispatch_w(const Weight* w, const DecodeParams& p, int MT, cudaStream_t stream,
                              bool pdl) {
    if (w->bits == 8) {
        if (w->scale_half) return dispatch_mt<8, true, false, HP, OUT_CS>(p, MT, stream, pdl);
        return dispatch_mt<8, false, false, HP, OUT_CS>(p, MT, stream, pdl);
    }
    if (w->has_zp) {
        if (w->scale_half) return dispatch_mt<4, true, true, HP, OUT_CS>(p, MT, stream, pdl);
        return dispatch_mt<4, false, true, HP, OUT_CS>(p, MT, stream, pdl);
    }
    if (w->scale_half) return dispatch_mt<4, true, false, HP, OUT_CS>(p, MT, stream, pdl);
    return dispatch_mt<4, false, false, HP, OUT_CS>(p, MT, stream, pdl);
}

int* device_error_word();   // ql_api.cu

cudaError_t launch_decode(const Weight* w, const ActView& act, bool hi_prec, float* C, int ldc,
                          int32_t* cs, cudaStream_t stream, bool pdl) {
    if (act.hp != (hi_prec ? 1 : 0)) return cudaErrorInvalidValue;   // layout depends on the mode
    DecodeParams p = {};
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
    const int MT = act.MT;
    if (MT != 1 && MT != 2 && MT != 4 && MT != 8) return cudaErrorInvalidValue;
    if ((MT == 1 && (act.TPB < 1 || act.TPB > 8)) || (MT > 1 && act.TPB != 8 * MT) ||
        act.TPBA < act.TPB || (act.TPBA & 3) || act.QREC != act.TPB * 4 * act.LB + act.TPBA * 8)
        return cudaErrorInvalidValue;
    if (decode_dp4a_applies(w, act)) return launch_decode_dp4a(w, act, hi_prec, C, ldc, cs, stream, pdl);
    if (cs) {
        return hi_prec ? dispatch_w<true, true>(w, p, MT, stream, pdl)
                       : dispatch_w<false, true>(w, p, MT, stream, pdl);
    }
    return hi_prec ? dispatch_w<true, false>(w, p, MT, stream, pdl)
                   : dispatch_w<false, false>(w, p, MT, stream, pdl);
}

}  // namespace ql
