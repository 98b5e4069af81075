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
//   * a record's 32 bytes of rows g and g+8 (byte = q(g) | q(g+8) << 4) give
//     x & 0xF0F0F0F0 = 16*q(g+8) and (x << 4) & 0xF0F0F0F0 = 16*q(g) per byte
//     -- two masks and a shift per 8 weights, no per-weight zero point;
//   * dp4a against the activation planes (hi - 128 signed, lo unsigned, or q8)
//     gives 16*sum hs*q and 16*sum lo*q exactly (|16*256*sum| < 2^31), so
//     sum q16*q = (256*S_hi + S_lo) >> 4 in int32;
//   * the zero point comes out through the activation side:
//     cs = sum q16*(q - zp) = sum q16*q - zp * sum q16, where the quantizer
//     stores sum q16 per (token, block) in the record;
//   * (float)cs * bscale and acc = fma(ascale, f, acc) in ascending block order,
//     the reference's FP32 chain.
// About 20 warp instructions per record at one token.
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

}  // namespace

template <bool HALF, bool ZP, int MTOK, bool HP, bool OUT_CS>
__global__ void __launch_bounds__(288) decode_dp4a_kernel(const Dp4aParams p) {
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

    if (warp == consumers) {
        // ------------------------------------------------------------ producer
        if (lane != 0) return;
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
        for (int i = 0; i < first; ++i) issue(i, true, false);
        pdl_wait();                                   // activations come from the previous grid
        for (int i = 0; i < first; ++i) issue(i, false, true);
        for (int i = first; i < nst; ++i) {
            const int s = i % p.STAGES;
            if (!mbar_wait(smem_u32(&empty_bar[s]), ((i / p.STAGES) - 1) & 1, p.err)) {
                for (int j = max(0, i - p.STAGES); j < i; ++j)      // let issued copies land
                    if (!mbar_wait(smem_u32(&full_bar[j % p.STAGES]), (j / p.STAGES) & 1, p.err)) break;
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
                const uint8_t* rec = Wst + j * REC;
                const uint4 wa = *reinterpret_cast<const uint4*>(rec + 32 * g);
                const uint4 wb = *reinterpret_cast<const uint4*>(rec + 32 * g + 16);
                const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                uint32_t e[8], o[8];                           // 16*q of row g, 16*q of row g+8
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    e[k] = (w[k] << 4) & 0xF0F0F0F0u;
                    o[k] = w[k] & 0xF0F0F0F0u;
                }
                float bs0, bs1;
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
                const uint8_t* qrec = Qst + j * p.QREC;
#pragma unroll
                for (int m = 0; m < MTOK; ++m) {
                    int sh0 = 0, sl0 = 0, sh1 = 0, sl1 = 0;
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        if (HP) {
                            // slot t: hs of k 4t.. and 16+4t.., then lo of the same k
                            const uint4 a = *reinterpret_cast<const uint4*>(qrec + (m * 4 + t) * 16);
                            sh0 = dp4a_su(a.x, e[2 * t], sh0);
                            sh1 = dp4a_su(a.x, o[2 * t], sh1);
                            sl0 = dp4a_uu(a.z, e[2 * t], sl0);
                            sl1 = dp4a_uu(a.z, o[2 * t], sl1);
                            sh0 = dp4a_su(a.y, e[2 * t + 1], sh0);
                            sh1 = dp4a_su(a.y, o[2 * t + 1], sh1);
                            sl0 = dp4a_uu(a.w, e[2 * t + 1], sl0);
                            sl1 = dp4a_uu(a.w, o[2 * t + 1], sl1);
                        } else {
                            const uint2 a = *reinterpret_cast<const uint2*>(qrec + (m * 4 + t) * 8);
                            sh0 = dp4a_su(a.x, e[2 * t], sh0);
                            sh1 = dp4a_su(a.x, o[2 * t], sh1);
                            sh0 = dp4a_su(a.y, e[2 * t + 1], sh0);
                            sh1 = dp4a_su(a.y, o[2 * t + 1], sh1);
                        }
                    }
                    // sum q16*q exactly (every term a multiple of 16), then the zero point
                    const int sq = *reinterpret_cast<const int*>(qrec + q_sum + 4 * m);
                    const int c0 = (HP ? (sh0 * 256 + sl0) : sh0) >> 4;
                    const int c1 = (HP ? (sh1 * 256 + sl1) : sh1) >> 4;
                    const int cs0 = c0 - zg * sq, cs1 = c1 - zg8 * sq;
                    if (OUT_CS) {
                        if (j0 + u < nb && row_ok && m < p.M) {
                            const int n0 = G * 16 + g;
                            p.CS[(static_cast<size_t>(m) * p.N + n0) * p.nblk + b0 + j] = cs0;
                            p.CS[(static_cast<size_t>(m) * p.N + n0 + 8) * p.nblk + b0 + j] = cs1;
                        }
                        continue;
                    }
                    f[u][0][m] = __fmul_rn(__int2float_rn(cs0), bs0);     // (float)cs * bscale
                    f[u][1][m] = __fmul_rn(__int2float_rn(cs1), bs1);
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

// ------------------------------------------------------------------ host side

int* device_error_word();   // ql_api.cu

namespace {

constexpr int D4_SMEM_BUDGET = 110 * 1024;   // dynamic shared memory per CTA: >= 2 CTAs per SM

struct D4Config {
    int Q4, SPLIT, BPS, STAGES;
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
// fewer than 128 quads stay on the tensor-core kernel (decode_dp4a_applies).
D4Config d4_plan(int G, int nblk, int rec, int qrec) {
    const int sms = d4_sms();
    const long long quads = (G + 3) / 4;
    D4Config c;
    c.Q4 = 1;
    c.SPLIT = 4;
    c.BPS = D4_C;
    c.STAGES = quads >= 3LL * sms ? 4 : 8;
    while (c.SPLIT > 1 && (nblk + c.BPS - 1) / c.BPS < 2 * c.SPLIT) c.SPLIT /= 2;
    if (c.STAGES % c.SPLIT) c.STAGES = ((c.STAGES + c.SPLIT - 1) / c.SPLIT) * c.SPLIT;
    if (c.STAGES < 2) c.STAGES = 2;
    (void)rec;
    (void)qrec;
    // Tuning override "Q4,SPLIT,BPS,STAGES" (0 keeps the planner's value); the
    // launch checks reject values that break the kernel's invariants.
    if (const char* env = std::getenv("BREEZE_QL_DP4A_CONFIG")) {
        int q = 0, sp = 0, b = 0, st = 0;
        if (std::sscanf(env, "%d,%d,%d,%d", &q, &sp, &b, &st) == 4) {
            if (q > 0) c.Q4 = q;
            if (sp > 0) c.SPLIT = sp;
            if (b > 0) c.BPS = b;
            if (st > 0) c.STAGES = st;
        }
    }
    return c;
}

template <bool HALF, bool ZP, int MTOK, bool HP, bool OUT_CS>
cudaError_t d4_launch(const Dp4aParams& p0, cudaStream_t stream, bool pdl) {
    constexpr int REC = 256 + (HALF ? 32 : 64) + (ZP ? 16 : 0);
    Dp4aParams p = p0;
    const D4Config c = d4_plan(p.G, p.nblk, REC, p.QREC);
    p.Q4 = c.Q4;
    p.SPLIT = c.SPLIT;
    p.BPS = c.BPS;
    p.STAGES = c.STAGES;
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
        consumers > 8 || (c.STAGES % c.SPLIT) || (p.QREC % 16) || (REC % 16) || (p.off_Q % 16))
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
    cfg.blockDim = dim3(32 * (consumers + 1));
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

}  // namespace

// INT4 weights at one or two tokens with at least 128 quads of row groups
// (N >= 8192) run this kernel unless BREEZE_QL_DECODE_DP4A=0.
bool decode_dp4a_applies(const Weight* w, const ActView& act) {
    static const int off = [] {
        const char* v = std::getenv("BREEZE_QL_DECODE_DP4A");
        return (v && v[0] == '0') ? 1 : 0;
    }();
    return !off && w->bits == 4 && act.MT == 1 && act.TPB >= 1 && act.TPB <= 2 && (w->G + 3) / 4 >= 128;
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
    return hi_prec ? d4_dispatch<true, false>(w, p, act.M, stream, pdl)
                   : d4_dispatch<false, false>(w, p, act.M, stream, pdl);
}

}  // namespace ql
