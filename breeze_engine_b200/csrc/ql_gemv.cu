// ql_gemv.cu -- decode (skinny) quantized GEMV/GEMM for M = 1..64 tokens.
//
// Computes C[m, n] = i4_matmul(A)[m, n] (kernel/quantized_matmul.cpp:270-318
// tile_kernel, :320-365 tile_kernel8) from pre-quantized activations.
//
// Design (HBM-streaming, warp specialised):
//   * CTA = R consumer warps + 1 producer warp.  Consumer warp w owns the
//     16-row weight group G = blockIdx.x*R + w for ALL of K, so every output's
//     FP32 chain acc = fma(ascale, f, acc) runs in ascending block order in one
//     thread's registers -- bit-identical to the reference, no split-K fixup.
//   * The producer's lane 0 streams stages of BPS blocks with 1-D bulk copies
//     (cp.async.bulk, no multicast) into a STAGES-deep shared-memory ring:
//     per consumer the W/S/Z chunks (contiguous in the prepacked layout), and
//     once per CTA the activation planes and scales for those blocks, shared
//     by all R row groups.  full[]/empty[] mbarriers hand stages over.
//   * Consumers: per block, one 16x32 weight fragment (LDS.128 INT8, LDS.64 +
//     7 ALU ops per word INT4), then per 8-token group two m16n8k32 integer
//     MMAs (hi plane s8 x s8, lo plane s8 x u8) seeded with the magic
//     constants of ql_common.cuh, and four packed-f32x2 ops per two outputs
//     for the exact rescale.
//   * With PDL the producer issues the first weight stages before waiting on
//     the quantizer grid (griddepcontrol.wait), overlapping its tail.
//
// Template parameters: BITS (4/8), HALF (fp16 scales), ZP (explicit INT4 zero
// points), MT (8-token groups, 1..8), HP (two-pass INT16 / single-pass INT8),
// OUT_CS (debug: write the per-block INT32 accumulators instead of C).
#include <algorithm>
#include "ql_common.cuh"
#include "ql_internal.h"

namespace ql {

struct DecodeParams {
    const uint8_t* W;
    const void* S;
    const uint8_t* Z;
    const uint8_t* hs;
    const uint8_t* lo;
    const float* as;
    float* C;
    int32_t* CS;
    int* err;
    int M, N, nblk, nblkZ, G, ldc;
    int R, BPS, STAGES;
    uint32_t stage_bytes;
    uint32_t off_S, off_Z, off_H, off_L, off_A;   // offsets inside a stage
};

template <int BITS, bool HALF, bool ZP>
struct WeightGeom {
    static constexpr int TB = BITS == 8 ? 512 : 256;        // tile bytes
    static constexpr int SB = HALF ? 32 : 64;               // scale bytes per tile
    static constexpr int ZB = ZP ? 8 : 0;                   // zero-point bytes per tile
};

template <int BITS, bool HALF, bool ZP, int MT, bool HP, bool OUT_CS>
__global__ void __launch_bounds__(160) decode_kernel(const DecodeParams p) {
    using Geo = WeightGeom<BITS, HALF, ZP>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                // full[STAGES], empty[STAGES]
    uint8_t* stages = smem + 128 * ((2 * p.STAGES * 8 + 127) / 128);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G0 = blockIdx.x * p.R;
    const int active = min(p.R, p.G - G0);
    const int nst = (p.nblk + p.BPS - 1) / p.BPS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.STAGES; ++s) {
            mbar_init(smem_u32(&bars[s]), 1);
            mbar_init(smem_u32(&bars[p.STAGES + s]), active);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == p.R) {
        // ------------------------------------------------------------ producer
        if (lane != 0) return;
        const size_t act_blk = static_cast<size_t>(MT) * 256;        // plane bytes per block
        auto issue = [&](int i, bool weights, bool acts) {
            const int s = i % p.STAGES;
            const uint32_t base = smem_u32(stages + static_cast<size_t>(s) * p.stage_bytes);
            const uint32_t full = smem_u32(&bars[s]);
            const int b0 = i * p.BPS;
            const int nb = min(p.BPS, p.nblk - b0);
            if (weights) {
                // everything this stage will receive: weights/scales/zero points
                // for each active row group, then the shared activation planes
                // (two in two-pass mode, one in single-pass mode) and scales
                uint32_t bytes = active * nb * (Geo::TB + Geo::SB) + (HP ? 2 : 1) * nb * act_blk +
                                 nb * MT * 32;
                if (ZP) bytes += active * ((nb + 1) & ~1) * 8;
                mbar_arrive_expect_tx(full, bytes);
                for (int w = 0; w < active; ++w) {
                    const size_t tile0 = static_cast<size_t>(G0 + w) * p.nblk + b0;
                    bulk_g2s(base + w * p.BPS * Geo::TB, p.W + tile0 * Geo::TB, nb * Geo::TB, full);
                    bulk_g2s(base + p.off_S + w * p.BPS * Geo::SB,
                             static_cast<const uint8_t*>(p.S) + tile0 * Geo::SB, nb * Geo::SB, full);
                    if (ZP) {
                        const size_t z0 = (static_cast<size_t>(G0 + w) * p.nblkZ + b0) * 8;
                        bulk_g2s(base + p.off_Z + w * p.BPS * 8, p.Z + z0, ((nb + 1) & ~1) * 8, full);
                    }
                }
            }
            if (acts) {
                if (HP) bulk_g2s(base + p.off_H, p.hs + b0 * act_blk, nb * act_blk, full);
                bulk_g2s(base + p.off_L, p.lo + b0 * act_blk, nb * act_blk, full);
                bulk_g2s(base + p.off_A, p.as + static_cast<size_t>(b0) * MT * 8, nb * MT * 32, full);
            }
        };
        const int first = min(p.STAGES, nst);
        for (int i = 0; i < first; ++i) issue(i, true, false);
        pdl_wait();                                   // activations come from the previous grid
        for (int i = 0; i < first; ++i) issue(i, false, true);
        for (int i = first; i < nst; ++i) {
            const int s = i % p.STAGES;
            if (!mbar_wait(smem_u32(&bars[p.STAGES + s]), ((i / p.STAGES) - 1) & 1, p.err)) return;
            issue(i, true, true);
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    if (warp >= active) return;
    const int G = G0 + warp;
    const int g = lane >> 2, t = lane & 3;

    uint64_t accA[MT], accB[MT];       // (row g | row g+8) x (tokens 2t, 2t+1) per token group
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) { accA[mt] = 0; accB[mt] = 0; }

    const uint64_t negc_lo = f2_pack(-12582912.0f, -12582912.0f);   // single-pass: -1.5*2^23

    for (int i = 0; i < nst; ++i) {
        const int s = i % p.STAGES;
        if (!mbar_wait(smem_u32(&bars[s]), (i / p.STAGES) & 1, p.err)) return;
        const uint8_t* st = stages + static_cast<size_t>(s) * p.stage_bytes;
        const uint8_t* Wst = st + warp * p.BPS * Geo::TB;
        const uint8_t* Sst = st + p.off_S + warp * p.BPS * Geo::SB;
        const uint8_t* Zst = st + p.off_Z + warp * p.BPS * 8;
        const uint8_t* Hst = st + p.off_H;
        const uint8_t* Lst = st + p.off_L;
        const float* Ast = reinterpret_cast<const float*>(st + p.off_A);
        const int b0 = i * p.BPS;
        const int nb = min(p.BPS, p.nblk - b0);
        for (int j = 0; j < nb; ++j) {
            // ---- weights: A fragment of the 16x32 tile
            uint32_t a[4];
            if (BITS == 8) {
                const uint4 v = *reinterpret_cast<const uint4*>(Wst + j * Geo::TB + lane * 16);
                a[0] = v.x; a[1] = v.y; a[2] = v.z; a[3] = v.w;
            } else {
                const uint2 v = *reinterpret_cast<const uint2*>(Wst + j * Geo::TB + lane * 8);
                uint32_t c0 = 0x78787878u, c1 = 0x78787878u;                  // zp = 8
                if (ZP) {
                    const uint32_t z = Zst[j * 8 + g];
                    c0 = (0x80u - (z & 15u)) * 0x01010101u;
                    c1 = (0x80u - (z >> 4)) * 0x01010101u;
                }
                a[0] = nib_even_s8(v.x, c0);
                a[1] = nib_odd_s8(v.x, c1);
                a[2] = nib_even_s8(v.y, c0);
                a[3] = nib_odd_s8(v.y, c1);
            }
            // ---- weight scales for rows g and g+8
            float bs0, bs1;
            if (HALF) {
                const __half2 h = *reinterpret_cast<const __half2*>(Sst + j * Geo::SB + g * 4);
                bs0 = __low2float(h);
                bs1 = __high2float(h);
            } else {
                const float2 f = *reinterpret_cast<const float2*>(Sst + j * Geo::SB + g * 8);
                bs0 = f.x;
                bs1 = f.y;
            }
            const uint64_t bsA = f2_pack(bs0, bs0), bsB = f2_pack(bs1, bs1);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int off = (j * MT + mt) * 256 + g * 16 + t * 4;
                int32_t l[4] = {LO_SEED, LO_SEED, LO_SEED, LO_SEED};
                const uint32_t l0 = *reinterpret_cast<const uint32_t*>(Lst + off);
                const uint32_t l1 = *reinterpret_cast<const uint32_t*>(Lst + off + 128);
                uint64_t yA, yB;
                if (HP) {
                    int32_t h[4] = {HI_SEED, HI_SEED, HI_SEED, HI_SEED};
                    const uint32_t h0 = *reinterpret_cast<const uint32_t*>(Hst + off);
                    const uint32_t h1 = *reinterpret_cast<const uint32_t*>(Hst + off + 128);
                    mma_s8s8(h, a, h0, h1);
                    mma_s8u8(l, a, l0, l1);
                    if (OUT_CS) {
                        const int tok0 = mt * 8 + 2 * t;
                        const int n0 = G * 16 + g;
                        const int b = b0 + j;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int tok = tok0 + (e & 1);
                            const int n = n0 + 8 * (e >> 1);
                            if (tok < p.M)
                                p.CS[(static_cast<size_t>(tok) * p.N + n) * p.nblk + b] =
                                    (h[e] - HI_SEED) * 256 + (l[e] - LO_SEED);
                        }
                        continue;
                    }
                    yA = cs_to_f2(h[0], h[1], l[0], l[1]);
                    yB = cs_to_f2(h[2], h[3], l[2], l[3]);
                } else {
                    mma_s8s8(l, a, l0, l1);
                    if (OUT_CS) {
                        const int tok0 = mt * 8 + 2 * t;
                        const int n0 = G * 16 + g;
                        const int b = b0 + j;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int tok = tok0 + (e & 1);
                            const int n = n0 + 8 * (e >> 1);
                            if (tok < p.M)
                                p.CS[(static_cast<size_t>(tok) * p.N + n) * p.nblk + b] = l[e] - LO_SEED;
                        }
                        continue;
                    }
                    yA = f2_add(i2_pack(l[0], l[1]), negc_lo);     // exact (|cs| < 2^22)
                    yB = f2_add(i2_pack(l[2], l[3]), negc_lo);
                }
                const float2 asv = *reinterpret_cast<const float2*>(Ast + (j * MT + mt) * 8 + 2 * t);
                const uint64_t as2 = f2_pack(asv.x, asv.y);
                accA[mt] = f2_fma(as2, f2_mul(yA, bsA), accA[mt]);
                accB[mt] = f2_fma(as2, f2_mul(yB, bsB), accB[mt]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars[p.STAGES + s]));
    }

    if (OUT_CS) return;
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

// ------------------------------------------------------------------ host side

struct DecodeConfig {
    int R, BPS, STAGES;
};

static int g_num_sms = 0;

constexpr int SMEM_BUDGET = 200 * 1024;   // dynamic shared memory per CTA (of 227 KB)

// Exact bytes of one ring stage (must match the carve-up in launch_t).
static int stage_bytes_for(int R, int BPS, int MT, int tb, int sb, bool zp, bool hp) {
    const int b = R * BPS * (tb + sb + (zp ? 8 : 0)) + (hp ? 2 : 1) * BPS * MT * 256 + BPS * MT * 32;
    return (b + 127) & ~127;
}

static DecodeConfig choose_config(int G, int nblk, int MT, int tb, int sb, bool zp, bool hp) {
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    DecodeConfig c;
    // Enough CTAs for ~2 per SM, as many row groups per CTA as that allows
    // (activation stages are shared by the R row groups of a CTA).
    c.R = 1;
    if (G >= 4 * 2 * g_num_sms) c.R = 4;
    else if (G >= 2 * 2 * g_num_sms) c.R = 2;
    // Stage: BPS blocks (even); aim for ~32 KB of copies in flight per CTA,
    // at least 2 stages, and stay inside the shared-memory budget.
    c.BPS = (c.R == 1) ? 16 : 8;
    const int nblk_even = (nblk + 1) & ~1;
    if (c.BPS > nblk_even) c.BPS = nblk_even;
    if (c.BPS < 2) c.BPS = 2;
    while (c.BPS > 2 && 2 * stage_bytes_for(c.R, c.BPS, MT, tb, sb, zp, hp) > SMEM_BUDGET) c.BPS -= 2;
    const int st = stage_bytes_for(c.R, c.BPS, MT, tb, sb, zp, hp);
    c.STAGES = std::max(3, std::min(8, 32768 / st));
    while (c.STAGES > 2 && c.STAGES * st > SMEM_BUDGET) --c.STAGES;
    return c;
}

template <int BITS, bool HALF, bool ZP, int MT, bool HP, bool OUT_CS>
static cudaError_t launch_t(const DecodeParams& p0, const DecodeConfig& c, cudaStream_t stream, bool pdl) {
    using Geo = WeightGeom<BITS, HALF, ZP>;
    DecodeParams p = p0;
    p.R = c.R;
    p.BPS = c.BPS;
    p.STAGES = c.STAGES;
    uint32_t off = c.R * c.BPS * Geo::TB;
    p.off_S = off;  off += c.R * c.BPS * Geo::SB;
    p.off_Z = off;  off += ZP ? c.R * c.BPS * 8 : 0;
    p.off_H = off;  off += HP ? c.BPS * MT * 256 : 0;
    p.off_L = off;  off += c.BPS * MT * 256;
    p.off_A = off;  off += c.BPS * MT * 32;
    p.stage_bytes = (off + 127) & ~127u;
    const size_t smem = 128 * ((2 * c.STAGES * 8 + 127) / 128) + static_cast<size_t>(c.STAGES) * p.stage_bytes;
    // Host-side guards: the carve-up must match the planner and fit the SM.
    if (static_cast<int>(p.stage_bytes) != stage_bytes_for(c.R, c.BPS, MT, Geo::TB, Geo::SB, ZP, HP) ||
        smem > 227 * 1024 || c.BPS < 2 || (c.BPS & 1) || c.STAGES < 2 || c.R < 1 || c.R > 4)
        return cudaErrorInvalidConfiguration;
    auto kern = decode_kernel<BITS, HALF, ZP, MT, HP, OUT_CS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.G + c.R - 1) / c.R);
    cfg.blockDim = dim3(32 * (c.R + 1));
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
    using Geo = WeightGeom<BITS, HALF, ZP>;
    const DecodeConfig c = choose_config(p.G, p.nblk, MT, Geo::TB, Geo::SB, ZP, HP);
    switch (MT) {
        case 1: return launch_t<BITS, HALF, ZP, 1, HP, OUT_CS>(p, c, stream, pdl);
        case 2: return launch_t<BITS, HALF, ZP, 2, HP, OUT_CS>(p, c, stream, pdl);
        case 4: return launch_t<BITS, HALF, ZP, 4, HP, OUT_CS>(p, c, stream, pdl);
        default: return launch_t<BITS, HALF, ZP, 8, HP, OUT_CS>(p, c, stream, pdl);
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
    DecodeParams p = {};
    p.W = w->W;
    p.S = w->S;
    p.Z = w->Z;
    p.hs = act.hs;
    p.lo = act.lo;
    p.as = act.as;
    p.C = C;
    p.CS = cs;
    p.err = device_error_word();
    p.M = act.M;
    p.N = w->N;
    p.nblk = w->nblk;
    p.nblkZ = w->nblkZ;
    p.G = w->G;
    p.ldc = ldc;
    // The kernel's activation stride per block is MT*256: the token-group
    // count of the template must equal the workspace's.
    const int MT = act.MT;
    if (MT != 1 && MT != 2 && MT != 4 && MT != 8) return cudaErrorInvalidValue;
    if (cs) {
        return hi_prec ? dispatch_w<true, true>(w, p, MT, stream, pdl)
                       : dispatch_w<false, true>(w, p, MT, stream, pdl);
    }
    return hi_prec ? dispatch_w<true, false>(w, p, MT, stream, pdl)
                   : dispatch_w<false, false>(w, p, MT, stream, pdl);
}

}  // namespace ql
