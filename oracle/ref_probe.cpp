// ref_probe.cpp -- TEST INFRASTRUCTURE ONLY (parity checker / CPU baseline).
//
// Compiles the reference's own kernel/quantized_matmul.cpp (included from
// where it lies in the reference checkout; nothing is copied) and adds three
// probe entry points that expose values its public C ABI keeps internal:
//
//   refprobe_quantize_i16  -- the reference quantize_A_i16
//                             (kernel/quantized_matmul.cpp:237-258)
//   refprobe_block_sums    -- the per-block INT32 accumulator
//                             cs = 256*(acc_hi - corr) + acc_lo
//                             (kernel/quantized_matmul.cpp:298-312, 262-268),
//                             recomputed from the handle's packed VNNI bytes
//                             and its stored corr, i.e. from the reference's
//                             own prepacked data, not from the ONNX input.
//   refprobe_replay        -- the FP32 chain acc = fma(ascale, f, acc) over
//                             those block sums (kernel/quantized_matmul.cpp:311-315);
//                             it must equal i4_matmul bit for bit, which
//                             checks that the probe reads the handle correctly.
//
// Built by oracle/Makefile into oracle/_ref/ (git-ignored).  The compiled
// library also exports the reference C ABI (i4_prepack_onnx, i4_matmul,
// i4_free, i4_set_hi_prec, i4_set_threads, ...), which is what bench.py's
// reference arm times.
#include "quantized_matmul.cpp"

namespace {

int packed_value(const PackedWeight* P, int n, int k) {
    const int t = n / 16, col = n % 16, kb = k / 32, g = (k % 32) / 4, j = k % 4;
    const size_t out_block = size_t(t) * P->nblk + kb;
    if (P->bits == 8) {
        const int8_t* dest = reinterpret_cast<const int8_t*>(P->B) + out_block * 8 * 64;
        return dest[g * 64 + col * 4 + j];
    }
    const uint8_t* dest = P->B + out_block * 8 * 32;
    const uint8_t byte = dest[g * 32 + col * 2 + j / 2];
    const int nib = (j & 1) ? (byte >> 4) : (byte & 15);
    return nib - P->zp[out_block * 16 + col];
}

}  // namespace

extern "C" {

void refprobe_quantize_i16(const float* A, int M, int K, uint8_t* hi, uint8_t* lo,
                           float* ascale) {
    quantize_A_i16(A, M, K, K / 32, hi, lo, ascale);
}

// cs: [M, N, nblk] int32.
int refprobe_block_sums(void* handle, const uint8_t* hi, const uint8_t* lo, int M,
                        int32_t* cs) {
    const auto* P = static_cast<const PackedWeight*>(handle);
    if (!P) return -1;
    const int N = P->N, K = P->K, nblk = P->nblk;
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            const int t = n / 16, col = n % 16;
            for (int kb = 0; kb < nblk; ++kb) {
                const size_t meta = (size_t(t) * nblk + kb) * 16 + col;
                int32_t acc_hi = 0, acc_lo = 0;
                for (int i = 0; i < 32; ++i) {
                    const int k = kb * 32 + i;
                    const int b = packed_value(P, n, k);
                    acc_hi += int32_t(hi[size_t(m) * K + k]) * b;
                    acc_lo += int32_t(lo[size_t(m) * K + k]) * b;
                }
                cs[(size_t(m) * N + n) * nblk + kb] = 256 * (acc_hi - P->corr[meta]) + acc_lo;
            }
        }
    return 0;
}

// Replays the reference FP32 chain over block sums with the handle's scales.
int refprobe_replay(void* handle, const int32_t* cs, const float* ascale, int M, float* C) {
    const auto* P = static_cast<const PackedWeight*>(handle);
    if (!P) return -1;
    const int N = P->N, nblk = P->nblk;
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            const int t = n / 16, col = n % 16;
            float acc = 0.0f;
            for (int kb = 0; kb < nblk; ++kb) {
                const float bscale = P->scales[(size_t(t) * nblk + kb) * 16 + col];
                const float f = float(cs[(size_t(m) * N + n) * nblk + kb]) * bscale;
                acc = std::fma(ascale[size_t(m) * nblk + kb], f, acc);
            }
            C[size_t(m) * N + n] = acc;
        }
    return 0;
}

}  // extern "C"
