// ql_api.cu -- the C ABI of libbreeze_ql.so (declared in include/breeze_ql.h).
//
// Reference-compatible entry points mirror kernel/quantized_matmul.cpp:472-574
// (i4_set_threads, i4_set_numa_split, i4_set_hi_prec, i4_prepack,
// i4_prepack_onnx, i4_free, i4_matmul) with the same argument meaning and the
// same failure behaviour (nullptr handle on a bad contract).  They take host
// pointers and are synchronous, so an unchanged ctypes or C++ caller works.
// The ql_* entry points take device pointers and a cudaStream_t (as void*),
// enqueue asynchronously and return an int status (0 = OK).
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <vector>
#include "ql_common.cuh"
#include "ql_internal.h"

#if defined(__GNUC__)
#define QL_API extern "C" __attribute__((visibility("default")))
#else
#define QL_API extern "C"
#endif

namespace ql {

// The device control block (ql_common.cuh): error word and wait limits.
__device__ DeviceCtl g_device_ctl = {0, 0, WAIT_LIMIT_NS, PEER_WAIT_LIMIT_NS};

namespace {

constexpr int MAX_DEVICES = 64;

std::mutex g_mu;
int g_hi_prec = 0;              // reference default: INT8 single pass (quantized_matmul.cpp:35)
thread_local int g_last_status = QL_OK;
thread_local cudaError_t g_last_cuda = cudaSuccess;

struct DeviceState {
    int* err_word = nullptr;
    cudaStream_t stream = nullptr;   // for the synchronous host-pointer entry points
    void* buf = nullptr;             // host-pointer staging: A, C and the activation workspace
    size_t buf_bytes = 0;
    void* ws = nullptr;              // workspace for ql_matmul_dev without a caller workspace
    size_t ws_bytes = 0;
    cudaStream_t copy_stream = nullptr;   // i4_matmul: output copies overlapping the matmul
    cudaEvent_t chunk_done[8] = {};       // i4_matmul: one per output column chunk
    int* host_err = nullptr;              // pinned copy of the device error word (i4_matmul)
    cudaEvent_t copies_done = nullptr;    // i4_matmul: the output copies joined back into the call's stream
};
DeviceState g_dev[MAX_DEVICES];

int set_status(int s, cudaError_t e = cudaSuccess) {
    g_last_status = s;
    if (e != cudaSuccess) g_last_cuda = e;
    return s;
}

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return set_status(QL_OK);
    if (e == cudaErrorMemoryAllocation) return set_status(QL_ENOMEM, e);
    return set_status(QL_ECUDA, e);
}

// RAII: make `dev` current for the scope of a call, restore afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) { ok = false; return; }
        if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

DeviceState* state_for(int dev) {
    if (dev < 0 || dev >= MAX_DEVICES) return nullptr;
    return &g_dev[dev];
}

// Grow-only device buffer (caller holds g_mu and has the right device current).
cudaError_t ensure(void** p, size_t* have, size_t need) {
    if (*have >= need) return cudaSuccess;
    if (*p) {
        cudaFree(*p);   // implicit device synchronisation: no kernel still uses it
        *p = nullptr;
        *have = 0;
    }
    cudaError_t e = cudaMalloc(p, need);
    if (e == cudaSuccess) *have = need;
    return e;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

Weight* allocate_weight(int N, int K, int bits, int scale_half, int has_zp) {
    if (N <= 0 || K <= 0 || N % 16 || K % 32 || (bits != 4 && bits != 8)) return nullptr;
    auto* w = new (std::nothrow) Weight{};
    if (!w) return nullptr;
    w->magic = WEIGHT_MAGIC;
    w->N = N;
    w->K = K;
    w->nblk = K / 32;
    w->bits = bits;
    w->scale_half = scale_half;
    w->has_zp = has_zp;
    w->G = N / 16;
    weight_geometry(bits, scale_half != 0, has_zp != 0, &w->TB, &w->SB, &w->ZB, &w->REC);
    cudaGetDevice(&w->device);
    const size_t tiles = static_cast<size_t>(w->G) * w->nblk;
    const size_t bytes = align256(tiles * w->REC);
    uint8_t* base = nullptr;
    if (cudaMalloc(&base, bytes) != cudaSuccess) {
        cudaGetLastError();
        delete w;
        return nullptr;
    }
    w->W = base;
    w->bytes = bytes;
    return w;
}

void free_weight(Weight* w) {
    if (!w) return;
    w->magic = 0;
    if (w->W) {
        DeviceGuard g(w->device);
        cudaFree(w->W);
    }
    delete w;
}

cudaStream_t internal_stream(DeviceState* st) {
    if (!st->stream) cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking);
    return st->stream;
}

// M > 64 tokens run the tcgen05 GEMM (ql_gemm.cu) unless BREEZE_QL_PREFILL=decode
// asks for the decode kernel over 64-token chunks (kept for comparison).
bool use_gemm(int M) {
    static const int force_decode = [] {
        const char* v = std::getenv("BREEZE_QL_PREFILL");
        return (v && std::strcmp(v, "decode") == 0) ? 1 : 0;
    }();
    return M > MAX_DECODE_TOKENS && !force_decode;
}

// Workspace for M tokens of K inputs: GEMM activation records for the tcgen05
// path, else one decode activation chunk per 64 tokens laid out by act_carve.
size_t chunk_bytes(int M, int nblk) { return act_bytes(std::min(M, MAX_DECODE_TOKENS), nblk); }
size_t ws_bytes_for(int M, int nblk) {
    if (M <= 0) return 0;
    if (use_gemm(M)) return gemm_act_bytes(M, nblk);
    const size_t chunks = static_cast<size_t>((M + MAX_DECODE_TOKENS - 1) / MAX_DECODE_TOKENS);
    return chunks * chunk_bytes(M, nblk);
}

// The INT4 FP16-operand prefill (ql_gemmw.cu) runs when the selector is
// automatic and the weight qualifies (INT4, fp16 scales); its workspace holds
// the FP16 activation records (sized for two-pass, the larger) and then the
// call's dequantized weights.
bool gemmw_applies(const Weight* w, int M) {
    return use_gemm(M) && gemmw_supports(w) && prefill_kernel() == QL_PREFILL_AUTO;
}
size_t gemmw_act_region(int M, int nblk) { return align256(gemmw_act_bytes(M, nblk, true)); }
size_t gemmw_ws_bytes(const Weight* w, int M) {
    return gemmw_act_region(M, w->nblk) + gemmw_weight_bytes(w);
}
// The workspace one call on `w` asks for (ql_workspace_bytes): the FP16-operand
// path's where it applies, else the quantized-activation records.
size_t ws_bytes_for_w(const Weight* w, int M) {
    const size_t base = ws_bytes_for(M, w->nblk);
    return gemmw_applies(w, M) ? std::max(base, gemmw_ws_bytes(w, M)) : base;
}

// Dequantize the weights and quantize A into the FP16-operand workspace.
int run_gemmw_prep(const Weight* w, const float* dA, int M, uint8_t* ws, cudaStream_t stream, bool hi_prec) {
    cudaError_t e = launch_dequant_w16(w, hi_prec, ws + gemmw_act_region(M, w->nblk), stream);
    if (e == cudaSuccess) e = launch_quantize_f16(dA, w->K, M, w->K, hi_prec, ws, stream);
    return cuda_status(e);
}

ActView chunk_view(void* ws, int M, int nblk, int c, bool hi_prec) {
    const int m0 = c * MAX_DECODE_TOKENS;
    const int mc = std::min(MAX_DECODE_TOKENS, M - m0);
    return act_carve(static_cast<uint8_t*>(ws) + static_cast<size_t>(c) * chunk_bytes(M, nblk), mc, nblk, hi_prec);
}

int run_quantize(const float* dA, int M, int K, void* ws, cudaStream_t stream, bool hi_prec) {
    const int nblk = K / 32;
    if (use_gemm(M))
        return cuda_status(launch_quantize_gemm(dA, K, M, K, hi_prec, static_cast<uint8_t*>(ws), stream));
    for (int c = 0; c * MAX_DECODE_TOKENS < M; ++c) {
        const ActView act = chunk_view(ws, M, nblk, c, hi_prec);
        cudaError_t e = launch_quantize_act(dA + static_cast<size_t>(c) * MAX_DECODE_TOKENS * K, K,
                                            act.M, K, hi_prec, act, stream);
        if (e != cudaSuccess) return cuda_status(e);
    }
    return set_status(QL_OK);
}

int run_compute(const Weight* w, const void* ws, int M, float* dC, int32_t* dCS, cudaStream_t stream,
                bool hi_prec, bool pdl, int ldc = 0) {
    if (ldc <= 0) ldc = w->N;
    if (use_gemm(M))
        return cuda_status(launch_gemm(w, static_cast<const uint8_t*>(ws), M, hi_prec, dC, ldc, dCS, stream));
    for (int c = 0; c * MAX_DECODE_TOKENS < M; ++c) {
        const ActView act = chunk_view(const_cast<void*>(ws), M, w->nblk, c, hi_prec);
        const size_t m0 = static_cast<size_t>(c) * MAX_DECODE_TOKENS;
        cudaError_t e = launch_decode(w, act, hi_prec, dC ? dC + m0 * ldc : nullptr, ldc,
                                      dCS ? dCS + m0 * w->N * w->nblk : nullptr, stream, pdl);
        if (e != cudaSuccess) return cuda_status(e);
    }
    return set_status(QL_OK);
}

// Quantize + matmul into a caller workspace of >= ws_bytes_for(M, nblk) bytes.
// Every kernel of the chain is launched with programmatic dependent launch and
// triggers its dependents early, so the next kernel streams its weights while
// the previous one drains; each waits (griddepcontrol.wait) for its predecessor
// before it reads activations or writes anything.
int run_matmul(const Weight* w, const float* dA, int M, float* dC, int32_t* dCS, void* ws,
               size_t ws_bytes, cudaStream_t stream, bool hi_prec) {
    if (reinterpret_cast<uintptr_t>(ws) % 16) return set_status(QL_EINVAL);   // 16-byte bulk copies
    if (gemmw_applies(w, M) && ws_bytes >= gemmw_ws_bytes(w, M)) {
        // INT4 prefill with room for the FP16 operands: dequantize once, then
        // the FP16-operand GEMM (a smaller workspace runs the streaming GEMM)
        uint8_t* base = static_cast<uint8_t*>(ws);
        int rc = run_gemmw_prep(w, dA, M, base, stream, hi_prec);
        if (rc != QL_OK) return rc;
        return cuda_status(launch_gemmw(w, base + gemmw_act_region(M, w->nblk), base, M, hi_prec, dC, w->N, dCS,
                                        stream));
    }
    if (ws_bytes < ws_bytes_for(M, w->nblk)) return set_status(QL_EINVAL);
    int rc = run_quantize(dA, M, w->K, ws, stream, hi_prec);
    if (rc != QL_OK) return rc;
    return run_compute(w, ws, M, dC, dCS, stream, hi_prec, /*pdl=*/true);
}

}  // namespace

int* device_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    DeviceState* st = state_for(dev);
    if (!st) return nullptr;
    if (!st->err_word) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_ctl) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        st->err_word = static_cast<int*>(p);
    }
    return st->err_word;
}

}  // namespace ql

using namespace ql;

// ------------------------------------------------------------------ settings

QL_API int ql_version(void) { return 1; }

QL_API int ql_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// i4_set_threads (kernel/quantized_matmul.cpp:474): accepted for source
// compatibility; the GPU kernels' results never depend on a thread count.
QL_API void i4_set_threads(int n) { (void)n; }

// i4_set_numa_split (:475): accepted, no NUMA replica on the GPU.
QL_API void i4_set_numa_split(int cpu) { (void)cpu; }

// i4_set_hi_prec (:476): process-global activation mode.
QL_API void i4_set_hi_prec(int on) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_hi_prec = on ? 1 : 0;
}

QL_API int ql_get_hi_prec(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_hi_prec;
}

// Prefill (M > 64) kernel selector: 0 = automatic (the single-CTA kind::f16
// GEMM for INT4 weights with fp16 scales in two-pass mode, else kind::i8), 1 =
// always kind::i8, 2 = the CTA-pair kind::f16 GEMM where it applies.  All give
// the same bits; process-global like i4_set_hi_prec.
static std::atomic<int> g_prefill_kernel{ql::QL_PREFILL_AUTO};
namespace ql {
int prefill_kernel() { return g_prefill_kernel.load(std::memory_order_relaxed); }
}  // namespace ql

QL_API int ql_set_prefill_kernel(int kind) {
    if (kind != ql::QL_PREFILL_AUTO && kind != ql::QL_PREFILL_I8 && kind != ql::QL_PREFILL_F16_PAIR &&
        kind != ql::QL_PREFILL_F16_STREAM)
        return set_status(QL_EINVAL);
    g_prefill_kernel.store(kind, std::memory_order_relaxed);
    return set_status(QL_OK);
}

// Limits of the bounded device waits on the current device: kernel-internal
// waits (default 1 s) and waits on another GPU's flags (default 5 s).  0 keeps
// a limit as it is.  Serialise with running calls.
QL_API int ql_set_wait_limits(unsigned long long wait_ns, unsigned long long peer_wait_ns) {
    int* w = device_error_word();
    if (!w) return set_status(QL_ECUDA);
    DeviceCtl* ctl = reinterpret_cast<DeviceCtl*>(w);
    cudaError_t e = cudaSuccess;
    if (wait_ns) e = cudaMemcpy(&ctl->wait_ns, &wait_ns, sizeof(wait_ns), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && peer_wait_ns)
        e = cudaMemcpy(&ctl->peer_wait_ns, &peer_wait_ns, sizeof(peer_wait_ns), cudaMemcpyHostToDevice);
    return cuda_status(e);
}

QL_API const char* ql_error_string(int code) {
    switch (code) {
        case QL_OK: return "ok";
        case QL_EINVAL: return "invalid argument";
        case QL_ENOMEM: return "device allocation failed";
        case QL_ECUDA: return "CUDA runtime error";
        case QL_ETIMEOUT: return "bounded device wait timed out";
        case QL_EDEVICE: return "handle belongs to another device";
        case QL_ENOTSUP: return "unsupported configuration";
        case QL_ESCRATCH: return "request exceeds the fixed scratch of ql_matmul_dev_noalloc";
        default: return "unknown error";
    }
}

QL_API int ql_last_status(void) { return g_last_status; }

QL_API const char* ql_last_cuda_error_string(void) { return cudaGetErrorString(g_last_cuda); }

// Reads (and optionally clears) the current device's error word, which kernels
// set instead of trapping when a bounded wait gives up.  Synchronises the device.
QL_API int ql_device_error(int clear) {
    int* w = device_error_word();
    if (!w) return set_status(QL_ECUDA);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_status(e);
    int v = 0;
    e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_status(e);
    if (clear && v) {
        const int z = 0;
        cudaMemcpy(w, &z, sizeof(int), cudaMemcpyHostToDevice);
    }
    return v;
}

// ------------------------------------------------------------------ prepack

// i4_prepack_onnx (kernel/quantized_matmul.cpp:505-520): host MatMulNBits
// arrays -> owning handle on the current device; nullptr on a bad contract
// (N,K <= 0, N%16, K%32, bits not 4/8, scale_bits not 16/32, INT8 with
// qzeros) or allocation failure.  Inputs are deep-copied; the caller may free
// them as soon as the call returns.
QL_API void* i4_prepack_onnx(const uint8_t* qw, const void* scales, const uint8_t* qzeros, int N,
                             int K, int bits, int scale_bits) {
    if (!qw || !scales || (scale_bits != 16 && scale_bits != 32) || (bits == 8 && qzeros) || N <= 0 || K <= 0 ||
        N % 16 || K % 32 || (bits != 4 && bits != 8)) {
        set_status(QL_EINVAL);
        return nullptr;
    }
    Weight* w = allocate_weight(N, K, bits, scale_bits == 16, bits == 4 && qzeros != nullptr);
    if (!w) {
        set_status(QL_ENOMEM);
        return nullptr;
    }
    const size_t nblk = w->nblk;
    const size_t qw_bytes = static_cast<size_t>(N) * nblk * (4 * bits);
    const size_t sc_bytes = static_cast<size_t>(N) * nblk * (scale_bits / 8);
    const size_t qz_bytes = w->has_zp ? static_cast<size_t>(N) * ((nblk + 1) / 2) : 0;
    uint8_t* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, align256(qw_bytes) + align256(sc_bytes) + align256(qz_bytes));
    if (e != cudaSuccess) {
        cudaGetLastError();
        free_weight(w);
        set_status(QL_ENOMEM);
        return nullptr;
    }
    uint8_t* d_qw = tmp;
    uint8_t* d_sc = tmp + align256(qw_bytes);
    uint8_t* d_qz = d_sc + align256(sc_bytes);
    cudaStream_t s = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        s = internal_stream(state_for(w->device));
    }
    e = cudaMemcpyAsync(d_qw, qw, qw_bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_sc, scales, sc_bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && qz_bytes) e = cudaMemcpyAsync(d_qz, qzeros, qz_bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = launch_prepack_onnx(w, d_qw, d_sc, w->has_zp ? d_qz : nullptr, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(tmp);
    if (e != cudaSuccess) {
        cuda_status(e);
        free_weight(w);
        return nullptr;
    }
    set_status(QL_OK);
    return w;
}

// Device-pointer prepack: the same contract with MatMulNBits arrays already in
// device memory, enqueued on `stream` (inputs must stay alive until it drains).
QL_API int ql_prepack_onnx_dev(const uint8_t* d_qw, const void* d_scales, const uint8_t* d_qzeros,
                               int N, int K, int bits, int scale_bits, void* stream,
                               void** out_handle) {
    if (!out_handle) return set_status(QL_EINVAL);
    *out_handle = nullptr;
    if (!d_qw || !d_scales || (scale_bits != 16 && scale_bits != 32) || (bits == 8 && d_qzeros))
        return set_status(QL_EINVAL);
    if (N <= 0 || K <= 0 || N % 16 || K % 32 || (bits != 4 && bits != 8)) return set_status(QL_EINVAL);
    Weight* w = allocate_weight(N, K, bits, scale_bits == 16, bits == 4 && d_qzeros != nullptr);
    if (!w) return set_status(QL_ENOMEM);
    cudaError_t e = launch_prepack_onnx(w, d_qw, d_scales, w->has_zp ? d_qzeros : nullptr,
                                        static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        free_weight(w);
        return cuda_status(e);
    }
    *out_handle = w;
    return set_status(QL_OK);
}

// i4_prepack (kernel/quantized_matmul.cpp:480-499): legacy entry taking the
// reference's already-transformed VNNI layout (srcB [N/16][nblk][8][32|64],
// srcScale fp32 [N/16][nblk][16], srcZp int8 [N/16][nblk][16] for INT4,
// srcCorr int32, which this library recomputes implicitly and ignores).
// INT4 zero points must lie in 0..15 (the MatMulNBits range).
QL_API void* i4_prepack(const uint8_t* srcB, const float* srcScale, const int8_t* srcZp,
                        const int32_t* srcCorr, int N, int K, int nblk, int bits) {
    if (!srcB || !srcScale || !srcCorr || (bits == 4 && !srcZp) || nblk != K / 32 || N <= 0 ||
        K <= 0 || N % 16 || K % 32 || (bits != 4 && bits != 8)) {
        set_status(QL_EINVAL);
        return nullptr;
    }
    const size_t metas = static_cast<size_t>(N) * nblk;
    if (bits == 4) {
        for (size_t i = 0; i < metas; ++i)
            if (srcZp[i] < 0 || srcZp[i] > 15) {
                set_status(QL_EINVAL);
                return nullptr;
            }
    }
    Weight* w = allocate_weight(N, K, bits, 0, bits == 4);
    if (!w) {
        set_status(QL_ENOMEM);
        return nullptr;
    }
    const size_t b_bytes = metas * (bits == 8 ? 32 : 16);
    const size_t s_bytes = metas * 4;
    const size_t z_bytes = bits == 4 ? metas : 0;
    uint8_t* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, align256(b_bytes) + align256(s_bytes) + align256(z_bytes));
    if (e != cudaSuccess) {
        cudaGetLastError();
        free_weight(w);
        set_status(QL_ENOMEM);
        return nullptr;
    }
    uint8_t* d_b = tmp;
    float* d_s = reinterpret_cast<float*>(tmp + align256(b_bytes));
    int8_t* d_z = reinterpret_cast<int8_t*>(tmp + align256(b_bytes) + align256(s_bytes));
    cudaStream_t s = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        s = internal_stream(state_for(w->device));
    }
    e = cudaMemcpyAsync(d_b, srcB, b_bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_s, srcScale, s_bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && z_bytes) e = cudaMemcpyAsync(d_z, srcZp, z_bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = launch_prepack_vnni(w, d_b, d_s, bits == 4 ? d_z : nullptr, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(tmp);
    if (e != cudaSuccess) {
        cuda_status(e);
        free_weight(w);
        return nullptr;
    }
    set_status(QL_OK);
    return w;
}

// i4_free (:522-524): null-safe.
QL_API void i4_free(void* handle) {
    if (!valid_weight(handle)) return;
    free_weight(static_cast<Weight*>(handle));
}

QL_API int ql_weight_info(const void* handle, int* N, int* K, int* bits, int* device,
                          unsigned long long* bytes) {
    if (!valid_weight(handle)) return set_status(QL_EINVAL);
    const auto* w = static_cast<const Weight*>(handle);
    if (N) *N = w->N;
    if (K) *K = w->K;
    if (bits) *bits = w->bits;
    if (device) *device = w->device;
    if (bytes) *bytes = w->bytes;
    return set_status(QL_OK);
}

// ------------------------------------------------------------------ packed-layout cache
// A packed handle serialised to host bytes: a fixed header, then the device
// records byte for byte.  Loading skips the MatMulNBits repack entirely (one
// host -> device copy per weight).  The header pins the record geometry and
// the library's layout version; a mismatch, a short buffer or a wrong payload
// checksum is rejected with QL_EINVAL before any device memory is touched.
namespace {
constexpr char PACK_MAGIC[8] = {'Q', 'L', 'P', 'A', 'C', 'K', '1', 0};
constexpr uint32_t PACK_VERSION = 1;     // record layout of ql_internal.h
struct PackHeader {
    char magic[8];
    uint32_t version, header_bytes;
    int32_t N, K, bits, scale_half, has_zp, REC;
    uint64_t payload_bytes;              // G * nblk * REC
    uint64_t checksum;                   // wrapping sum of the payload's 64-bit words (x odd index weights)
};
static_assert(sizeof(PackHeader) == 56, "packed-layout header");

uint64_t payload_checksum(const uint8_t* p, size_t n) {
    uint64_t sum = 0x9E3779B97F4A7C15ull;
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        uint64_t v;
        std::memcpy(&v, p + i, 8);
        sum += v * (2 * (i >> 3) + 1);
    }
    for (; i < n; ++i) sum += static_cast<uint64_t>(p[i]) << ((i & 7) * 8);
    return sum;
}
}  // namespace

QL_API size_t ql_weight_serialized_bytes(const void* handle) {
    if (!valid_weight(handle)) return 0;
    const auto* w = static_cast<const Weight*>(handle);
    return sizeof(PackHeader) + static_cast<size_t>(w->G) * w->nblk * w->REC;
}

QL_API int ql_weight_serialize(const void* handle, void* host_buf, size_t bytes) {
    if (!valid_weight(handle) || !host_buf) return set_status(QL_EINVAL);
    const auto* w = static_cast<const Weight*>(handle);
    const size_t payload = static_cast<size_t>(w->G) * w->nblk * w->REC;
    if (bytes < sizeof(PackHeader) + payload) return set_status(QL_EINVAL);
    DeviceGuard guard(w->device);
    if (!guard.ok) return set_status(QL_ECUDA);
    uint8_t* out = static_cast<uint8_t*>(host_buf);
    cudaError_t e = cudaMemcpy(out + sizeof(PackHeader), w->W, payload, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_status(e);
    PackHeader h{};
    std::memcpy(h.magic, PACK_MAGIC, 8);
    h.version = PACK_VERSION;
    h.header_bytes = sizeof(PackHeader);
    h.N = w->N;
    h.K = w->K;
    h.bits = w->bits;
    h.scale_half = w->scale_half;
    h.has_zp = w->has_zp;
    h.REC = w->REC;
    h.payload_bytes = payload;
    h.checksum = payload_checksum(out + sizeof(PackHeader), payload);
    std::memcpy(out, &h, sizeof(h));
    return set_status(QL_OK);
}

QL_API int ql_weight_deserialize(const void* host_buf, size_t bytes, void** out_handle) {
    if (!out_handle) return set_status(QL_EINVAL);
    *out_handle = nullptr;
    if (!host_buf || bytes < sizeof(PackHeader)) return set_status(QL_EINVAL);
    PackHeader h;
    std::memcpy(&h, host_buf, sizeof(h));
    if (std::memcmp(h.magic, PACK_MAGIC, 8) != 0 || h.version != PACK_VERSION ||
        h.header_bytes != sizeof(PackHeader))
        return set_status(QL_EINVAL);
    if (h.N <= 0 || h.K <= 0 || h.N % 16 || h.K % 32 || (h.bits != 4 && h.bits != 8) ||
        (h.scale_half != 0 && h.scale_half != 1) || (h.has_zp != 0 && h.has_zp != 1) || (h.bits == 8 && h.has_zp))
        return set_status(QL_EINVAL);
    int TB, SB, ZB, REC;
    weight_geometry(h.bits, h.scale_half != 0, h.has_zp != 0, &TB, &SB, &ZB, &REC);
    const size_t payload = static_cast<size_t>(h.N / 16) * (h.K / 32) * REC;
    if (h.REC != REC || h.payload_bytes != payload || bytes < sizeof(PackHeader) + payload)
        return set_status(QL_EINVAL);
    const uint8_t* src = static_cast<const uint8_t*>(host_buf) + sizeof(PackHeader);
    if (payload_checksum(src, payload) != h.checksum) return set_status(QL_EINVAL);
    Weight* w = allocate_weight(h.N, h.K, h.bits, h.scale_half, h.has_zp);
    if (!w) return set_status(QL_ENOMEM);
    cudaError_t e = cudaMemcpy(w->W, src, payload, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        free_weight(w);
        return cuda_status(e);
    }
    *out_handle = w;
    return set_status(QL_OK);
}

// ------------------------------------------------------------------ matmul

// Workspace bytes ql_matmul_dev_ws needs for M rows (0 for M <= 0).
QL_API size_t ql_workspace_bytes(const void* handle, int M) {
    if (!valid_weight(handle) || M <= 0) return 0;
    const auto* w = static_cast<const Weight*>(handle);
    return ws_bytes_for_w(w, M);
}

static int check_call(const void* handle, const float* dA, int M, const void* dOut) {
    if (!valid_weight(handle) || M < 0) return QL_EINVAL;
    if (M == 0) return QL_OK;
    if (!dA || !dOut) return QL_EINVAL;
    if (reinterpret_cast<uintptr_t>(dA) % 16) return QL_EINVAL;     // 16-byte vector loads
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return QL_ECUDA;
    if (dev != static_cast<const Weight*>(handle)->device) return QL_EDEVICE;
    return QL_OK;
}

// C[M,N] = matmul(A[M,K]) with a caller workspace of >= ql_workspace_bytes().
// The handle's device must be current.  Asynchronous on `stream`.
QL_API int ql_matmul_dev_ws(void* handle, const float* dA, int M, float* dC, void* ws,
                            size_t ws_bytes, void* stream) {
    const int c = check_call(handle, dA, M, dC);
    if (c != QL_OK || M == 0) return set_status(c);
    if (!ws) return set_status(QL_EINVAL);
    return run_matmul(static_cast<Weight*>(handle), dA, M, dC, nullptr, ws, ws_bytes,
                      static_cast<cudaStream_t>(stream), ql_get_hi_prec() != 0);
}

// Same, with the library's per-device workspace.  Calls that share a device
// are serialised on the host; the workspace is reused in stream order.
QL_API int ql_matmul_dev(void* handle, const float* dA, int M, float* dC, void* stream) {
    const int c = check_call(handle, dA, M, dC);
    if (c != QL_OK || M == 0) return set_status(c);
    const auto* w = static_cast<const Weight*>(handle);
    const bool hp = ql_get_hi_prec() != 0;
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState* st = state_for(w->device);
    const size_t need = ws_bytes_for_w(w, M);
    cudaError_t e = ensure(&st->ws, &st->ws_bytes, need);
    if (e != cudaSuccess) return cuda_status(e);
    return run_matmul(w, dA, M, dC, nullptr, st->ws, st->ws_bytes, static_cast<cudaStream_t>(stream), hp);
}

// Scratch bytes for M quantized activation rows of width K (0 for M <= 0).
QL_API size_t ql_act_workspace_bytes(int M, int K) {
    if (M <= 0 || K <= 0 || K % 32) return 0;
    return ws_bytes_for(M, K / 32);
}

// Quantize activations once into `ws` (the kernels' layout) so several
// weights that share the input (Q/K/V, gate/up) reuse them.
QL_API int ql_quantize_act_dev(const float* dA, int M, int K, int hi_prec, void* ws, size_t ws_bytes,
                               void* stream) {
    if (M < 0 || K <= 0 || K % 32) return set_status(QL_EINVAL);
    if (M == 0) return set_status(QL_OK);
    if (!dA || !ws || reinterpret_cast<uintptr_t>(dA) % 16 || reinterpret_cast<uintptr_t>(ws) % 16 ||
        ws_bytes < ws_bytes_for(M, K / 32))
        return set_status(QL_EINVAL);
    return run_quantize(dA, M, K, ws, static_cast<cudaStream_t>(stream), hi_prec != 0);
}

// C[M,N] from activations quantized by ql_quantize_act_dev with the same M, K
// and hi_prec.  Up to 64 tokens stream the packed weights once per call; more
// tokens run the tensor-core GEMM (or, with BREEZE_QL_PREFILL=decode, stream
// them once per 64-token chunk).
QL_API int ql_matmul_quantized_dev(void* handle, const void* ws, int M, int hi_prec, float* dC,
                                   void* stream) {
    if (!valid_weight(handle) || M < 0) return set_status(QL_EINVAL);
    if (M == 0) return set_status(QL_OK);
    if (!ws || !dC || reinterpret_cast<uintptr_t>(ws) % 16) return set_status(QL_EINVAL);
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return set_status(QL_ECUDA);
    const auto* w = static_cast<const Weight*>(handle);
    if (dev != w->device) return set_status(QL_EDEVICE);
    return run_compute(w, ws, M, dC, nullptr, static_cast<cudaStream_t>(stream), hi_prec != 0, true);
}

// ------------------------------------------------------------------ fused RMSNorm prologue
//
// The reference decoder runs rmsnorm into a scratch row and then i4_matmul on
// it (kernel/qwen35_decoder.cpp:133-141, 405-407), which re-reads the row to
// quantize it.  Here the row factors are computed once (ql_norm.cu) and the
// quantizer applies x * inv * w while it loads the row, so the normalised
// activations never round-trip through memory unless the caller asks for them.
// Workspace: the quantized activations, then M fp32 row factors.
namespace {
size_t norm_ws_bytes(int M, int nblk) {
    return align256(ws_bytes_for(M, nblk)) + align256(static_cast<size_t>(M) * sizeof(float));
}

int run_quantize_norm(const float* dX, const float* dW, float eps, int M, int K, void* ws, float* dHn,
                      cudaStream_t stream, bool hi_prec) {
    const int nblk = K / 32;
    if (use_gemm(M)) {
        // row factors into the workspace's tail, then the GEMM-layout quantizer
        float* row_inv = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + align256(ws_bytes_for(M, nblk)));
        cudaError_t e = launch_rmsnorm_factors(dX, K, M, K, eps, row_inv, stream);
        if (e != cudaSuccess) return cuda_status(e);
        const NormArgs n{row_inv, dW, dHn, K};
        return cuda_status(launch_quantize_gemm(dX, K, M, K, hi_prec, static_cast<uint8_t*>(ws), stream, &n));
    }
    for (int c = 0; c * MAX_DECODE_TOKENS < M; ++c) {    // factors and quantizer in one launch per chunk
        const ActView act = chunk_view(ws, M, nblk, c, hi_prec);
        const size_t m0 = static_cast<size_t>(c) * MAX_DECODE_TOKENS;
        const NormArgs n{nullptr, dW, dHn ? dHn + m0 * K : nullptr, K};
        cudaError_t e = launch_quantize_act_norm(dX + m0 * K, K, act.M, K, eps, hi_prec, act, n, stream);
        if (e != cudaSuccess) return cuda_status(e);
    }
    return set_status(QL_OK);
}

int check_norm_args(const float* dX, const float* dW, int M, int K, const float* dHn) {
    if (M < 0 || K <= 0 || K % 32) return QL_EINVAL;
    if (M == 0) return QL_OK;
    if (!dX || !dW) return QL_EINVAL;
    if (reinterpret_cast<uintptr_t>(dX) % 16 || reinterpret_cast<uintptr_t>(dW) % 16 ||
        reinterpret_cast<uintptr_t>(dHn) % 16)
        return QL_EINVAL;        // 16-byte vector loads and stores
    return QL_OK;
}
}  // namespace

QL_API size_t ql_norm_act_workspace_bytes(int M, int K) {
    if (M <= 0 || K <= 0 || K % 32) return 0;
    return norm_ws_bytes(M, K / 32);
}

QL_API int ql_quantize_act_rmsnorm_dev(const float* dX, const float* dNormW, float eps, int M, int K,
                                       int hi_prec, void* ws, size_t ws_bytes, float* dHn, void* stream) {
    const int c = check_norm_args(dX, dNormW, M, K, dHn);
    if (c != QL_OK || M == 0) return set_status(c);
    if (!ws || reinterpret_cast<uintptr_t>(ws) % 16 || ws_bytes < norm_ws_bytes(M, K / 32))
        return set_status(QL_EINVAL);
    return run_quantize_norm(dX, dNormW, eps, M, K, ws, dHn, static_cast<cudaStream_t>(stream), hi_prec != 0);
}

QL_API int ql_matmul_rmsnorm_dev(void* handle, const float* dX, const float* dNormW, float eps, int M,
                                 float* dC, void* stream) {
    int c = check_call(handle, dX, M, dC);
    if (c != QL_OK || M == 0) return set_status(c);
    const auto* w = static_cast<const Weight*>(handle);
    c = check_norm_args(dX, dNormW, M, w->K, nullptr);
    if (c != QL_OK) return set_status(c);
    const bool hp = ql_get_hi_prec() != 0;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState* st = state_for(w->device);
    cudaError_t e = ensure(&st->ws, &st->ws_bytes, norm_ws_bytes(M, w->nblk));
    if (e != cudaSuccess) return cuda_status(e);
    const int rc = run_quantize_norm(dX, dNormW, eps, M, w->K, st->ws, nullptr, s, hp);
    if (rc != QL_OK) return rc;
    return run_compute(w, st->ws, M, dC, nullptr, s, hp, /*pdl=*/true);
}

// ------------------------------------------------------------------ fused SiLU * up prologue
//
// The reference decoder's MLP evaluates g1 = siluf(g1) * g2 into a scratch row
// and then i4_matmul(md, g1) (kernel/qwen35_decoder.cpp:408-409), which re-reads
// it to quantize it.  Here the quantizer reads the gate and up projections'
// outputs and quantizes silu(gate) * up directly, with the reference's
// arithmetic (ql_quant.cuh: the host library's expf method in double, then
// x / (1 + e) and * up in fp32), so the product never round-trips through
// memory unless the caller asks for it (dOut).
namespace {
int check_silu_args(const float* dG, const float* dU, int ld, int M, int K, const float* dOut) {
    if (M < 0 || K <= 0 || K % 32 || ld < K || ld % 4) return QL_EINVAL;
    if (M == 0) return QL_OK;
    if (!dG || !dU) return QL_EINVAL;
    if (reinterpret_cast<uintptr_t>(dG) % 16 || reinterpret_cast<uintptr_t>(dU) % 16 ||
        reinterpret_cast<uintptr_t>(dOut) % 16)
        return QL_EINVAL;        // 16-byte vector loads and stores
    return QL_OK;
}

int run_quantize_silu(const float* dG, const float* dU, int ld, int M, int K, void* ws, float* dOut,
                      cudaStream_t stream, bool hi_prec) {
    const int nblk = K / 32;
    if (use_gemm(M))
        return cuda_status(launch_quantize_gemm_silu(dG, dU, ld, M, K, hi_prec, static_cast<uint8_t*>(ws), dOut,
                                                     stream));
    for (int c = 0; c * MAX_DECODE_TOKENS < M; ++c) {
        const ActView act = chunk_view(ws, M, nblk, c, hi_prec);
        const size_t m0 = static_cast<size_t>(c) * MAX_DECODE_TOKENS;
        cudaError_t e = launch_quantize_act_silu(dG + m0 * ld, dU + m0 * ld, ld, act.M, K, hi_prec, act,
                                                 dOut ? dOut + m0 * K : nullptr, stream);
        if (e != cudaSuccess) return cuda_status(e);
    }
    return set_status(QL_OK);
}
}  // namespace

QL_API int ql_quantize_act_silu_mul_dev(const float* dGate, const float* dUp, int ld, int M, int K, int hi_prec,
                                        void* ws, size_t ws_bytes, float* dOut, void* stream) {
    const int c = check_silu_args(dGate, dUp, ld, M, K, dOut);
    if (c != QL_OK || M == 0) return set_status(c);
    if (!ws || reinterpret_cast<uintptr_t>(ws) % 16 || ws_bytes < ws_bytes_for(M, K / 32)) return set_status(QL_EINVAL);
    return run_quantize_silu(dGate, dUp, ld, M, K, ws, dOut, static_cast<cudaStream_t>(stream), hi_prec != 0);
}

QL_API int ql_matmul_silu_mul_dev(void* handle, const float* dGate, const float* dUp, int ld, int M, float* dC,
                                  void* stream) {
    int c = check_call(handle, dGate, M, dC);
    if (c != QL_OK || M == 0) return set_status(c);
    const auto* w = static_cast<const Weight*>(handle);
    c = check_silu_args(dGate, dUp, ld, M, w->K, nullptr);
    if (c != QL_OK) return set_status(c);
    const bool hp = ql_get_hi_prec() != 0;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState* st = state_for(w->device);
    cudaError_t e = ensure(&st->ws, &st->ws_bytes, ws_bytes_for(M, w->nblk));
    if (e != cudaSuccess) return cuda_status(e);
    const int rc = run_quantize_silu(dGate, dUp, ld, M, w->K, st->ws, nullptr, s, hp);
    if (rc != QL_OK) return rc;
    return run_compute(w, st->ws, M, dC, nullptr, s, hp, /*pdl=*/true);
}

// ------------------------------------------------------------------ concatenated weights
//
// Records are laid out row group by row group (rec[G][nblk][REC]), so stacking
// weights along N is a byte concatenation of their record arrays.  One handle
// over [gate; up] runs both projections that share an input in one launch
// (kernel/qwen35_decoder.cpp:406-407 makes two i4_matmul calls).
QL_API int ql_weight_concat(void* const* handles, int count, void** out_handle) {
    if (!out_handle) return set_status(QL_EINVAL);
    *out_handle = nullptr;
    if (!handles || count <= 0) return set_status(QL_EINVAL);
    if (!valid_weight(handles[0])) return set_status(QL_EINVAL);
    const auto* first = static_cast<const Weight*>(handles[0]);
    long long total_n = 0;
    for (int i = 0; i < count; ++i) {
        if (!valid_weight(handles[i])) return set_status(QL_EINVAL);
        const auto* h = static_cast<const Weight*>(handles[i]);
        if (h->K != first->K || h->bits != first->bits || h->scale_half != first->scale_half ||
            h->has_zp != first->has_zp || h->device != first->device)
            return set_status(QL_EINVAL);
        total_n += h->N;
    }
    if (total_n > (1LL << 30)) return set_status(QL_EINVAL);
    DeviceGuard guard(first->device);
    if (!guard.ok) return set_status(QL_ECUDA);
    Weight* w = allocate_weight(static_cast<int>(total_n), first->K, first->bits, first->scale_half,
                                first->has_zp);
    if (!w) return set_status(QL_ENOMEM);
    cudaStream_t s = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        s = internal_stream(state_for(first->device));
    }
    size_t off = 0;
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < count && e == cudaSuccess; ++i) {
        const auto* h = static_cast<const Weight*>(handles[i]);
        const size_t n = static_cast<size_t>(h->G) * h->nblk * h->REC;
        e = cudaMemcpyAsync(w->W + off, h->W, n, cudaMemcpyDeviceToDevice, s);
        off += n;
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        free_weight(w);
        return cuda_status(e);
    }
    *out_handle = w;
    return set_status(QL_OK);
}

// ------------------------------------------------------------------ no-allocation variant
//
// Some callers cannot allocate device memory at the time they run a layer:
// serving runtimes whose allocator owns all of HBM (weights and KV cache are
// reserved up front and nothing else may allocate), and per-token decode loops
// that cannot pay for an allocation or for the device-wide synchronisation
// that freeing one implies.  For them,
// ql_matmul_dev_noalloc keeps the quantized activations in a fixed scratch
// array compiled into this library instead of a workspace.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds these QL_NOALLOC_SCRATCH_BYTES until the process exits.  Host
// code cannot use the symbol as an address, so the first call on each device
// (with that device current) looks up its device address once with
// cudaGetSymbolAddress and caches it; make that first call before any stream
// capture.  All calls share the one array and it keeps the last call's
// contents; nothing needs to start at zero, because the quantizer writes every
// byte the matmul reads (padded token rows included).  Calls whose work
// overlaps on the GPU (different streams, or a second call before the first
// finished on another stream) race on the array: serialise them.
static __device__ __align__(256) uint8_t g_noalloc_scratch[QL_NOALLOC_SCRATCH_BYTES];

namespace {
void* g_noalloc_addr[MAX_DEVICES] = {};
}  // namespace

QL_API int ql_matmul_dev_noalloc(void* handle, const float* dA, int M, float* dC, void* stream) {
    const int c = check_call(handle, dA, M, dC);
    if (c != QL_OK || M == 0) return set_status(c);
    const auto* w = static_cast<const Weight*>(handle);
    if (ws_bytes_for(M, w->nblk) > QL_NOALLOC_SCRATCH_BYTES) return set_status(QL_ESCRATCH);
    const bool hp = ql_get_hi_prec() != 0;
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_noalloc_addr[w->device]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || !p) return cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
            g_noalloc_addr[w->device] = p;
        }
        scratch = g_noalloc_addr[w->device];
    }
    return run_matmul(w, dA, M, dC, nullptr, scratch, QL_NOALLOC_SCRATCH_BYTES,
                      static_cast<cudaStream_t>(stream), hp);
}

// Per-block INT32 accumulators cs[M][N][K/32] = sum_k q16 * (w - zp), produced
// by the decode kernel's own integer MMA path (parity checks of the INT32 stage).
QL_API int ql_block_sums_dev(void* handle, const float* dA, int M, int32_t* dCS, void* stream) {
    const int c = check_call(handle, dA, M, dCS);
    if (c != QL_OK || M == 0) return set_status(c);
    const auto* w = static_cast<const Weight*>(handle);
    const bool hp = ql_get_hi_prec() != 0;
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState* st = state_for(w->device);
    cudaError_t e = ensure(&st->ws, &st->ws_bytes, ws_bytes_for_w(w, M));
    if (e != cudaSuccess) return cuda_status(e);
    return run_matmul(w, dA, M, nullptr, dCS, st->ws, st->ws_bytes, static_cast<cudaStream_t>(stream), hp);
}

// The activation quantizer in the reference's layout: hi/lo u8 [M][K] and
// ascale fp32 [M][K/32] (quantize_A_i16, kernel/quantized_matmul.cpp:237-258).
QL_API int ql_quantize_dev(const float* dA, int M, int K, uint8_t* dHi, uint8_t* dLo,
                           float* dAscale, void* stream) {
    if (M < 0 || K <= 0 || K % 32) return set_status(QL_EINVAL);
    if (M == 0) return set_status(QL_OK);
    if (!dA || !dHi || !dLo || !dAscale) return set_status(QL_EINVAL);
    return cuda_status(launch_quantize_ref(dA, M, K, dHi, dLo, dAscale, static_cast<cudaStream_t>(stream)));
}

// i4_matmul (kernel/quantized_matmul.cpp:526-552): host A[M,K] fp32 in, host
// C[M,N] fp32 out, synchronous.  Like the reference it returns nothing; a
// failure leaves C untouched and is reported by ql_last_status().
// Output columns per chunk of the synchronous host-pointer call: outputs of at
// least 2 MB are split into one column chunk per MB, up to 8 (measured on B200,
// LM head 4096 x 151936 INT8 through i4_matmul: 2 MB at M = 4 -> 2 chunks 187 us,
// 4.9 MB at M = 8 -> 4 chunks 202 us against 213 with 8, 9.7 MB at M = 16 -> 8
// chunks 266 us against 360 with one), in multiples of 128 columns, so every chunk is whole GEMM tiles and decode row groups); each
// chunk's matmul runs on the call's stream and its device -> host copy starts
// on a second stream as soon as it is done, overlapping the next chunk.
// After a synchronous call: a bounded wait of one of its kernels gave up if the
// error word (copied to host_err behind the call's work) is set.  The call then
// reports that code (QL_ETIMEOUT) instead of QL_OK, and the word is cleared so
// the next call starts clean.
static int take_device_error(DeviceState* st, int* err_word, cudaStream_t s) {
    const int v = st->host_err ? *st->host_err : 0;
    if (!v) return set_status(QL_OK);
    if (err_word && cudaMemsetAsync(err_word, 0, sizeof(int), s) == cudaSuccess) cudaStreamSynchronize(s);
    return set_status(v);
}

static int output_chunks(int M, int N) {
    const size_t bytes = static_cast<size_t>(M) * N * 4;
    int chunks = static_cast<int>(std::min<size_t>(8, bytes / (1024 * 1024)));
    if (const char* v = std::getenv("BREEZE_QL_OUTPUT_CHUNKS")) {      // tuning override (0: planner)
        const int c = std::atoi(v);
        if (c > 0) chunks = std::min(c, 8);
    }
    while (chunks > 1 && N / chunks < 128) --chunks;
    return std::max(1, chunks);
}

// A decode-size call whose A is pinned host memory that this device can read
// (and 16-byte aligned) skips the host -> device copy: the quantizer reads A
// over the bus itself, once, which removes one copy operation from the call's
// critical path.  nullptr: copy A in as usual.
static const float* direct_host_view(const float* A) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, A) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (attr.type != cudaMemoryTypeHost || !attr.devicePointer) return nullptr;
    if (reinterpret_cast<uintptr_t>(attr.devicePointer) % 16) return nullptr;
    return static_cast<const float*>(attr.devicePointer);
}

// Enqueues one host-pointer call on s (and the copy stream, joined back into
// s): copy A in, quantize and multiply (in output column chunks whose copies
// overlap the next chunk), copy C and the device error word out.  Nothing
// here synchronises; the caller drains both streams.
static int enqueue_host_call(const Weight* w, const float* A, int M, float* C, DeviceState* st, cudaStream_t s,
                             bool hp, float* dA, float* dC, void* ws, size_t ws_bytes, int* err_word) {
    cudaError_t e = cudaSuccess;
    const float* direct = use_gemm(M) ? nullptr : direct_host_view(A);
    if (direct) {
        dA = const_cast<float*>(direct);           // read by the quantizer only
    } else {
        e = cudaMemcpyAsync(dA, A, static_cast<size_t>(M) * w->K * 4, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return cuda_status(e);
    }
    const int chunks = output_chunks(M, w->N);
    if (chunks == 1) {
        int rc = run_matmul(w, dA, M, dC, nullptr, ws, ws_bytes, s, hp);
        if (rc != QL_OK) return rc;
        e = cudaMemcpyAsync(C, dC, static_cast<size_t>(M) * w->N * 4, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess && err_word)
            e = cudaMemcpyAsync(st->host_err, err_word, sizeof(int), cudaMemcpyDeviceToHost, s);
        return cuda_status(e);
    }
    const bool fp16_ops = gemmw_applies(w, M);      // the workspace was sized for it
    uint8_t* wbase = static_cast<uint8_t*>(ws);
    int rc = fp16_ops ? run_gemmw_prep(w, dA, M, wbase, s, hp) : run_quantize(dA, M, w->K, ws, s, hp);
    if (rc != QL_OK) return rc;
    // column chunks of whole 128-column tiles; the last takes the remainder
    const int per = ((w->N / chunks) / 128) * 128;
    for (int i = 0; i < chunks && e == cudaSuccess; ++i) {
        const int n0 = i * per;
        const int nc = (i == chunks - 1) ? w->N - n0 : per;
        Weight view = *w;                         // rows n0 .. n0+nc of the same records
        view.N = nc;
        view.G = nc / 16;
        view.W = w->W + static_cast<size_t>(n0 / 16) * w->nblk * w->REC;
        if (fp16_ops) {
            const uint8_t* wd = wbase + gemmw_act_region(M, w->nblk) + static_cast<size_t>(n0 / 128) * w->nblk * WREC16;
            rc = cuda_status(launch_gemmw(&view, wd, wbase, M, hp, dC + n0, w->N, nullptr, s));
        } else {
            rc = run_compute(&view, ws, M, dC + n0, nullptr, s, hp, /*pdl=*/i == 0, /*ldc=*/w->N);
        }
        if (rc != QL_OK) break;
        e = cudaEventRecord(st->chunk_done[i], s);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st->copy_stream, st->chunk_done[i], 0);
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(C + n0, static_cast<size_t>(w->N) * 4, dC + n0, static_cast<size_t>(w->N) * 4,
                                  static_cast<size_t>(nc) * 4, M, cudaMemcpyDeviceToHost, st->copy_stream);
    }
    // the copy stream joins back into s (also after a failure, so a capture ends cleanly)
    cudaError_t ej = cudaEventRecord(st->copies_done, st->copy_stream);
    if (ej == cudaSuccess) ej = cudaStreamWaitEvent(s, st->copies_done, 0);
    if (rc != QL_OK) return rc;
    if (e == cudaSuccess) e = ej;
    if (e == cudaSuccess && err_word)
        e = cudaMemcpyAsync(st->host_err, err_word, sizeof(int), cudaMemcpyDeviceToHost, s);
    return cuda_status(e);
}

QL_API void i4_matmul(void* handle, const float* A, int M, float* C) {
    if (!valid_weight(handle) || M < 0 || (M > 0 && (!A || !C))) {
        set_status(QL_EINVAL);
        return;
    }
    if (M == 0) {
        set_status(QL_OK);
        return;
    }
    const auto* w = static_cast<const Weight*>(handle);
    const bool hp = ql_get_hi_prec() != 0;
    DeviceGuard guard(w->device);
    if (!guard.ok) {
        set_status(QL_ECUDA);
        return;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState* st = state_for(w->device);
    cudaStream_t s = internal_stream(st);
    const size_t a_bytes = align256(static_cast<size_t>(M) * w->K * 4);
    const size_t c_bytes = align256(static_cast<size_t>(M) * w->N * 4);
    const size_t ws_bytes = ws_bytes_for_w(w, M);
    cudaError_t e = ensure(&st->buf, &st->buf_bytes, a_bytes + c_bytes + ws_bytes);
    if (e != cudaSuccess) {
        cuda_status(e);
        return;
    }
    float* dA = static_cast<float*>(st->buf);
    float* dC = reinterpret_cast<float*>(static_cast<uint8_t*>(st->buf) + a_bytes);
    void* ws = static_cast<uint8_t*>(st->buf) + a_bytes + c_bytes;
    int* err_word = device_error_word();
    if (!st->host_err) {
        e = cudaHostAlloc(reinterpret_cast<void**>(&st->host_err), sizeof(int), cudaHostAllocDefault);
        if (e != cudaSuccess) {
            st->host_err = nullptr;
            cuda_status(e);
            return;
        }
    }
    if (!st->copy_stream) {
        e = cudaStreamCreateWithFlags(&st->copy_stream, cudaStreamNonBlocking);
        for (int i = 0; i < 8 && e == cudaSuccess; ++i)
            e = cudaEventCreateWithFlags(&st->chunk_done[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&st->copies_done, cudaEventDisableTiming);
        if (e != cudaSuccess) {
            cuda_status(e);
            return;
        }
    }
    *st->host_err = 0;

    const int rc = enqueue_host_call(w, A, M, C, st, s, hp, dA, dC, ws, ws_bytes, err_word);
    // both streams drain before returning (also after a failure, so no copy is in flight)
    const cudaError_t e1 = cudaStreamSynchronize(s);
    const cudaError_t e2 = cudaStreamSynchronize(st->copy_stream);
    if (rc != QL_OK) return;
    e = (e1 != cudaSuccess) ? e1 : e2;
    if (e == cudaSuccess) take_device_error(st, err_word, s);
    else cuda_status(e);
}

// i4_matmul_region (kernel/quantized_matmul.cpp:554-572): called by EVERY
// thread of the caller's OpenMP parallel region (the reference's Phi decoder
// keeps one region open for its whole forward, kernel/phi35_decoder.cpp:179-211).
// One thread makes the synchronous i4_matmul call and the single construct's
// barrier holds the others until the output is complete, as the reference's
// closing barrier does.  au8/ascale are the caller's CPU quantization scratch
// in the reference; the GPU path quantizes into device memory and leaves them
// untouched.  Called outside a parallel region it is i4_matmul.  Unlike the
// reference there is no M <= 8 limit.  The status is that of the thread that
// ran the call.
QL_API void i4_matmul_region(void* handle, const float* A, int M, float* C, uint8_t* au8, float* ascale) {
    (void)au8;
    (void)ascale;
#pragma omp single
    i4_matmul(handle, A, M, C);
}

// The FP16-operand prefill GEMM alone, on a workspace a previous
// ql_matmul_dev_ws call with the same handle, M and activation mode has just
// filled (it still holds that call's dequantized weights and FP16 activations):
// the kernel-only timing of a prefill call, without its dequantize and quantize
// passes.  QL_ENOTSUP where the call would not take that path.
QL_API int ql_prefill_gemm_dev(void* handle, const void* ws, size_t ws_bytes, int M, int hi_prec, float* dC,
                               void* stream) {
    if (!valid_weight(handle) || M <= 0 || !ws || !dC || reinterpret_cast<uintptr_t>(ws) % 16)
        return set_status(QL_EINVAL);
    const auto* w = static_cast<const Weight*>(handle);
    if (!gemmw_applies(w, M)) return set_status(QL_ENOTSUP);
    if (ws_bytes < gemmw_ws_bytes(w, M)) return set_status(QL_EINVAL);
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return set_status(QL_ECUDA);
    if (dev != w->device) return set_status(QL_EDEVICE);
    const uint8_t* base = static_cast<const uint8_t*>(ws);
    return cuda_status(launch_gemmw(w, base + gemmw_act_region(M, w->nblk), base, M, hi_prec != 0, dC, w->N,
                                    nullptr, static_cast<cudaStream_t>(stream)));
}
