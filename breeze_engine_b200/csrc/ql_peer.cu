// ql_peer.cu -- one-shot all-gather of column-parallel outputs over peer memory.
//
// A column-parallel layer leaves each of P GPUs with its own [M, N/P] slice of
// the output; every GPU needs the full [M, N].  At decode sizes (M <= 16, a
// few hundred KB to a few MB) an NCCL all-gather is latency-bound.  Here each
// GPU stores its slice straight into every peer's output buffer over NVLink
// (plain stores through CUDA IPC mappings: no bulk/TMA copy and no multicast
// touches another GPU's memory), then the GPUs hand-shake through flags.
//
// Region of one GPU (one cudaMalloc, exported as one IPC handle):
//   [0, 256)            flags: word q = the last epoch GPU q posted here
//   [256, 256 + bytes)  the full [M, N] fp32 output, written by all GPUs
// One kernel per call, with e = 2 * calls + 1 (a device counter, so CUDA-graph
// replays use the right value without changing kernel arguments): every CTA
// posts e ("ready": this GPU's readers of the previous result ran before this
// launch, in stream order) to every peer, waits until every peer posted >= e,
// and stores its share of the slice into every peer's buffer; the last CTA to
// finish fences at system scope, posts e + 1 ("done"), waits until every peer
// posted >= e + 1 and advances the counter, so the result is complete when the
// kernel ends.
// Every wait is bounded (the device's peer wait limit, 5 s by default): on
// expiry the device error word gets QL_ETIMEOUT and the kernel returns, so a
// missing peer cannot hang a GPU.  Callers check the word after their gathers
// (ql_device_error, or the Python wrapper's check()).
#include <algorithm>
#include <cstring>

#include "ql_common.cuh"
#include "ql_internal.h"

#if defined(__GNUC__)
#define QL_API extern "C" __attribute__((visibility("default")))
#else
#define QL_API extern "C"
#endif

namespace ql {

int* device_error_word();   // ql_api.cu

namespace {

constexpr int MAX_PEERS = 8;
constexpr size_t FLAG_BYTES = 256;
constexpr size_t CAP_OFFSET = 128;      // inside the flag header: the region's output capacity (u64)
constexpr int PUT_THREADS = 256;
constexpr uint32_t EXCHANGE_MAGIC = 0x51504558u;   // "QPEX"
// Peers run on other GPUs driven by other processes, whose launches can lag
// this one's by more than a kernel-internal wait: the flag waits use the
// device's peer limit (5 s unless set by ql_set_wait_limits).
// The public header states the handle size as QL_IPC_HANDLE_BYTES = 64.
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");

struct Exchange {
    uint32_t magic;
    int device, rank, world;
    size_t bytes;                       // output capacity
    uint8_t* region;                    // this GPU's region
    uint8_t* peer[MAX_PEERS];           // every GPU's region, mapped here (peer[rank] = region)
    unsigned int* counter;              // calls made (device)
    unsigned int* blocks_done;          // CTAs of the current put kernel that finished (device)
};

struct PeerArgs {
    uint8_t* peer[MAX_PEERS];
    int P, rank;
    unsigned int* counter;
    unsigned int* blocks_done;
    int* err;
};

__device__ __forceinline__ void post_flag(uint8_t* region, int rank, unsigned int e) {
    unsigned int* f = reinterpret_cast<unsigned int*>(region) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(f), "r"(e) : "memory");
}

__device__ __forceinline__ unsigned int read_flag(const uint8_t* region, int q) {
    unsigned int v;
    const unsigned int* f = reinterpret_cast<const unsigned int*>(region) + q;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    return v;
}

// Lanes q < P wait until GPU q posted >= e in this GPU's flags; bounded.
__device__ bool wait_flags(const uint8_t* region, int P, unsigned int e, int* err) {
    const int q = threadIdx.x & 31;
    bool ok = true;
    if (q < P) {
        const uint64_t t0 = global_ns();
        uint64_t limit = WAIT_CHECK_NS;                // the device limit is read once this much has passed
        bool read = false;
        while (static_cast<int>(read_flag(region, q) - e) < 0) {
            if (global_ns() - t0 > limit) {
                if (!read) {
                    limit = peer_wait_limit(err);
                    read = true;
                    continue;
                }
                record_error(err, QL_ETIMEOUT);
                ok = false;
                break;
            }
        }
    }
    return __all_sync(0xffffffffu, ok);
}

__global__ void __launch_bounds__(PUT_THREADS) peer_put_kernel(const float* __restrict__ src, int M, int Nl,
                                                               PeerArgs a) {
    pdl_wait();                                      // the slice comes from the previous grid
    const unsigned int e = 2u * *a.counter + 1u;
    __shared__ int ok;
    if (threadIdx.x < 32) {
        if (threadIdx.x < a.P) post_flag(a.peer[threadIdx.x], a.rank, e);    // ready (idempotent per CTA)
        const bool w = wait_flags(a.peer[a.rank], a.P, e, a.err);
        if (threadIdx.x == 0) ok = w;
    }
    __syncthreads();
    if (ok) {
        const int nq = Nl / 4;                       // float4 per row of the slice
        const size_t ldc = static_cast<size_t>(Nl) * a.P;
        const long long total = static_cast<long long>(M) * nq;
        for (long long i = blockIdx.x * static_cast<long long>(PUT_THREADS) + threadIdx.x; i < total;
             i += static_cast<long long>(gridDim.x) * PUT_THREADS) {
            const int m = static_cast<int>(i / nq), j = static_cast<int>(i % nq);
            const float4 v = __ldg(reinterpret_cast<const float4*>(src + static_cast<size_t>(m) * Nl) + j);
            const size_t off = static_cast<size_t>(m) * ldc + static_cast<size_t>(a.rank) * Nl + 4 * j;
            for (int p = 0; p < a.P; ++p)
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.peer[p] + FLAG_BYTES) + off) = v;
        }
    }
    // The CTA's stores are ordered before its thread 0 by the barrier; thread 0
    // fences at system scope and counts the CTA done.  The last CTA posts
    // "done" to every peer, its first warp waits for every peer's "done" and
    // advances the call counter (every other CTA has read it by then).
    __syncthreads();
    if (threadIdx.x < 32) {
        unsigned int last = 0;
        if (threadIdx.x == 0) {
            __threadfence_system();
            last = atomicAdd(a.blocks_done, 1u) == gridDim.x - 1 ? 1u : 0u;
            if (last) {
                *a.blocks_done = 0u;
                __threadfence_system();
                for (int p = 0; p < a.P; ++p) post_flag(a.peer[p], a.rank, e + 1u);
            }
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            wait_flags(a.peer[a.rank], a.P, e + 1u, a.err);
            if (threadIdx.x == 0) *a.counter = (e + 1u) / 2u;
        }
    }
}

int status_of(cudaError_t e) {
    if (e == cudaSuccess) return QL_OK;
    if (e == cudaErrorMemoryAllocation) return QL_ENOMEM;
    return QL_ECUDA;
}

bool valid_exchange(const void* x) {
    return x && static_cast<const Exchange*>(x)->magic == EXCHANGE_MAGIC;
}

}  // namespace
}  // namespace ql

using namespace ql;

// Region of `bytes` output capacity (plus the flags) on the current device;
// writes the IPC handle (QL_IPC_HANDLE_BYTES bytes) that peers open.
QL_API int ql_peer_exchange_create(size_t bytes, void* ipc_handle, void** out) {
    if (!out) return QL_EINVAL;
    *out = nullptr;
    if (!ipc_handle || bytes == 0 || bytes % 16) return QL_EINVAL;
    auto* x = new (std::nothrow) Exchange{};
    if (!x) return QL_ENOMEM;
    cudaError_t e = cudaGetDevice(&x->device);
    void* region = nullptr;
    void* ctr = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&region, FLAG_BYTES + bytes);
    if (e == cudaSuccess) e = cudaMemset(region, 0, FLAG_BYTES + bytes);
    // the capacity, for peers to read at connect time (flags use bytes 0..31)
    const unsigned long long cap = bytes;
    if (e == cudaSuccess) e = cudaMemcpy(static_cast<uint8_t*>(region) + CAP_OFFSET, &cap, sizeof(cap),
                                         cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&ctr, 2 * sizeof(unsigned int));
    if (e == cudaSuccess) e = cudaMemset(ctr, 0, 2 * sizeof(unsigned int));
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, region);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (region) cudaFree(region);
        if (ctr) cudaFree(ctr);
        delete x;
        return status_of(e);
    }
    std::memcpy(ipc_handle, &h, sizeof(h));
    x->magic = EXCHANGE_MAGIC;
    x->bytes = bytes;
    x->region = static_cast<uint8_t*>(region);
    x->counter = static_cast<unsigned int*>(ctr);
    x->blocks_done = x->counter + 1;
    x->rank = -1;
    *out = x;
    return QL_OK;
}

// Maps every peer's region: `handles` holds world handles of
// QL_IPC_HANDLE_BYTES bytes in rank order (this rank's own entry is ignored).
QL_API int ql_peer_exchange_connect(void* exchange, int rank, int world, const void* handles) {
    if (!valid_exchange(exchange) || !handles || world < 1 || world > MAX_PEERS || rank < 0 || rank >= world)
        return QL_EINVAL;
    auto* x = static_cast<Exchange*>(exchange);
    if (x->rank >= 0) return QL_EINVAL;              // connected already
    for (int q = 0; q < world; ++q) {
        if (q == rank) {
            x->peer[q] = x->region;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(q) * sizeof(h), sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int r = 0; r < q; ++r)
                if (r != rank && x->peer[r]) cudaIpcCloseMemHandle(x->peer[r]);
            return status_of(e);
        }
        x->peer[q] = static_cast<uint8_t*>(p);
    }
    // Every GPU stores into every region: the usable capacity is the smallest.
    size_t cap_min = x->bytes;
    for (int q = 0; q < world; ++q) {
        if (q == rank) continue;
        unsigned long long cap = 0;
        const cudaError_t e = cudaMemcpy(&cap, x->peer[q] + CAP_OFFSET, sizeof(cap), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) {
            for (int r = 0; r < world; ++r)
                if (r != rank && x->peer[r]) cudaIpcCloseMemHandle(x->peer[r]);
            return status_of(e);
        }
        cap_min = std::min<size_t>(cap_min, cap);
    }
    x->bytes = cap_min;
    x->rank = rank;
    x->world = world;
    return QL_OK;
}

// This GPU's full-output buffer ([M, Nl * world] fp32 after a gather).
QL_API float* ql_peer_exchange_output(void* exchange) {
    if (!valid_exchange(exchange)) return nullptr;
    return reinterpret_cast<float*>(static_cast<Exchange*>(exchange)->region + FLAG_BYTES);
}

// Gathers the slices dShard [M, Nl] (row-major, 16-byte aligned, Nl % 4 == 0)
// of all GPUs into every GPU's output buffer, enqueued on `stream`.  Every GPU
// of the exchange makes the same sequence of calls.  The result is complete
// for kernels enqueued after this call on the same stream and stays valid until
// this GPU's next call.
QL_API int ql_peer_allgather_cols_dev(void* exchange, const float* dShard, int M, int Nl, void* stream) {
    if (!valid_exchange(exchange)) return QL_EINVAL;
    auto* x = static_cast<Exchange*>(exchange);
    if (x->rank < 0 || M < 0 || Nl <= 0 || Nl % 4 || !dShard || reinterpret_cast<uintptr_t>(dShard) % 16)
        return QL_EINVAL;
    if (static_cast<size_t>(M) * Nl * x->world * sizeof(float) > x->bytes) return QL_EINVAL;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return QL_ECUDA;
    if (dev != x->device) return QL_EDEVICE;
    PeerArgs a = {};
    for (int q = 0; q < x->world; ++q) a.peer[q] = x->peer[q];
    a.P = x->world;
    a.rank = x->rank;
    a.counter = x->counter;
    a.blocks_done = x->blocks_done;
    a.err = device_error_word();
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const long long work = static_cast<long long>(M) * (Nl / 4);
    const unsigned grid = static_cast<unsigned>(std::max(1LL, std::min(148LL, (work + PUT_THREADS - 1) / PUT_THREADS)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(PUT_THREADS);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return status_of(cudaLaunchKernelEx(&cfg, peer_put_kernel, dShard, M, Nl, a));
}

QL_API int ql_peer_exchange_destroy(void* exchange) {
    if (!valid_exchange(exchange)) return QL_EINVAL;
    auto* x = static_cast<Exchange*>(exchange);
    x->magic = 0;
    cudaDeviceSynchronize();
    if (x->rank >= 0)
        for (int q = 0; q < x->world; ++q)
            if (q != x->rank && x->peer[q]) cudaIpcCloseMemHandle(x->peer[q]);
    cudaFree(x->region);
    cudaFree(x->counter);
    delete x;
    return QL_OK;
}
