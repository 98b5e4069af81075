/*
 * breeze_ql.h -- C ABI of libbreeze_ql.so, the sm_100a (B200) quantized-linear
 * library that replaces Breeze's AVX-512 VNNI kernel (kernel/quantized_matmul.cpp).
 *
 * Two groups of entry points:
 *
 *  1. Reference-compatible (host pointers, synchronous), same names, argument
 *     meaning and failure behaviour as kernel/quantized_matmul.cpp:472-574, so
 *     the unchanged ctypes bridge (breeze/cpu_backend.py:14-54) or the native
 *     decoders that link i4_matmul (kernel/qwen35_decoder.cpp:124) can bind them.
 *     Handles own device memory on the device current at prepack time.
 *
 *  2. Device-pointer entry points (ql_*): inputs/outputs in device memory,
 *     cudaStream_t passed as void*, asynchronous, int status (0 = QL_OK).
 *     The handle's device must be the current device.
 *
 * Numerics (both groups, two-pass mode): activations are quantized per 32-wide
 * K block to INT16 exactly as quantize_A_i16 (kernel/quantized_matmul.cpp:237-258);
 * per-block INT32 accumulators sum_k q16*(w-zp) are exact; the FP32 rescale
 * acc = fma(ascale, (float)cs * bscale, acc) runs in ascending block order, so
 * outputs are bit-identical to i4_matmul on the same inputs.
 */
#ifndef BREEZE_QL_H
#define BREEZE_QL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes of the ql_* entry points. */
enum {
    QL_OK = 0,
    QL_EINVAL = 1,    /* bad argument or contract violation            */
    QL_ENOMEM = 2,    /* device allocation failed                      */
    QL_ECUDA = 3,     /* CUDA runtime error (see ql_last_cuda_error_string) */
    QL_ETIMEOUT = 4,  /* a bounded device wait gave up                 */
    QL_EDEVICE = 5,   /* handle belongs to another device              */
    QL_ENOTSUP = 6,   /* unsupported configuration                     */
    QL_ESCRATCH = 7   /* request exceeds the fixed scratch of ql_matmul_dev_noalloc */
};

/* Bytes of the fixed device scratch behind ql_matmul_dev_noalloc. */
#define QL_NOALLOC_SCRATCH_BYTES (8u << 20)

/* ---------------------------------------------------------------- group 1 */

/* Replaces i4_set_threads (kernel/quantized_matmul.cpp:474).  Accepted and
 * ignored: GPU results do not depend on a thread count. */
void i4_set_threads(int n);

/* Replaces i4_set_numa_split (kernel/quantized_matmul.cpp:475).  Accepted and
 * ignored: there is no NUMA weight replica on the GPU. */
void i4_set_numa_split(int cpu);

/* Replaces i4_set_hi_prec (kernel/quantized_matmul.cpp:476).  Process-global:
 * 1 = two-pass INT16 activations, 0 = single-pass INT8 (the default, as in the
 * reference).  Serialise with running calls. */
void i4_set_hi_prec(int on);

/* Replaces i4_prepack_onnx (kernel/quantized_matmul.cpp:505-520).  qw: uint8
 * MatMulNBits weights [N][K/32][16] (bits 4) or [N][K/32][32] (bits 8);
 * scales: [N][K/32] fp16 (scale_bits 16) or fp32 (32); qzeros: packed INT4
 * zero points [N][ceil(K/64)] or NULL (zp 8; must be NULL for bits 8).
 * Returns an owning handle on the current device, or NULL on a bad contract
 * (N,K <= 0, N%16, K%32, bits not 4/8, scale_bits not 16/32, INT8 with
 * qzeros) or allocation failure.  Inputs may be freed after the call. */
void* i4_prepack_onnx(const uint8_t* qw, const void* scales, const uint8_t* qzeros, int N, int K,
                      int bits, int scale_bits);

/* Replaces i4_prepack (kernel/quantized_matmul.cpp:480-499), the legacy entry
 * taking the reference's VNNI layout: srcB [N/16][nblk][8][32 or 64],
 * srcScale fp32 [N/16][nblk][16], srcZp int8 [N/16][nblk][16] (INT4, values
 * 0..15), srcCorr int32 [N/16][nblk][16] (required, not used).  NULL on a bad
 * contract or allocation failure. */
void* i4_prepack(const uint8_t* srcB, const float* srcScale, const int8_t* srcZp,
                 const int32_t* srcCorr, int N, int K, int nblk, int bits);

/* Replaces i4_free (kernel/quantized_matmul.cpp:522-524).  NULL-safe. */
void i4_free(void* handle);

/* Replaces i4_matmul (kernel/quantized_matmul.cpp:526-552): C[M,N] =
 * A[M,K] @ dequant(W).T with host fp32 row-major A and C, synchronous.  Like
 * the reference it returns nothing; a failure leaves C untouched and sets
 * ql_last_status(), which also reports QL_ETIMEOUT when a bounded device wait
 * of the call gave up.  Page-locked (pinned) host buffers are fastest: at
 * decode sizes (M <= 64) a pinned, 16-byte aligned A is read by the quantizer
 * directly instead of being copied in, and outputs of 2 MB or more are copied
 * back in column chunks that overlap the matmul; pageable buffers work too. */
void i4_matmul(void* handle, const float* A, int M, float* C);

/* Replaces i4_matmul_region (kernel/quantized_matmul.cpp:554-572): the same
 * product, called by every thread of the caller's OpenMP parallel region (the
 * Phi decoder's persistent region, kernel/phi35_decoder.cpp:179-211).  One
 * thread issues the synchronous GPU call; the others wait at the barrier that
 * ends it, so C is complete in every thread on return.  au8 (2*M*K bytes) and
 * ascale (M*K/32 floats) are the reference's CPU quantization scratch: accepted
 * and left untouched.  Outside a parallel region it behaves as i4_matmul. */
void i4_matmul_region(void* handle, const float* A, int M, float* C, uint8_t* au8, float* ascale);

/* ---------------------------------------------------------------- group 2 */

/* Library ABI version (no counterpart in the reference). */
int ql_version(void);

/* Number of visible CUDA devices (0 when none or the driver is absent);
 * backs available() of the Python bridge (breeze/cpu_backend.py:57). */
int ql_device_count(void);

/* Current activation mode (the value last given to i4_set_hi_prec). */
int ql_get_hi_prec(void);

/* Prefill kernel selector (no counterpart in the reference, whose i4_matmul
 * has one CPU path): 0 = automatic -- M > 64 tokens with INT4 weights and
 * fp16 scales run the FP16-operand tcgen05 GEMM (the weights dequantized once
 * per call into the workspace, ql_workspace_bytes) when the call has that
 * workspace, else the kind::f16 GEMM that unpacks them per tile (two-pass);
 * every other prefill the kind::i8 GEMM; 1 = always the kind::i8 GEMM; 2 =
 * the per-tile-unpack kind::f16 GEMM on CTA pairs (cta_group::2) where it
 * applies; 3 = that GEMM on single CTAs.  All kernels give the reference's
 * bits; the switch exists for comparison and testing.  Process-global;
 * returns QL_EINVAL for any other value. */
int ql_set_prefill_kernel(int kind);

/* Status of this thread's last call, and its description. */
int ql_last_status(void);
const char* ql_error_string(int code);
const char* ql_last_cuda_error_string(void);

/* Synchronises the current device and returns its device error word (set by
 * a kernel whose bounded wait gave up; 0 = none).  clear != 0 resets it.
 * The synchronous i4_matmul reads and clears the word after every call and
 * reports a set word through ql_last_status() (QL_ETIMEOUT); callers of the
 * asynchronous ql_* entry points check it with this function after they
 * synchronise. */
int ql_device_error(int clear);

/* Limits of the bounded device waits on the current device (no counterpart in
 * the reference, whose CPU code has no device waits): wait_ns for waits inside
 * one kernel (default 1 s), peer_wait_ns for waits on another GPU's flags in
 * the peer exchange (default 5 s).  0 keeps a limit unchanged.  A wait that
 * runs out sets QL_ETIMEOUT in the device error word and its kernel returns.
 * Serialise with running calls. */
#define QL_DEFAULT_WAIT_NS 1000000000ull
#define QL_DEFAULT_PEER_WAIT_NS 5000000000ull
int ql_set_wait_limits(unsigned long long wait_ns, unsigned long long peer_wait_ns);

/* Device-pointer twin of i4_prepack_onnx: the same contract with the
 * MatMulNBits arrays already in device memory, enqueued on `stream`. */
int ql_prepack_onnx_dev(const uint8_t* d_qw, const void* d_scales, const uint8_t* d_qzeros, int N,
                        int K, int bits, int scale_bits, void* stream, void** out_handle);

/* Handle metadata (any pointer may be NULL). */
int ql_weight_info(const void* handle, int* N, int* K, int* bits, int* device,
                   unsigned long long* bytes);

/* Scratch bytes ql_matmul_dev_ws needs for M rows (quantized activations;
 * M > 64 uses the tensor-core GEMM's record layout, so the size is not linear
 * in M across that boundary; for INT4 weights with fp16 scales it also holds
 * the call's FP16-dequantized weights, 2.125 bytes per weight -- a smaller
 * workspace of at least the activation records runs the per-tile-unpack GEMM). */
size_t ql_workspace_bytes(const void* handle, int M);

/* Device twin of i4_matmul (kernel/quantized_matmul.cpp:528): dA [M,K] fp32
 * (16-byte aligned), dC [M,N] fp32, asynchronous on `stream`, with the
 * caller's workspace (16-byte aligned) of at least ql_workspace_bytes(handle, M)
 * bytes.  Up to 64 rows run the weight-streaming decode kernel; more rows run
 * the tcgen05 GEMM.  Both give the reference's bits. */
int ql_matmul_dev_ws(void* handle, const float* dA, int M, float* dC, void* ws, size_t ws_bytes,
                     void* stream);

/* Same with the library's per-device workspace (allocated on first use). */
int ql_matmul_dev(void* handle, const float* dA, int M, float* dC, void* stream);

/* Split form of ql_matmul_dev_ws (no counterpart in the reference, whose
 * i4_matmul re-quantizes per call, kernel/quantized_matmul.cpp:532-536):
 * quantize dA [M,K] once into `ws` (>= ql_act_workspace_bytes(M, K) bytes),
 * then run any number of weights with the same K over it.  hi_prec selects
 * the activation mode explicitly and must match between the two calls. */
size_t ql_act_workspace_bytes(int M, int K);
int ql_quantize_act_dev(const float* dA, int M, int K, int hi_prec, void* ws, size_t ws_bytes,
                        void* stream);
int ql_matmul_quantized_dev(void* handle, const void* ws, int M, int hi_prec, float* dC,
                            void* stream);

/* Fused RMSNorm prologue (no counterpart in the reference's C ABI; it
 * replaces the reference decoder's rmsnorm-then-i4_matmul pair,
 * kernel/qwen35_decoder.cpp:133-141 followed by :329/:395/:406-407/:421):
 * the activations quantized are hn = rmsnorm(dX, dNormW, eps) row by row,
 *   inv = 1.0f / sqrtf((float)(sum_j (double)x_j^2 / K) + eps),  hn_j = x_j * inv * w_j,
 * bit-identical to the reference's serial double sum and fp32 products, so
 * the result equals i4_matmul(handle, hn, M, C) on the reference's own hn.
 * ql_quantize_act_rmsnorm_dev: the split form of ql_quantize_act_dev (then
 * ql_matmul_quantized_dev, once per weight sharing the normalised input);
 * its workspace is >= ql_norm_act_workspace_bytes(M, K) bytes (the quantized
 * activations plus M row factors); dHn (16-byte aligned, may be NULL)
 * receives hn [M,K].  ql_matmul_rmsnorm_dev: one call with the library's
 * workspace and the process-wide activation mode (i4_set_hi_prec).  dX and
 * dNormW are 16-byte aligned device pointers, K % 32 == 0. */
size_t ql_norm_act_workspace_bytes(int M, int K);
int ql_quantize_act_rmsnorm_dev(const float* dX, const float* dNormW, float eps, int M, int K,
                                int hi_prec, void* ws, size_t ws_bytes, float* dHn, void* stream);
int ql_matmul_rmsnorm_dev(void* handle, const float* dX, const float* dNormW, float eps, int M,
                          float* dC, void* stream);

/* Fused SiLU * up prologue (no counterpart in the reference's C ABI; it
 * replaces the reference decoder's g1 = siluf(g1) * g2 loop before its down
 * projection, kernel/qwen35_decoder.cpp:408-409, siluf at :129): the values
 * quantized are silu(gate) * up element by element,
 *   x / (1.0f + expf(-x)) * u,
 * with the host C library's expf reproduced bit for bit (the same method and
 * roundings in double precision, checked against the library over all 2^32
 * inputs), so the result equals i4_matmul(handle, g1, M, C) on the reference's
 * own g1.  dGate and dUp are [M, K] with rows `ld` floats apart (ld >= K,
 * ld % 4 == 0; e.g. the halves of a concatenated gate|up output, ld = 2K,
 * dUp = dGate + K), 16-byte aligned, K % 32 == 0.
 * ql_quantize_act_silu_mul_dev: the split form of ql_quantize_act_dev (then
 * ql_matmul_quantized_dev) with a workspace of >= ql_act_workspace_bytes(M, K)
 * bytes; dOut (16-byte aligned, may be NULL) receives the products [M, K].
 * ql_matmul_silu_mul_dev: one call with the library's workspace and the
 * process-wide activation mode (i4_set_hi_prec). */
int ql_quantize_act_silu_mul_dev(const float* dGate, const float* dUp, int ld, int M, int K, int hi_prec,
                                 void* ws, size_t ws_bytes, float* dOut, void* stream);
int ql_matmul_silu_mul_dev(void* handle, const float* dGate, const float* dUp, int ld, int M, float* dC,
                           void* stream);

/* One handle stacking `count` weights along N (no counterpart in the
 * reference, which calls i4_matmul once per projection that shares an input,
 * e.g. gate and up at kernel/qwen35_decoder.cpp:406-407).  All handles need
 * the same K, bits, scale type, zero-point presence and device (QL_EINVAL
 * otherwise); output columns follow the handles' order.  Results are those
 * of the separate weights, bit for bit.  The sources stay valid; finish any
 * ql_prepack_onnx_dev writing them before the call.  Free with i4_free. */
int ql_weight_concat(void* const* handles, int count, void** out_handle);

/* One-shot all-gather of column-parallel outputs over peer memory (no
 * counterpart in the reference, which runs on one CPU; the multi-GPU step that
 * replaces an NCCL all-gather of the [M, N/P] output slices at decode sizes,
 * where the collective is latency-bound).  One process per GPU:
 *   ql_peer_exchange_create   allocates this GPU's region (output capacity
 *                             `bytes`, plus flags) and writes its CUDA IPC
 *                             handle (QL_IPC_HANDLE_BYTES bytes);
 *   ql_peer_exchange_connect  maps every peer's region, given all GPUs'
 *                             handles in rank order (world <= 8);
 *                             The usable capacity is the smallest of all
 *                             GPUs' `bytes`;
 *   ql_peer_allgather_cols_dev  every GPU stores its slice dShard [M, Nl]
 *                             (Nl % 4 == 0, 16-byte aligned) into every GPU's
 *                             output [M, Nl * world] over NVLink, then the
 *                             GPUs hand-shake through the flags (each wait
 *                             bounded by the peer wait limit, 5 s unless set
 *                             by ql_set_wait_limits; on expiry QL_ETIMEOUT in
 *                             the device error word, which the caller checks
 *                             with ql_device_error after synchronising).  All
 *                             GPUs make the same sequence of calls.  The
 *                             result, at ql_peer_exchange_output(), is
 *                             complete for work enqueued after the call on the
 *                             same stream and valid until this GPU's next
 *                             call.  The kernels' arguments do not change
 *                             between calls, so the call can be captured in a
 *                             CUDA graph. */
#define QL_IPC_HANDLE_BYTES 64
int ql_peer_exchange_create(size_t bytes, void* ipc_handle, void** exchange);
int ql_peer_exchange_connect(void* exchange, int rank, int world, const void* handles);
float* ql_peer_exchange_output(void* exchange);
int ql_peer_allgather_cols_dev(void* exchange, const float* dShard, int M, int Nl, void* stream);
int ql_peer_exchange_destroy(void* exchange);

/* ql_matmul_dev without any device allocation (no counterpart in the
 * reference, which allocates its activation scratch on every call,
 * kernel/quantized_matmul.cpp:532-534).  For callers that cannot allocate
 * device memory when they run a layer: serving runtimes whose allocator owns
 * all of HBM (weights and KV cache are reserved up front and nothing else may
 * call cudaMalloc), and per-token loops that cannot pay for an allocation or
 * the device-wide synchronisation a free implies.  The quantized activations live in a fixed
 * QL_NOALLOC_SCRATCH_BYTES array compiled into the library, held by every GPU
 * that loads it until exit; requests that need more (ql_workspace_bytes(handle,
 * M) larger than that) return QL_ESCRATCH.  The first call on a device looks up
 * the array's device address (make it before any stream capture).  All calls
 * share the array: calls whose work overlaps on the GPU race, so serialise them.
 * Same numerics and arguments as ql_matmul_dev. */
int ql_matmul_dev_noalloc(void* handle, const float* dA, int M, float* dC, void* stream);

/* The FP16-operand prefill GEMM alone (no counterpart in the reference): re-runs
 * the tensor-core GEMM of the last ql_matmul_dev_ws call made with the same
 * handle, M (> 64), activation mode and workspace, on the dequantized weights
 * and FP16 activations that call left in the workspace -- the kernel-only
 * timing of a prefill call.  QL_ENOTSUP where that call does not take the
 * FP16-operand path (not INT4 with fp16 scales, or a selector other than 0). */
int ql_prefill_gemm_dev(void* handle, const void* ws, size_t ws_bytes, int M, int hi_prec, float* dC,
                        void* stream);

/* Packed-layout cache (no counterpart in the reference, which repacks every
 * MatMulNBits weight on each load, breeze/qwen35_cpu.py:71-89 ->
 * kernel/quantized_matmul.cpp:505-520; the survey's next step for 27B loads).
 * ql_weight_serialized_bytes: size of the serialised form of a handle (0 for
 * an invalid handle).  ql_weight_serialize: writes a versioned header and the
 * handle's device records into host_buf (>= that many bytes).
 * ql_weight_deserialize: checks the header, sizes and payload checksum
 * (QL_EINVAL on any mismatch, before touching device memory) and creates a new
 * handle on the current device with one host -> device copy. */
size_t ql_weight_serialized_bytes(const void* handle);
int ql_weight_serialize(const void* handle, void* host_buf, size_t bytes);
int ql_weight_deserialize(const void* host_buf, size_t bytes, void** out_handle);

/* The per-block INT32 accumulators cs[M][N][K/32] = sum_k q16*(w-zp) of the
 * reference's tile_kernel (kernel/quantized_matmul.cpp:298-312, 262-268),
 * produced by this library's own integer MMA path (INT32 parity checks). */
int ql_block_sums_dev(void* handle, const float* dA, int M, int32_t* dCS, void* stream);

/* The activation quantizer in the reference's layout: dHi/dLo u8 [M][K] and
 * dAscale fp32 [M][K/32] (quantize_A_i16, kernel/quantized_matmul.cpp:237-258). */
int ql_quantize_dev(const float* dA, int M, int K, uint8_t* dHi, uint8_t* dLo, float* dAscale,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BREEZE_QL_H */
