// ql_common.cuh -- shared device helpers for the sm_100a quantized-linear kernels.
//
// Numerics contract (reference kernel/quantized_matmul.cpp):
//   q16 = clamp(lrint(a * inv), +-32767) per 32-wide K block (quantize_A_i16 :237-258)
//   cs  = sum_k q16 * (w - zp)        (INT32, exact; :298-312, :262-268)
//   f   = (float)cs * bscale          (one rounding)
//   acc = fma(ascale, f, acc)         (one rounding, blocks in ascending order; :311-315)
//
// The kernels split q16 = 256*(hi - 128) + lo into a signed plane hs = hi - 128
// and an unsigned plane lo and accumulate S_hi = sum hs*(w-zp), S_lo = sum lo*(w-zp)
// with integer MMAs.  Both accumulators are seeded with "magic" integers so that
// their bit patterns read as floats are exact:
//   float(HI_SEED + S_hi) = 1.5*2^31 + 256*S_hi   (|S_hi| <= 2^19 < 2^22)
//   float(LO_SEED + S_lo) = 1.5*2^23 + S_lo       (|S_lo| <= 2^20 < 2^22)
// Then (hF - C12) is exact (a multiple of 256 below 2^28) and
// (hF - C12) + lF rounds once to RN(256*S_hi + S_lo) = (float)cs, which is
// exactly the reference's int->float conversion.  No I2F instruction is needed.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace ql {

constexpr int BLOCK_K = 32;                       // MatMulNBits block size (fixed)
constexpr int32_t HI_SEED = 0x4F400000;           // bits of 1.5 * 2^31
constexpr int32_t LO_SEED = 0x4B400000;           // bits of 1.5 * 2^23
constexpr float C12 = 3233808384.0f;              // 1.5*2^31 + 1.5*2^23 = 771 * 2^22 (exact)

// Error codes shared by the C ABI and the device error word.
enum : int {
    QL_OK = 0,
    QL_EINVAL = 1,        // bad argument / contract violation
    QL_ENOMEM = 2,        // device allocation failed
    QL_ECUDA = 3,         // CUDA runtime error
    QL_ETIMEOUT = 4,      // a bounded device wait gave up (device error word)
    QL_EDEVICE = 5,       // handle lives on a different device than requested
    QL_ENOTSUP = 6,       // unsupported configuration
    QL_ESCRATCH = 7,      // request needs more than the fixed scratch of the no-alloc entry point
};

// ---------------------------------------------------------------- device control block
// One per device (defined in ql_api.cu).  Kernels get a pointer to its first
// member, the device error word: they record the first failure there instead
// of trapping, and the host reads and clears it (ql_device_error, and the
// synchronous entry points after every call).  The same block holds the
// limits of the bounded waits, settable from the host (ql_set_wait_limits).
struct DeviceCtl {
    int err;                          // device error word (0 = none)
    int pad;
    unsigned long long wait_ns;       // limit of a kernel-internal wait
    unsigned long long peer_wait_ns;  // limit of a wait on another GPU's flag
};
constexpr unsigned long long WAIT_LIMIT_NS = 1000000000ull;        // 1 s (default)
constexpr unsigned long long PEER_WAIT_LIMIT_NS = 5000000000ull;   // 5 s (default)

__device__ __forceinline__ void record_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// The wait limits in force.  Waits read them only once they have lasted
// WAIT_CHECK_NS (a global load, kept off the fast path of the pipelines'
// waits, which usually end within microseconds), so limits below 1 ms act as 1 ms.
constexpr unsigned long long WAIT_CHECK_NS = 1000000ull;
__device__ __forceinline__ uint64_t wait_limit(const int* err) {
    return err ? *reinterpret_cast<const volatile unsigned long long*>(&reinterpret_cast<const DeviceCtl*>(err)->wait_ns)
               : WAIT_LIMIT_NS;
}
__device__ __forceinline__ uint64_t peer_wait_limit(const int* err) {
    return err ? *reinterpret_cast<const volatile unsigned long long*>(
                     &reinterpret_cast<const DeviceCtl*>(err)->peer_wait_ns)
               : PEER_WAIT_LIMIT_NS;
}

// ---------------------------------------------------------------- shared-memory helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy ones.  Every thread that read a stage filled by a bulk copy runs
// it before the stage is handed back to the producer: the mbarrier release
// alone does not order those reads against the next bulk copy's writes into
// the same bytes (measured on B200: without it the decode kernel, releasing
// each stage before its relay wait, intermittently produced wrong outputs for
// its last token groups at 57-64 tokens; with it, none in repeated runs).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    return done != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about `ns` nanoseconds have passed.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(bar), "r"(parity), "r"(ns) : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: gives up after the device's wait limit (1 s unless set by
// ql_set_wait_limits) of wall time, records QL_ETIMEOUT in the device error
// word and returns false, so no wait in these kernels can spin forever.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    uint64_t limit = WAIT_CHECK_NS;
    bool read = false;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > limit) {
            if (read) break;
            limit = wait_limit(err);
            read = true;
        }
    }
    record_error(err, QL_ETIMEOUT);
    return false;
}

// 1-D bulk copy global -> shared completing on an mbarrier (no multicast).
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// ---------------------------------------------------------------- packed f32x2 arithmetic
// sm_100 packed FP32 pairs: one instruction, two independently rounded lanes
// (no FTZ), bit-identical to the scalar add/mul/fma on each lane.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ uint64_t i2_pack(int32_t lo, int32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// Exact (float)cs for two elements from seeded hi/lo accumulator pairs.
__device__ __forceinline__ uint64_t cs_to_f2(int32_t h0, int32_t h1, int32_t l0, int32_t l1) {
    const uint64_t negc = f2_pack(-C12, -C12);
    const uint64_t d = f2_add(i2_pack(h0, h1), negc);      // exact: 256*S_hi - 1.5*2^23
    return f2_add(d, i2_pack(l0, l1));                      // one rounding: RN(cs)
}

// ---------------------------------------------------------------- INT4 nibble unpack
// x holds 8 nibbles; returns the even nibbles (bits 0-3 of each byte) or the odd
// ones as 4 bytes, converted to the signed byte (q - zp) with zp folded into
// c = (0x80 - zp) * 0x01010101:  (q + 0x80 - zp) never carries across bytes
// (0x71..0x8F), and ^0x80 maps it back to q - zp in two's complement.
__device__ __forceinline__ uint32_t nib_even_s8(uint32_t x, uint32_t c) {
    return ((x & 0x0F0F0F0Fu) + c) ^ 0x80808080u;
}
__device__ __forceinline__ uint32_t nib_odd_s8(uint32_t x, uint32_t c) {
    return (((x >> 4) & 0x0F0F0F0Fu) + c) ^ 0x80808080u;
}

// ---------------------------------------------------------------- legacy-tensor-core MMA
// mma.sync m16n8k32, A = weights (s8, 16 rows x 32 k), B = activations (8 tokens x 32 k).
__device__ __forceinline__ void mma_s8s8(int32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8u8(int32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Same MMAs with a separate (loop-invariant) C operand: d = a*b + c.
__device__ __forceinline__ void mma_s8s8_c(int32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                           uint32_t b1, const int32_t (&c)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
          "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}
__device__ __forceinline__ void mma_s8u8_c(int32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                           uint32_t b1, const int32_t (&c)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
          "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}

// ---------------------------------------------------------------- PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace ql
