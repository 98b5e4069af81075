/*
 * expf_ref.c -- TEST INFRASTRUCTURE ONLY: a restatement of the single-precision
 * exponential the reference's SiLU calls, and an exhaustive checker of it
 * against the host C library.
 *
 * The reference decoder computes the MLP's SiLU * up product as
 *     g1[i] = siluf(g1[i]) * g2[i],   siluf(x) = x / (1.0f + std::exp(-x))
 * (kernel/qwen35_decoder.cpp:129, :408), so its bits depend on the host libm's
 * expf, which is not correctly rounded (its documented error bound is about
 * 0.502 ulp): a correctly rounded exponential differs from it on a fraction of
 * inputs near rounding midpoints, and a changed last bit of a SiLU output can
 * change the down projection's activation scale.  The GPU path therefore
 * follows the method that libm's expf uses, which is published (the
 * table-driven double-precision scheme of the Arm optimized-routines project,
 * used by glibc since 2.27):
 *     k = round(x * 32 / ln 2),  r = x * 32 / ln 2 - k,
 *     exp(x) = 2^(k/32) * 2^(r/32),
 *     2^(r/32) ~ 1 + c2 r + c1 r^2 + c0 r^3          (|r| <= 1/2),
 * all in double, with 2^(i/32) from a 32-entry table (computed here as the
 * correctly rounded doubles of 2^(i/32); entries stored minus i << 47 so that
 * adding k << 47 scales by 2^(k/32)), the published minimax coefficients, the
 * rounding of x*32/ln2 to an integer done by adding and subtracting 1.5*2^52,
 * and one final rounding of the double result to float.  Inputs of magnitude
 * >= 88 take the special cases: overflow to +inf above log(2^128), zero below
 * log(2^-150), x + x for NaN and +inf, 0 for -inf.
 *
 * Where the C library's expf is built with FMA contraction (the x86-64 variant
 * selected on CPUs with FMA), the product x * 32/ln2 is fused into both the
 * rounding shift and the reduced argument, and c0 r + c1, c2 r + 1 and
 * z r^2 + y are fused multiply-adds; ql_expf_restated(x, 1) does the same,
 * ql_expf_restated(x, 0) fuses nothing.  ql_expf_check() compares one of them
 * with the library's expf on every float bit pattern in [lo, hi] and reports
 * the mismatches: zero over all 2^32 inputs for the FMA form on the hosts this
 * project runs on (the plain form differs on 2 inputs, 32.5646324 and
 * -63.0994606, by one ulp).  That is what lets the CUDA SiLU prologue
 * (expf_host_method in breeze_engine_b200/csrc/ql_quant.cuh) promise the
 * reference's bits.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* 2^(i/32) rounded to double, minus i << 47, for i = 0..31. */
static const uint64_t EXP2_32[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

static double as_double(uint64_t u) {
    double d;
    memcpy(&d, &u, 8);
    return d;
}
static uint64_t as_u64(double d) {
    uint64_t u;
    memcpy(&u, &d, 8);
    return u;
}
static uint32_t as_u32(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

float ql_expf_restated(float x, int use_fma) {
    const double invln2_32 = 0x1.71547652b82fep+0 * 32;     /* 32 / ln 2 */
    const double shift = 0x1.8p+52;                         /* rounds to an integer when added */
    const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;  /* the method's minimax coefficients, */
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;       /* scaled for r in units of 1/32 */
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32;
    const uint32_t top = (as_u32(x) >> 20) & 0x7ff;
    if (top >= ((as_u32(88.0f) >> 20) & 0x7ff)) {
        if (as_u32(x) == as_u32(-INFINITY)) return 0.0f;
        if (top >= ((as_u32(INFINITY) >> 20) & 0x7ff)) return x + x;   /* NaN, +inf */
        if (x > 0x1.62e42ep6f) return INFINITY;                          /* above log(2^128) */
        if (x < -0x1.9fe368p6f) return 0.0f;                             /* below log(2^-150) */
    }
    const double xd = (double)x;
    double z = invln2_32 * xd;
    /* the FMA build fuses the product x * 32/ln2 into the rounding shift and
       into the reduced argument r (both use the unrounded product) */
    double kd = use_fma ? fma(invln2_32, xd, shift) : z + shift;
    const uint64_t ki = as_u64(kd);
    kd -= shift;
    const double r = use_fma ? fma(invln2_32, xd, -kd) : z - kd;
    const uint64_t t = EXP2_32[ki % 32] + (ki << 47);
    const double s = as_double(t);
    double y;
    if (use_fma) {
        z = fma(c0, r, c1);
        const double r2 = r * r;
        y = fma(c2, r, 1.0);
        y = fma(z, r2, y);
    } else {
        z = c0 * r + c1;
        const double r2 = r * r;
        y = c2 * r + 1.0;
        y = z * r2 + y;
    }
    y = y * s;
    return (float)y;
}

/* The reference's SiLU times up, on this restatement. */
float ql_silu_mul_restated(float g, float u, int use_fma) {
    return (g / (1.0f + ql_expf_restated(-g, use_fma))) * u;
}

/* out[i] = silu(g[i]) * u[i] for n elements (the FMA form). */
void ql_silu_mul_array(const float* g, const float* u, float* out, long long n) {
    for (long long i = 0; i < n; ++i) out[i] = ql_silu_mul_restated(g[i], u[i], 1);
}

/* Mismatches of the restatement against the library's expf over the float bit
 * patterns lo..hi (inclusive); NaN results compare equal to any NaN.  The first
 * mismatching pattern, if any, goes to *first. */
typedef float (*expf_fn)(float);
static volatile expf_fn lib_expf = expf;

unsigned long long ql_expf_check(uint32_t lo, uint32_t hi, int use_fma, uint32_t* first) {
    unsigned long long bad = 0;
    int64_t first_bad = -1;
#pragma omp parallel for reduction(+ : bad) schedule(static)
    for (int64_t i = (int64_t)lo; i <= (int64_t)hi; ++i) {
        float x;
        const uint32_t u = (uint32_t)i;
        memcpy(&x, &u, 4);
        const float a = lib_expf(x), b = ql_expf_restated(x, use_fma);
        if (a != a && b != b) continue;
        if (as_u32(a) != as_u32(b)) {
            ++bad;
#pragma omp critical
            if (first_bad < 0 || i < first_bad) first_bad = i;
        }
    }
    if (first) *first = first_bad < 0 ? 0u : (uint32_t)first_bad;
    return bad;
}
