// f32 exp with exactly the results of glibc's expf (the reference's libm).
//
// The reference's silu (native_engine/decoder.rs:1081) and router softmax
// (moe.rs:181-243, via ft-kernel-cpu) call Rust's f32::exp, which lowers to a
// call of the platform libm's expf.  On the x86-64 Linux hosts it runs on that
// is glibc (>= 2.28), whose expf is the published optimized-routines
// algorithm (Szabolcs Nagy, ARM): with N = 32,
//   z = x * (N / ln 2) in double;  k = round-to-nearest(z) via the 1.5 * 2^52
//   shift;  r = z - k (glibc's x86-64 build contracts this into one fused
//   multiply-add, x * (N / ln 2) - k);  s = 2^(k / N) built from a 32-entry
//   table of 2^(i / N) and an exponent shift;
//   exp(x) = s * (C0 r^3 + C1 r^2 + C2 r + 1), C_j the exp2 series fit of
//   the publication divided by N^(3-j);  the double result rounded once to f32;
//   x > 0x1.62e42ep6 -> +inf, x < -0x1.9fe368p6 -> +0, NaN -> NaN.
// It is not correctly rounded (about 7.6e-5 of the floats in [-104, 89]
// differ from the correctly rounded value by an ulp), so a correctly rounded
// device exp would not match the reference; this one matches glibc 2.39's
// expf on all 2^32 inputs (tests/test_host.py builds it on the host and
// compares exhaustively).  The table entry i holds the bits of the double
// nearest to 2^(i/32) minus (i << 47) (so that adding k << 47 rebuilds the
// exponent); tests/test_host.py recomputes it from the mathematics.
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define FOCR_HD __host__ __device__ __forceinline__
#else
#define FOCR_HD inline
#endif

#define FOCR_EXP2_TAB_INIT \
    { \
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL, \
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL, \
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL, \
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL, \
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL, \
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL, \
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL, \
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL \
    }

#if defined(__CUDACC__)
static __device__ const uint64_t focr_exp2_tab_dev[32] = FOCR_EXP2_TAB_INIT;
#endif
static const uint64_t focr_exp2_tab_host[32] = FOCR_EXP2_TAB_INIT;

FOCR_HD double focr_bits_to_double(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
    double d;
    memcpy(&d, &u, 8);
    return d;
#endif
}

FOCR_HD uint64_t focr_double_to_bits(double d) {
#if defined(__CUDA_ARCH__)
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u;
    memcpy(&u, &d, 8);
    return u;
#endif
}

FOCR_HD float libm_expf(float x) {
    if (x != x) return x + x;
    if (x > 0x1.62e42ep6f) return INFINITY;
    if (x < -0x1.9fe368p6f) return 0.0f;
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32, shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32,
                 c2 = 0x1.62e42ff0c52d6p-1 / 32;
    const double xd = (double)x;
    const double z = inv_ln2_n * xd;
    double kd = z + shift;
    const uint64_t ki = focr_double_to_bits(kd);
    kd = kd - shift;
    const double r = fma(inv_ln2_n, xd, -kd);
#if defined(__CUDA_ARCH__)
    uint64_t t = focr_exp2_tab_dev[ki & 31];
#else
    uint64_t t = focr_exp2_tab_host[ki & 31];
#endif
    t += ki << 47;
    const double s = focr_bits_to_double(t);
    const double r2 = r * r;
    const double p = c0 * r + c1;
    double y = c2 * r + 1.0;
    y = p * r2 + y;
    y = y * s;
    return (float)y;
}
