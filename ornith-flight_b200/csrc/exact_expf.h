/*
 * exact_expf.h — expf(x) for x <= 0 that reproduces the host C library's
 * result bit-for-bit, for use in the routing softmax.
 *
 * Why: the reference's router softmax (engine/src/model.c:1031) and
 * model_get_routing (model.c:312) call the host C library's expf. On the
 * x86-64 hosts this engine targets that is GNU libc >= 2.28, whose expf is
 * NOT correctly rounded (about 97k of the 2^31 non-positive inputs differ
 * from the once-rounded exact value). Bit-exact top-k weights therefore need
 * the library's own method, restated here:
 *
 *   Method (Szabolcs Nagy, "expf" of ARM optimized-routines, adopted by GNU
 *   libc 2.28): exp(x) = 2^(k/N) * 2^(r/N) with N = 32,
 *   z = x * N/ln2, k = nearest integer of z, r = z - k in [-1/2, 1/2];
 *   2^(k/N) comes from a 32-entry table of 2^(i/N) (exponent bits folded in),
 *   2^(r/N) from a cubic polynomial; everything in double, rounded once to
 *   float at the end. The x86-64 build of the library selects its FMA
 *   variant on FMA-capable CPUs, where the compiler contracts z*... + c into
 *   fused multiply-adds, including the two uses of x*N/ln2; that is the form
 *   written below.
 *
 * Table entries are the round-to-nearest doubles of 2^(i/32), minus i<<47 so
 * that adding k<<47 yields 2^(k/32). Validated exhaustively against the host
 * library over every float x <= 0 (tests/test_exact_expf.py builds this header
 * as host code and compares all 2^31 inputs); the GPU test compares device
 * results against the host library on a strided sample.
 *
 * Attribution: the method, the 2^(i/32) table and the polynomial
 * coefficients are those published in ARM optimized-routines (math/expf.c,
 * math/exp2f_data.c; Copyright (c) 2017-2018, Arm Limited;
 * SPDX-License-Identifier: MIT OR Apache-2.0 WITH LLVM-exception), from which
 * GNU libc 2.28 took its expf. The numeric constants below restate those
 * published values; the code around them is this library's own.
 *
 * Inputs below -0x1.9fe368p6 (where the result underflows) return +0, as the
 * library does. Only x <= 0 is supported; routing never produces x > 0.
 */
#ifndef OFB_EXACT_EXPF_H
#define OFB_EXACT_EXPF_H

#include <stdint.h>
#include <string.h>

#include <math.h>
#ifdef __CUDACC__
#define OFB_HD __device__ __forceinline__
#else
#define OFB_HD static inline
#endif
/* fused multiply-add, one rounding (device: the DFMA instruction) */
#define OFB_FMA(a, b, c) fma((a), (b), (c))

#ifdef __CUDACC__
__device__ __constant__ static const unsigned long long ofb_exp2_tab[32] = {
#else
static const unsigned long long ofb_exp2_tab[32] = {
#endif
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
};

OFB_HD double ofb_bits_to_double(unsigned long long u) {
#ifdef __CUDACC__
    return __longlong_as_double((long long)u);
#else
    double d;
    memcpy(&d, &u, 8);
    return d;
#endif
}

OFB_HD unsigned long long ofb_double_to_bits(double d) {
#ifdef __CUDACC__
    return (unsigned long long)__double_as_longlong(d);
#else
    unsigned long long u;
    memcpy(&u, &d, 8);
    return u;
#endif
}

OFB_HD float ofb_exact_expf(float x) {
    /* N/ln2, the rounding shift 1.5*2^52, and the cubic for 2^(r/N) with
     * coefficients scaled by 1/N^3, 1/N^2, 1/N. */
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32;
    if (x < -0x1.9fe368p6f) return 0.0f; /* underflow, including -inf */
    double xd = (double)x;
    double kd = OFB_FMA(inv_ln2_n, xd, shift);
    unsigned long long ki = ofb_double_to_bits(kd);
    kd -= shift;
    double r = OFB_FMA(inv_ln2_n, xd, -kd);
    unsigned long long t = ofb_exp2_tab[ki & 31];
    t += ki << 47;
    double s = ofb_bits_to_double(t);
    double z = OFB_FMA(c0, r, c1);
    double r2 = r * r;
    double y = OFB_FMA(c2, r, 1.0);
    y = OFB_FMA(z, r2, y);
    y = y * s;
    return (float)y;
}

#endif
