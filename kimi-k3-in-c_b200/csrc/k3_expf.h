/* k3_expf.h -- a single-precision exp that returns, bit for bit, what glibc's expf
 * returns on x86-64 hosts with FMA, so that the router's sigmoid scores on the GPU
 * equal the CPU engine's (k3_ops.c:451 calls expf from libm).
 *
 * glibc's expf is the algorithm published by Szabolcs Nagy in ARM's
 * optimized-routines (2017-2018): with N = 32,
 *     z  = x * N / ln2,  k = round(z) (by adding and subtracting 1.5 * 2^52),  r = z - k
 *     2^(k/N) is read from a 32-entry table of 2^(i/N) with the exponent added in,
 *     exp(x) ~= 2^(k/N) * (C2 r + 1 + (C0 r + C1) r^2)
 * evaluated in double and rounded once to float. It is not correctly rounded (about
 * 0.502 ULP), so a correctly rounded exp disagrees with it on ~170k floats. The x86-64
 * FMA build contracts every multiply-add of that evaluation, including the two uses of
 * x * N / ln2; this restatement does the same with explicit fma(), and a test compares
 * it with the host libm over every float in the scores' range.
 *
 * Inputs are assumed in [-103.9, 88.7] (the router's scores are far inside); outside,
 * the result saturates to 0 or +inf as expf does, and NaN propagates.
 *
 * The 2^(i/32) table holds the correctly rounded doubles; the CPU tests recompute them
 * with 60-digit decimal arithmetic.
 *
 * Attribution and licence of the restated method and its table: ARM optimized-routines,
 * single-precision e^x, Copyright (c) 2017-2018, Arm Limited, SPDX-License-Identifier: MIT
 * (the project is also offered under Apache-2.0 WITH LLVM-exception); GNU libc carries the
 * same method. The MIT licence notice:
 *
 *   Permission is hereby granted, free of charge, to any person obtaining a copy of this
 *   software and associated documentation files (the "Software"), to deal in the Software
 *   without restriction, including without limitation the rights to use, copy, modify,
 *   merge, publish, distribute, sublicense, and/or sell copies of the Software, and to
 *   permit persons to whom the Software is furnished to do so, subject to the following
 *   conditions:
 *
 *   The above copyright notice and this permission notice shall be included in all copies
 *   or substantial portions of the Software.
 *
 *   THE SOFTWARE IS PROVIDED "AS IS", WITHOUT WARRANTY OF ANY KIND, EXPRESS OR IMPLIED,
 *   INCLUDING BUT NOT LIMITED TO THE WARRANTIES OF MERCHANTABILITY, FITNESS FOR A
 *   PARTICULAR PURPOSE AND NONINFRINGEMENT. IN NO EVENT SHALL THE AUTHORS OR COPYRIGHT
 *   HOLDERS BE LIABLE FOR ANY CLAIM, DAMAGES OR OTHER LIABILITY, WHETHER IN AN ACTION OF
 *   CONTRACT, TORT OR OTHERWISE, ARISING FROM, OUT OF OR IN CONNECTION WITH THE SOFTWARE
 *   OR THE USE OR OTHER DEALINGS IN THE SOFTWARE.
 */
#ifndef K3_EXPF_H
#define K3_EXPF_H

#include <stdint.h>

#if defined(__CUDACC__)
#define K3_HD __device__ __forceinline__
#else
#define K3_HD static inline
#endif

#ifdef __CUDACC__
__device__ __constant__ static const uint64_t k3_exp2_tab_d[32] = {
#else
static const uint64_t k3_exp2_tab_h[32] = {
#endif
    0x3ff0000000000000ull, 0x3ff059b0d3158574ull, 0x3ff0b5586cf9890full, 0x3ff11301d0125b51ull,
    0x3ff172b83c7d517bull, 0x3ff1d4873168b9aaull, 0x3ff2387a6e756238ull, 0x3ff29e9df51fdee1ull,
    0x3ff306fe0a31b715ull, 0x3ff371a7373aa9cbull, 0x3ff3dea64c123422ull, 0x3ff44e086061892dull,
    0x3ff4bfdad5362a27ull, 0x3ff5342b569d4f82ull, 0x3ff5ab07dd485429ull, 0x3ff6247eb03a5585ull,
    0x3ff6a09e667f3bcdull, 0x3ff71f75e8ec5f74ull, 0x3ff7a11473eb0187ull, 0x3ff82589994cce13ull,
    0x3ff8ace5422aa0dbull, 0x3ff93737b0cdc5e5ull, 0x3ff9c49182a3f090ull, 0x3ffa5503b23e255dull,
    0x3ffae89f995ad3adull, 0x3ffb7f76f2fb5e47ull, 0x3ffc199bdd85529cull, 0x3ffcb720dcef9069ull,
    0x3ffd5818dcfba487ull, 0x3ffdfc97337b9b5full, 0x3ffea4afa2a490daull, 0x3fff50765b6e4540ull,
};

#ifdef __CUDACC__
#define K3_EXP2_TAB k3_exp2_tab_d
#define K3_AS_DOUBLE(u) __longlong_as_double((long long)(u))
#define K3_AS_U64(d) ((uint64_t)__double_as_longlong(d))
#define K3_FMA(a, b, c) __fma_rn((a), (b), (c))
#define K3_AS_UINT32(f) __float_as_uint(f)
#else
#include <math.h>
#include <string.h>
static inline double k3_as_double_(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
static inline uint64_t k3_as_u64_(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }
static inline uint32_t k3_as_u32f_(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
#define K3_EXP2_TAB k3_exp2_tab_h
#define K3_AS_DOUBLE(u) k3_as_double_(u)
#define K3_AS_U64(d) k3_as_u64_(d)
#define K3_FMA(a, b, c) fma((a), (b), (c))
#define K3_AS_UINT32(f) k3_as_u32f_(f)
#endif

K3_HD float k3_expf(float x)
{
    /* 0x1.62e42ep6 ~ 88.72: overflow above; below -0x1.9fe368p6 ~ -103.97: underflow */
    if (x != x) return x + x;
    if (x > 0x1.62e42ep6f) return (float)(x * 0x1p127) * 0x1p127f; /* +inf */
    if (x < -0x1.9fe368p6f) return 0.0f;
    const double InvLn2N = 0x1.71547652b82fep+0 * 32.0;
    const double SHIFT = 0x1.8p+52;
    const double C0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
    const double C1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
    const double C2 = 0x1.62e42ff0c52d6p-1 / 32;
    const double xd = (double)x;
    double kd = K3_FMA(InvLn2N, xd, SHIFT);
    const uint64_t ki = K3_AS_U64(kd);
    kd -= SHIFT;
    const double r = K3_FMA(InvLn2N, xd, -kd);
    uint64_t t = K3_EXP2_TAB[ki % 32] - ((uint64_t)(ki % 32) << 47);
    t += ki << 47;
    const double s = K3_AS_DOUBLE(t);
    const double r2 = r * r;
    const double z = K3_FMA(C0, r, C1);
    double y = K3_FMA(C2, r, 1.0);
    y = K3_FMA(z, r2, y);
    y = y * s;
    return (float)y;
}

#endif /* K3_EXPF_H */
