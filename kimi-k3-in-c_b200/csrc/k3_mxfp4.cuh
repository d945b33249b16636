// k3_mxfp4.cuh -- device building blocks for MXFP4 (E2M1 codes + E8M0 group scales)
// row dot products, shared by the single-matrix GEMV, the config-0 expert and the MoE
// expert kernels.
//
// Layout (the CPU engine's, include/k3/k3.h:523-560): packed [rows][in/2] bytes, the
// low nibble of each byte is the even element; scales [rows][in/group] bytes.
//
// FAST PATH (group == 32, in % 32 == 0, 16-byte aligned rows): one 16-byte load is one
// whole scale group of one row. Lane `l` of a warp owns chunks l, l+32, l+64, ... of
// every row it touches, so the activation slice each lane needs is the same for every
// row: it is staged once per CTA in shared memory (fp32, swizzled so that the eight
// 16-byte reads of one chunk by eight consecutive lanes hit eight different bank
// groups) and re-read per row.
//
// Per chunk the codes go E2M1 -> f16x2 with cvt.rn.f16x2.e2m1x2 (exact), f16 -> f32
// (exact), and are multiplied into packed f32 pairs with fma.rn.f32x2. The 32 products
// of a group are summed in fp32, multiplied by the group's power-of-two scale (exact)
// and added to the row accumulator; a scale byte of 255 contributes nothing, as in
// k3_ops.c:1478 and 1536. The CPU engine accumulates in double (k3_ops.c:1433); fp32
// accumulation here stays far inside the 1e-3 relative contract.
#pragma once
#include "k3_common.cuh"

namespace k3 {

// Index (in float4 units) of logical float4 k (0..7) of chunk c in the swizzled x tile.
__device__ __forceinline__ int xs_idx(int c, int k) { return (c << 3) + (k ^ (c & 7)); }

// Stage x[0..in) (fp32, in % 32 == 0) into the swizzled shared tile.
__device__ __forceinline__ void stage_x_mxfp4(float4 *xs, const float *x, int in)
{
    const int nf4 = in >> 2;
    const int nb = blockDim.x;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    // up to 8 loads in flight per thread before the stores
    for (int f0 = threadIdx.x; f0 < nf4; f0 += 8 * nb) {
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (f0 + i * nb < nf4) v[i] = x4[f0 + i * nb];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int f = f0 + i * nb;
            if (f < nf4) xs[xs_idx(f >> 3, f & 7)] = v[i];
        }
    }
}

// Same, for x in memory that may not be 16-byte aligned.
__device__ __forceinline__ void stage_x_mxfp4_scalar(float4 *xs, const float *x, int in)
{
    const int nf4 = in >> 2;
#pragma unroll 8
    for (int f = threadIdx.x; f < nf4; f += blockDim.x) {
        const int c = f >> 3, k = f & 7;
        xs[xs_idx(c, k)] = make_float4(x[4 * f], x[4 * f + 1], x[4 * f + 2], x[4 * f + 3]);
    }
}

// Dot product of one 16-byte group (32 codes) with its 32 activations, unscaled.
__device__ __forceinline__ float mxfp4_chunk_dot(const uint4 w, const float4 *xs, int c)
{
    float2 acc = make_float2(0.f, 0.f);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
        uint32_t h[4];
        e2m1x8_to_f16x8(words[q], h);
        const float4 xa = xs[xs_idx(c, 2 * q)];
        const float4 xb = xs[xs_idx(c, 2 * q + 1)];
        acc = ffma2(f16x2_to_f32x2(h[0]), make_float2(xa.x, xa.y), acc);
        acc = ffma2(f16x2_to_f32x2(h[1]), make_float2(xa.z, xa.w), acc);
        acc = ffma2(f16x2_to_f32x2(h[2]), make_float2(xb.x, xb.y), acc);
        acc = ffma2(f16x2_to_f32x2(h[3]), make_float2(xb.z, xb.w), acc);
    }
    return acc.x + acc.y;
}

// Folds one group into a row accumulator with the E8M0 scale byte `sb`.
__device__ __forceinline__ float mxfp4_fold(float racc, float dot, uint32_t sb)
{
    const float s = e8m0_to_f32(sb);
    const float r = fmaf(dot, s, racc);
    return sb == 255u ? racc : r;
}

// R rows (row pointers pr[r], scale pointers sr[r]) against the staged x of `nch`
// chunks; returns per-lane partial sums in acc[r] (not yet reduced across the warp).
// NCHMAX bounds the chunks per lane (nch <= 32 * NCHMAX).
template <int R, int NCHMAX>
__device__ __forceinline__ void mxfp4_rows_partial(float acc[R],
                                                   const unsigned char *const pr[R],
                                                   const unsigned char *const sr[R],
                                                   const float4 *xs, int nch)
{
    const int lane = threadIdx.x & 31;
    uint4 w[R][NCHMAX];
    uint32_t sb[R][NCHMAX];
#pragma unroll
    for (int r = 0; r < R; r++) {
#pragma unroll
        for (int j = 0; j < NCHMAX; j++) {
            const int c = lane + 32 * j;
            if (c < nch) {
                w[r][j] = ldg_nc_v4(pr[r] + 16 * (size_t)c);
                sb[r][j] = __ldg(sr[r] + c);
            } else {
                w[r][j] = make_uint4(0, 0, 0, 0);
                sb[r][j] = 255u;
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0.f;
#pragma unroll
    for (int j = 0; j < NCHMAX; j++) {
        const int c = lane + 32 * j;
        if (c < nch) {
#pragma unroll
            for (int r = 0; r < R; r++)
                acc[r] = mxfp4_fold(acc[r], mxfp4_chunk_dot(w[r][j], xs, c), sb[r][j]);
        }
    }
}

}  // namespace k3
