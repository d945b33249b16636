// k3_gemv.cuh -- bf16 / fp32 row-dot building blocks (y = W x, W row-major).
//
// The CPU engine's k3_matmul / k3_matmul_bf16 (k3_ops.c:265-291, 1108-1213) sum each row
// in double with sixteen accumulators. Here each lane sums its slice of the row in fp32
// with packed f32x2 FMAs and the warp combines the slices; fp32 accumulation is within
// the 1e-3 relative contract for the decode shapes (rows of 7168 and 2048 terms).
//
// Chunk = 16 bytes of W: 8 bf16 or 4 fp32 elements. Lane `l` owns chunks l, l+32, ...;
// the activations are staged per CTA in shared memory as fp32.
#pragma once
#include "k3_common.cuh"

namespace k3 {

// bf16 chunk c covers x[8c .. 8c+8) = float4 2c and 2c+1; they are stored swapped on
// every other group of four chunks so that eight consecutive lanes reading float4 k of
// their chunks hit eight distinct bank groups.
__device__ __forceinline__ int xb_idx(int c, int k) { return 2 * c + (k ^ ((c >> 2) & 1)); }

// Each thread issues up to 8 loads before its first store (a loop with a run-time count
// and one load per iteration would pay the memory latency once per iteration).
__device__ __forceinline__ void stage_x_bf16(float4 *xs, const float *x, int in)
{
    const int nf4 = in >> 2;
    const int nb = blockDim.x;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        const float4 *x4 = reinterpret_cast<const float4 *>(x);
        for (int f0 = threadIdx.x; f0 < nf4; f0 += 8 * nb) {
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; i++)
                if (f0 + i * nb < nf4) v[i] = __ldg(x4 + f0 + i * nb);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int f = f0 + i * nb;
                if (f < nf4) xs[xb_idx(f >> 1, f & 1)] = v[i];
            }
        }
    } else {
        for (int f0 = threadIdx.x; f0 < nf4; f0 += 8 * nb) {
            float4 v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int f = f0 + i * nb;
                if (f < nf4) v[i] = make_float4(x[4 * f], x[4 * f + 1], x[4 * f + 2], x[4 * f + 3]);
            }
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int f = f0 + i * nb;
                if (f < nf4) xs[xb_idx(f >> 1, f & 1)] = v[i];
            }
        }
    }
}

__device__ __forceinline__ float2 bf16x2_to_f32x2(uint32_t w)
{
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ float2 bf16_chunk_dot(const uint4 w, const float4 *xs, int c, float2 acc)
{
    const float4 xa = xs[xb_idx(c, 0)];
    const float4 xb = xs[xb_idx(c, 1)];
    acc = ffma2(bf16x2_to_f32x2(w.x), make_float2(xa.x, xa.y), acc);
    acc = ffma2(bf16x2_to_f32x2(w.y), make_float2(xa.z, xa.w), acc);
    acc = ffma2(bf16x2_to_f32x2(w.z), make_float2(xb.x, xb.y), acc);
    acc = ffma2(bf16x2_to_f32x2(w.w), make_float2(xb.z, xb.w), acc);
    return acc;
}

// R rows of bf16 W (row pointers pr[r]) against staged x of `nch` chunks (in / 8).
// Loads go in segments of SEG chunks per lane per row to bound registers.
template <int R, int SEG>
__device__ __forceinline__ void bf16_rows_partial(float acc[R], const uint16_t *const pr[R],
                                                  const float4 *xs, int nch)
{
    const int lane = threadIdx.x & 31;
    float2 a2[R];
#pragma unroll
    for (int r = 0; r < R; r++) a2[r] = make_float2(0.f, 0.f);
    for (int base = 0; base < nch; base += 32 * SEG) {
        uint4 w[R][SEG];
#pragma unroll
        for (int r = 0; r < R; r++) {
#pragma unroll
            for (int j = 0; j < SEG; j++) {
                const int c = base + lane + 32 * j;
                w[r][j] = (c < nch) ? ldg_nc_v4(pr[r] + 8 * (size_t)c) : make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int j = 0; j < SEG; j++) {
            const int c = base + lane + 32 * j;
            if (c < nch) {
#pragma unroll
                for (int r = 0; r < R; r++) a2[r] = bf16_chunk_dot(w[r][j], xs, c, a2[r]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = a2[r].x + a2[r].y;
}

}  // namespace k3
