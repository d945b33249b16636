// k3_mxfp4.cu -- k3_mxfp4_dequant and k3_matmul_mxfp4 (include/k3/k3.h) on sm_100a.
//
//   k3_mxfp4_dequant  follows k3_ops.c:1787-1817 and is bit-exact: every output is the
//                     fp32 product E2M1[code] * 2^(scale-127), as on the CPU.
//   k3_matmul_mxfp4   follows k3_ops.c:1380-1785 (y = W x straight out of MXFP4,
//                     scale 255 contributes nothing, odd `in` and group > 64 rejected).
#include "k3_mxfp4.cuh"
#include "k3_moe.cuh"
#include "k3_ops.cuh"

namespace k3 {

// Code -> fp32 value. Bit 3 is the sign; code 8 is -0.0 (k3_ops.c:1066-1069).
__device__ __forceinline__ float e2m1_value(uint32_t code)
{
    // magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6 as fp32 bit patterns (low 16 bits are zero)
    const uint32_t mag = code & 7u;
    const uint32_t hi = (mag == 0) ? 0u : (mag == 1) ? 0x3F00u : (mag == 2) ? 0x3F80u
                      : (mag == 3) ? 0x3FC0u : (mag == 4) ? 0x4000u : (mag == 5) ? 0x4040u
                      : (mag == 6) ? 0x4080u : 0x40C0u;
    return __uint_as_float(((hi | ((code & 8u) << 12)) << 16));
}

// One thread per packed byte: two outputs.
__global__ void k_mxfp4_dequant(float *out, const unsigned char *packed,
                                const unsigned char *scales, int rows, int pcols, int group)
{
    const int width = pcols * 2;
    const int ngrp = (width + group - 1) / group;
    const size_t total = (size_t)rows * pcols;
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < total;
         b += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(b / pcols);
        const int j = (int)(b % pcols);
        const uint32_t byte = packed[b];
        const int i0 = 2 * j, i1 = 2 * j + 1;
        const uint32_t s0 = scales[(size_t)r * ngrp + i0 / group];
        const uint32_t s1 = scales[(size_t)r * ngrp + i1 / group];
        const float m0 = e8m0_to_f32(s0), m1 = e8m0_to_f32(s1);
        // the same single fp32 multiply as the CPU: E2M1 value times the power of two
        out[(size_t)r * width + i0] = __fmul_rn(e2m1_value(byte & 15u), m0);
        out[(size_t)r * width + i1] = __fmul_rn(e2m1_value(byte >> 4), m1);
    }
}

// Any even `in`, any group >= 1: one warp per row, lanes over groups. Used when the
// fast path's layout conditions do not hold.
__global__ void k_mxfp4_gemv_generic(float *y, const float *x, const unsigned char *packed,
                                     const unsigned char *scales, int in, int rows, int group)
{
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int pcols = in / 2;
    const int ngrp = (in + group - 1) / group;
    for (int r = warp; r < rows; r += nwarps) {
        const unsigned char *pr = packed + (size_t)r * pcols;
        const unsigned char *sr = scales + (size_t)r * ngrp;
        float acc = 0.f;
        for (int gi = lane; gi < ngrp; gi += 32) {
            const uint32_t sb = sr[gi];
            if (sb == 255u) continue;
            const int lo = gi * group;
            const int hi = min(in, lo + group);
            float sub = 0.f;
            for (int i = lo; i < hi; i++) {
                const uint32_t byte = pr[i >> 1];
                const uint32_t code = (i & 1) ? (byte >> 4) : (byte & 15u);
                sub = fmaf(e2m1_value(code), x[i], sub);
            }
            acc = fmaf(sub, e8m0_to_f32(sb), acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[r] = acc;
    }
}

// Fast path: group 32, in % 32 == 0, 16-byte aligned rows. x staged once per CTA.
template <int R, int NCHMAX>
__global__ void __launch_bounds__(256) k_mxfp4_gemv_fast(float *y, const float *x,
                                                         const unsigned char *packed,
                                                         const unsigned char *scales,
                                                         int in, int rows, int x_aligned)
{
    extern __shared__ float4 xs[];
    if (x_aligned) stage_x_mxfp4(xs, x, in);
    else stage_x_mxfp4_scalar(xs, x, in);
    __syncthreads();
    const int nch = in >> 5;
    const int pcols = in >> 1;
    const int ngrp = in >> 5;
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r0 = warp * R; r0 < rows; r0 += nwarps * R) {
        const unsigned char *pr[R];
        const unsigned char *sr[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int rr = min(r0 + r, rows - 1);
            pr[r] = packed + (size_t)rr * pcols;
            sr[r] = scales + (size_t)rr * ngrp;
        }
        float acc[R];
        mxfp4_rows_partial<R, NCHMAX>(acc, pr, sr, xs, nch);
#pragma unroll
        for (int r = 0; r < R; r++) {
            const float v = warp_sum(acc[r]);
            if (lane == 0 && r0 + r < rows) y[r0 + r] = v;
        }
    }
}

static bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// Launches y = W x on device pointers. Chooses the fast kernel when it applies.
int mxfp4_gemv(float *y, const float *x, const unsigned char *packed,
               const unsigned char *scales, int in, int rows, int group, cudaStream_t s)
{
    if (rows <= 0 || in <= 0) return K3D_OK;
    // tensor-core path: 16-row tiles streamed by bulk copies (k3_mxfp4_mma.cu)
    if (group == 32 && mma_supported(in, rows, 1) && aligned16(packed) && aligned16(scales)) {
        char *ws = (char *)scratch((size_t)2 * in * sizeof(__half) + 256, 2);
        if (!ws) return k3d_status();
        __half *xb = (__half *)ws;
        float *xs = (float *)(ws + (size_t)2 * in * sizeof(__half));
        MoeWork w{};
        w.single.p2 = packed;
        w.single.s2 = scales;
        w.single_mode = 1;
        w.ntok_single = 1;
        w.K = 1;
        K3_TRY(xsplit(xb, xs, x, in, 1, in, s));
        return mxfp4_mma_launch(1, w, 1, in, rows, xb, xs, 1, y, s);
    }
    const bool fast = group == 32 && (in % 32) == 0 && aligned16(packed) && in <= 32 * 32 * 8;
    if (fast) {
        const int nch = in / 32;
        const int threads = 256;
        const size_t smem = (size_t)in * sizeof(float);
        const int rows_per_cta = 8 * 2 * 4;
        int grid = (rows + rows_per_cta - 1) / rows_per_cta;
        const int cap = sm_count() * 4;
        if (grid > cap) grid = cap;
        if (grid < 1) grid = 1;
        const int xa = aligned16(x);
        if (nch <= 32) {
            static bool attr = false;
            if (!attr) {
                allow_smem_max(k_mxfp4_gemv_fast<2, 1>);
                attr = true;
            }
            k_mxfp4_gemv_fast<2, 1><<<grid, threads, smem, s>>>(y, x, packed, scales, in, rows, xa);
        } else if (nch <= 64) {
            static bool attr = false;
            if (!attr) {
                allow_smem_max(k_mxfp4_gemv_fast<2, 2>);
                attr = true;
            }
            k_mxfp4_gemv_fast<2, 2><<<grid, threads, smem, s>>>(y, x, packed, scales, in, rows, xa);
        } else if (nch <= 128) {
            static bool attr = false;
            if (!attr) {
                allow_smem_max(k_mxfp4_gemv_fast<2, 4>);
                attr = true;
            }
            k_mxfp4_gemv_fast<2, 4><<<grid, threads, smem, s>>>(y, x, packed, scales, in, rows, xa);
        } else {
            static bool attr = false;
            if (!attr) {
                allow_smem_max(k_mxfp4_gemv_fast<2, 8>);
                attr = true;
            }
            k_mxfp4_gemv_fast<2, 8><<<grid, threads, smem, s>>>(y, x, packed, scales, in, rows, xa);
        }
    } else {
        const int threads = 256;
        int grid = (rows + 7) / 8;
        if (grid > sm_count() * 8) grid = sm_count() * 8;
        k_mxfp4_gemv_generic<<<grid, threads, 0, s>>>(y, x, packed, scales, in, rows, group);
    }
    note_launch();
    return check_launch("mxfp4 gemv");
}

}  // namespace k3

using namespace k3;

extern "C" {

void k3_mxfp4_dequant(float *out, const unsigned char *packed, const unsigned char *scales,
                      int rows, int pcols, int group)
{
    if (ensure_ctx()) return;
    if (rows < 0 || pcols < 0 || group <= 0) {
        fail(K3D_EINVAL, "k3_mxfp4_dequant rows=%d pcols=%d group=%d", rows, pcols, group);
        return;
    }
    if (rows == 0 || pcols == 0) return;
    const int width = 2 * pcols;
    const int ngrp = (width + group - 1) / group;
    Stage st;
    const unsigned char *P = (const unsigned char *)st.weight(packed, (size_t)rows * pcols);
    const unsigned char *S = (const unsigned char *)st.weight(scales, (size_t)rows * ngrp);
    float *O = (float *)st.out(out, (size_t)rows * width * sizeof(float));
    if (st.err) return;
    const size_t total = (size_t)rows * pcols;
    int grid = (int)((total + 255) / 256);
    if (grid > sm_count() * 16) grid = sm_count() * 16;
    k_mxfp4_dequant<<<grid, 256, 0, stream()>>>(O, P, S, rows, pcols, group);
    note_launch();
    if (check_launch("mxfp4 dequant")) return;
    st.finish();
}

void k3_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                     const unsigned char *scales, int in, int rows, int group)
{
    if (ensure_ctx()) return;
    // The CPU engine aborts on these two (k3_ops.c:1383-1401); here they are recorded.
    if (in & 1) { fail(K3D_EINVAL, "k3_matmul_mxfp4 called with odd in=%d", in); return; }
    if (group > 64 || group <= 0) {
        fail(K3D_EINVAL, "k3_matmul_mxfp4 called with group=%d (must be 1..64)", group);
        return;
    }
    if (rows <= 0 || in <= 0) return;
    const int ngrp = (in + group - 1) / group;
    Stage st;
    const unsigned char *P = (const unsigned char *)st.weight(packed, (size_t)rows * (in / 2));
    const unsigned char *S = (const unsigned char *)st.weight(scales, (size_t)rows * ngrp);
    const float *X = (const float *)st.in(x, (size_t)in * sizeof(float));
    float *Y = (float *)st.out(y, (size_t)rows * sizeof(float));
    if (st.err) return;
    if (mxfp4_gemv(Y, X, P, S, in, rows, group, stream())) return;
    st.finish();
}

}  // extern "C"
