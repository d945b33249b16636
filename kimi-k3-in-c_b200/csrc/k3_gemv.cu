// k3_gemv.cu -- fp32 and bf16 GEMVs: k3_matmul and k3_matmul_bf16 (include/k3/k3.h,
// following k3_ops.c:265-291 and 1108-1213) and k3d_gemv_bf16, plus the fused
// gate|up -> SiLU*mul GEMV used by the shared and dense SwiGLU MLPs.
#include <cstdlib>

#include "k3_gemv.cuh"
#include "k3_ops.cuh"

namespace k3 {

enum { EPI_STORE = 0, EPI_ACCUM = 1 };

// y[t][r] (+)= W[r] . x[t] for up to NT tokens, bf16 W, in % 8 == 0, 16-byte rows.
template <int R, int SEG, int NT>
__global__ void __launch_bounds__(256) k_gemv_bf16(float *y, const float *x, const uint16_t *W,
                                                   int in, int out, int T, int accumulate)
{
    pdl_wait();
    pdl_trigger();
    extern __shared__ float4 xs[];
    const int nf4 = in >> 2;
    for (int t = 0; t < T; t++) stage_x_bf16(xs + (size_t)t * nf4, x + (size_t)t * in, in);
    __syncthreads();
    const int nch = in >> 3;
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r0 = warp * R; r0 < out; r0 += nwarps * R) {
        const uint16_t *pr[R];
#pragma unroll
        for (int r = 0; r < R; r++) pr[r] = W + (size_t)min(r0 + r, out - 1) * in;
        if (NT == 1) {
            float acc[R];
            bf16_rows_partial<R, SEG>(acc, pr, xs, nch);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const float v = warp_sum(acc[r]);
                if (lane == 0 && r0 + r < out) {
                    float *dst = y + (r0 + r);
                    *dst = accumulate ? *dst + v : v;
                }
            }
        } else {
            for (int t = 0; t < T; t++) {
                float acc[R];
                bf16_rows_partial<R, SEG>(acc, pr, xs + (size_t)t * nf4, nch);
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const float v = warp_sum(acc[r]);
                    if (lane == 0 && r0 + r < out) {
                        float *dst = y + (size_t)t * out + (r0 + r);
                        *dst = accumulate ? *dst + v : v;
                    }
                }
            }
        }
    }
}

// act[t][i] = silu(Wg[i] . x[t]) * (Wu[i] . x[t]) for bf16 gate/up matrices.
template <int SEG>
__global__ void __launch_bounds__(256) k_gemv_bf16_swiglu(float *act, const float *x,
                                                          const uint16_t *Wg, const uint16_t *Wu,
                                                          int in, int inter, int T)
{
    pdl_wait();
    pdl_trigger();
    extern __shared__ float4 xs[];
    const int nf4 = in >> 2;
    for (int t = 0; t < T; t++) stage_x_bf16(xs + (size_t)t * nf4, x + (size_t)t * in, in);
    __syncthreads();
    const int nch = in >> 3;
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int i = warp; i < inter; i += nwarps) {
        const uint16_t *pr[2] = {Wg + (size_t)i * in, Wu + (size_t)i * in};
        for (int t = 0; t < T; t++) {
            float acc[2];
            bf16_rows_partial<2, SEG>(acc, pr, xs + (size_t)t * nf4, nch);
            const float g = warp_sum(acc[0]);
            const float u = warp_sum(acc[1]);
            if (lane == 0) act[(size_t)t * inter + i] = silu_f(g) * u;
        }
    }
}

// fp32 W, in % 4 == 0, 16-byte rows: chunk = 4 elements = one float4 of x (no swizzle
// needed, consecutive lanes read consecutive float4s).
template <int R, int SEG>
__global__ void __launch_bounds__(256) k_gemv_f32(float *y, const float *x, const float *W,
                                                  int in, int out)
{
    extern __shared__ float4 xs[];
    const int nf4 = in >> 2;
    for (int f = threadIdx.x; f < nf4; f += blockDim.x)
        xs[f] = make_float4(x[4 * f], x[4 * f + 1], x[4 * f + 2], x[4 * f + 3]);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r0 = warp * R; r0 < out; r0 += nwarps * R) {
        float2 a2[R];
#pragma unroll
        for (int r = 0; r < R; r++) a2[r] = make_float2(0.f, 0.f);
        for (int base = 0; base < nf4; base += 32 * SEG) {
            uint4 w[R][SEG];
#pragma unroll
            for (int r = 0; r < R; r++) {
                const float *pr = W + (size_t)min(r0 + r, out - 1) * in;
#pragma unroll
                for (int j = 0; j < SEG; j++) {
                    const int c = base + lane + 32 * j;
                    w[r][j] = (c < nf4) ? ldg_nc_v4(pr + 4 * (size_t)c) : make_uint4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int j = 0; j < SEG; j++) {
                const int c = base + lane + 32 * j;
                if (c < nf4) {
                    const float4 xv = xs[c];
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        a2[r] = ffma2(make_float2(__uint_as_float(w[r][j].x), __uint_as_float(w[r][j].y)),
                                      make_float2(xv.x, xv.y), a2[r]);
                        a2[r] = ffma2(make_float2(__uint_as_float(w[r][j].z), __uint_as_float(w[r][j].w)),
                                      make_float2(xv.z, xv.w), a2[r]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++) {
            const float v = warp_sum(a2[r].x + a2[r].y);
            if (lane == 0 && r0 + r < out) y[r0 + r] = v;
        }
    }
}

// Any shape / alignment: one warp per row, lanes over elements.
template <typename WT>
__global__ void k_gemv_generic(float *y, const float *x, const WT *W, int in, int out,
                               int accumulate)
{
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r = warp; r < out; r += nwarps) {
        const WT *row = W + (size_t)r * in;
        float acc = 0.f;
        for (int i = lane; i < in; i += 32) {
            float w;
            if (sizeof(WT) == 2) w = bf16_to_f32((uint16_t)row[i]);
            else w = (float)row[i];
            acc = fmaf(w, x[i], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[r] = accumulate ? y[r] + acc : acc;
    }
}

// Up to 8 weight matrices sharing the input x (q|k|v|g|b|f_a of a KDA layer, q_a|kv_a|g
// of an MLA layer): one launch over the concatenated row space.
template <typename K>
static void allow_smem(K kern)
{
    allow_smem_max(kern);
}
int grid_for(int rows, int rows_per_cta);

struct Segs {
    const uint16_t *W[8];
    float *y[8];
    int rows[8];
    int start[9];      // prefix of rows
    int n;
};

template <int R, int SEG>
__global__ void __launch_bounds__(256) k_gemv_bf16_multi(Segs S, const float *x, int in, int T)
{
    pdl_wait();
    pdl_trigger();
    extern __shared__ float4 xs[];
    const int nf4 = in >> 2;
    for (int t = 0; t < T; t++) stage_x_bf16(xs + (size_t)t * nf4, x + (size_t)t * in, in);
    __syncthreads();
    const int nch = in >> 3;
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int total = S.start[S.n];
    for (int r0 = warp * R; r0 < total; r0 += nwarps * R) {
        const uint16_t *pr[R];
        float *dst[R];
        int seg_rows[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            const int gr = min(r0 + r, total - 1);
            int sgi = 0;
            while (sgi + 1 < S.n && gr >= S.start[sgi + 1]) sgi++;
            const int lr = gr - S.start[sgi];
            pr[r] = S.W[sgi] + (size_t)lr * in;
            dst[r] = S.y[sgi] + lr;
            seg_rows[r] = S.rows[sgi];
        }
        for (int t = 0; t < T; t++) {
            float acc[R];
            bf16_rows_partial<R, SEG>(acc, pr, xs + (size_t)t * nf4, nch);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const float v = warp_sum(acc[r]);
                if (lane == 0 && r0 + r < total) dst[r][(size_t)t * seg_rows[r]] = v;
            }
        }
    }
}

// Logits with a fused argmax: key[t] = max over rows of (ordered float bits << 32 |
// ~row), so the largest logit wins and, among equal logits, the lowest row (the first
// maximum, as the CPU's argmax scan returns).
__device__ __forceinline__ unsigned long long argmax_pack(float v, int row)
{
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (uint32_t)row);
}

template <int R, int SEG>
__global__ void __launch_bounds__(256) k_gemv_bf16_argmax(float *y, unsigned long long *key,
                                                          const float *x, const uint16_t *W,
                                                          int in, int out, int T)
{
    pdl_wait();
    pdl_trigger();
    extern __shared__ float4 xs[];
    const int nf4 = in >> 2;
    for (int t = 0; t < T; t++) stage_x_bf16(xs + (size_t)t * nf4, x + (size_t)t * in, in);
    __syncthreads();
    const int nch = in >> 3;
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    unsigned long long best[4] = {0, 0, 0, 0};
    for (int r0 = warp * R; r0 < out; r0 += nwarps * R) {
        const uint16_t *pr[R];
#pragma unroll
        for (int r = 0; r < R; r++) pr[r] = W + (size_t)min(r0 + r, out - 1) * in;
        for (int t = 0; t < T; t++) {
            float acc[R];
            bf16_rows_partial<R, SEG>(acc, pr, xs + (size_t)t * nf4, nch);
#pragma unroll
            for (int r = 0; r < R; r++) {
                const float v = warp_sum(acc[r]);
                if (lane == 0 && r0 + r < out) {
                    if (y) y[(size_t)t * out + r0 + r] = v;
                    const unsigned long long k = argmax_pack(v, r0 + r);
                    if (v == v && k > best[t]) best[t] = k;
                }
            }
        }
    }
    if (lane == 0)
        for (int t = 0; t < T; t++)
            if (best[t]) atomicMax(key + t, best[t]);
}

__global__ void k_argmax_finish(int *next, const unsigned long long *key, int T)
{
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < T) next[t] = (int)(0xffffffffu - (uint32_t)(key[t] & 0xffffffffu));
}

static bool al16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// Batches of more than four tokens go to the tensor-core GEMM (k3_gemm_tc.cu), which reads
// each weight once per 128 tokens, on the two streams it keeps workspace for.
static bool use_gemm_tc(int in, int T, const float *x, cudaStream_t s)
{
    return T > 4 && in % 64 == 0 && al16(x) && (s == stream() || s == side_stream());
}

// key[t] = the packed first maximum of logits row t (lowest index among equal values; NaN
// never wins), as argmax_pack makes it. grid T, 1024 threads.
__global__ void k_rows_argmax(unsigned long long *key, const float *y, int out)
{
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    unsigned long long best = 0;
    for (int r = threadIdx.x; r < out; r += blockDim.x) {
        const float v = y[(size_t)t * out + r];
        const unsigned long long k = argmax_pack(v, r);
        if (v == v && k > best) best = k;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v > best ? v : best;
    }
    __shared__ unsigned long long red[32];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        best = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            best = v > best ? v : best;
        }
        if (threadIdx.x == 0) key[t] = best;
    }
}

// Keys of rows [v0, v0 + n) of a larger vocabulary: local row r becomes global row v0 + r
// (the low word holds 0xffffffff - row); an empty key (no finite logit) stays empty.
__global__ void k_key_offset(unsigned long long *key, int T, int v0)
{
    const int t = threadIdx.x;
    if (t >= T || !key[t]) return;
    const uint32_t lo = (uint32_t)(key[t] & 0xffffffffu) - (uint32_t)v0;
    key[t] = (key[t] & 0xffffffff00000000ull) | lo;
}

// The streamed GEMVs (k3_gemv_stream.cu) where the shape allows, on the library stream
// (work on the side stream, which runs beside the main stream's one-CTA-per-SM kernels,
// keeps the register-staged kernels); K3_GEMV_STREAM=0 in the environment selects the
// register-staged kernels everywhere.
static const bool g_gemv_stream = [] {
    const char *v = getenv("K3_GEMV_STREAM");
    return !(v && v[0] == '0');
}();

int grid_for(int rows, int rows_per_cta);
// CTAs for `rows` rows when one pass of a CTA covers rows_per_pass rows: one pass per CTA
// up to 8 CTAs per SM, grid-striding beyond that.
int grid_for(int rows, int rows_per_pass)
{
    int grid = (rows + rows_per_pass - 1) / rows_per_pass;
    const int cap = sm_count() * 8;
    if (grid > cap) grid = cap;
    return grid < 1 ? 1 : grid;
}

int gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out, int T,
              int accumulate, cudaStream_t s)
{
    if (out <= 0 || T <= 0) return K3D_OK;
    if (T <= 4 && g_gemv_stream && s == stream()) {
        float *ys[1] = {y};
        const int rows[1] = {out};
        if (gemv_stream_multi(1, &W, ys, rows, x, in, T, accumulate, s)) return check_launch("gemv bf16 stream");
    }
    if (use_gemm_tc(in, T, x, s) && al16(W)) return gemm_bf16_tc(1, &W, &y, &out, x, in, T, accumulate, 0, s);
    const bool fast = (in % 8) == 0 && al16(W) && (size_t)in * 4 * min(T, 4) <= 200 * 1024;
    if (!fast) {
        for (int t = 0; t < T; t++) {
            k_gemv_generic<uint16_t><<<grid_for(out, 8), 256, 0, s>>>(
                y + (size_t)t * out, x + (size_t)t * in, W, in, out, accumulate);
            note_launch();
        }
        return check_launch("gemv bf16 generic");
    }
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) {
        allow_smem(k_gemv_bf16<2, 7, 1>);
        allow_smem(k_gemv_bf16<2, 7, 4>);
        init |= dev_bit();
    }
    for (int t0 = 0; t0 < T; t0 += 4) {
        const int nt = min(4, T - t0);
        const size_t smem = (size_t)nt * in * sizeof(float);
        if (nt == 1)
            launch_pdl(k_gemv_bf16<2, 7, 1>, dim3(grid_for(out, 16)), dim3(256), smem, s, 
                y + (size_t)t0 * out, x + (size_t)t0 * in, W, in, out, 1, accumulate);
        else
            launch_pdl(k_gemv_bf16<2, 7, 4>, dim3(grid_for(out, 16)), dim3(256), smem, s, 
                y + (size_t)t0 * out, x + (size_t)t0 * in, W, in, out, nt, accumulate);
        note_launch();
    }
    return check_launch("gemv bf16");
}

int gemv_bf16_swiglu(float *act, const float *x, const uint16_t *Wg, const uint16_t *Wu,
                     int in, int inter, int T, cudaStream_t s)
{
    if (inter <= 0 || T <= 0) return K3D_OK;
    if (T <= 4 && g_gemv_stream && s == stream() && gemv_stream_swiglu(act, x, Wg, Wu, in, inter, T, s))
        return check_launch("gemv bf16 swiglu stream");
    if (use_gemm_tc(in, T, x, s) && al16(Wg) && al16(Wu)) {
        const uint16_t *Ws[2] = {Wg, Wu};
        float *Ys[2] = {act, act};
        const int rows[2] = {inter, inter};
        return gemm_bf16_tc(2, Ws, Ys, rows, x, in, T, 0, 1, s);
    }
    if ((in % 8) != 0 || !al16(Wg) || !al16(Wu) || (size_t)in * 4 * 4 > 200 * 1024)
        return fail(K3D_EINVAL, "swiglu gemv needs in %% 8 == 0 and aligned rows (in=%d)", in);
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) { allow_smem(k_gemv_bf16_swiglu<7>); init |= dev_bit(); }
    for (int t0 = 0; t0 < T; t0 += 4) {
        const int nt = min(4, T - t0);
        const size_t smem = (size_t)nt * in * sizeof(float);
        launch_pdl(k_gemv_bf16_swiglu<7>, dim3(grid_for(inter, 8)), dim3(256), smem, s, 
            act + (size_t)t0 * inter, x + (size_t)t0 * in, Wg, Wu, in, inter, nt);
        note_launch();
    }
    return check_launch("gemv bf16 swiglu");
}

const float *norm_to_scratch(const float *x, const NormIn &ni, int n, int rows, cudaStream_t s)
{
    float *xn = (float *)scratch((size_t)n * rows * sizeof(float), 0);
    if (!xn) return nullptr;
    if (rmsnorm(xn, x, ni.w, n, rows, ni.eps, s)) return nullptr;
    return xn;
}

int gemv_bf16_multi(int nseg, const uint16_t *const *W, float *const *y, const int *rows,
                    const float *x, int in, int T, cudaStream_t s, const NormIn *ni)
{
    if (nseg < 1 || nseg > 8 || T < 1)
        return fail(K3D_EINVAL, "multi-segment GEMV: %d segments, T=%d", nseg, T);
    if (T > 4) {
        if (ni) {
            x = norm_to_scratch(x, *ni, in, T, s);
            if (!x) return k3d_status();
        }
        if (!use_gemm_tc(in, T, x, s)) return fail(K3D_EINVAL, "multi-segment GEMV: T=%d needs in %% 64 == 0", T);
        return gemm_bf16_tc(nseg, W, y, rows, x, in, T, 0, 0, s);
    }
    if (g_gemv_stream && s == stream() && gemv_stream_multi(nseg, W, y, rows, x, in, T, 0, s, ni))
        return check_launch("gemv bf16 multi stream");
    if (ni) {
        x = norm_to_scratch(x, *ni, in, T, s);
        if (!x) return k3d_status();
    }
    Segs S;
    S.n = nseg;
    S.start[0] = 0;
    for (int i = 0; i < nseg; i++) {
        if (!al16(W[i])) return fail(K3D_EINVAL, "multi-segment GEMV: unaligned matrix");
        S.W[i] = W[i];
        S.y[i] = y[i];
        S.rows[i] = rows[i];
        S.start[i + 1] = S.start[i] + rows[i];
    }
    if ((in % 8) != 0 || (size_t)in * 4 * T > 200 * 1024)
        return fail(K3D_EINVAL, "multi-segment GEMV: in=%d", in);
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) { allow_smem(k_gemv_bf16_multi<2, 7>); init |= dev_bit(); }
    launch_pdl(k_gemv_bf16_multi<2, 7>, dim3(grid_for(S.start[nseg], 16)), dim3(256), (size_t)T * in * 4, s, S, x, in, T);
    note_launch();
    return check_launch("gemv bf16 multi");
}

// The LM head's argmax keys: key[t] = argmax_pack of the first maximum of logits row t
// (local rows 0..out-1); y receives the logits when non-null.
int lm_head_keys(float *y, unsigned long long *key, const float *x, const uint16_t *W, int in, int out, int T,
                 cudaStream_t s, const NormIn *ni)
{
    if (T < 1 || (in % 8) != 0 || !al16(W))
        return fail(K3D_EINVAL, "lm head: T=%d in=%d", T, in);
    if (T > 4) {
        // a batch: logits by the tensor-core GEMM, then one argmax per row
        if (ni) {
            x = norm_to_scratch(x, *ni, in, T, s);
            if (!x) return k3d_status();
        }
        if (!use_gemm_tc(in, T, x, s)) return fail(K3D_EINVAL, "lm head: T=%d needs in %% 64 == 0", T);
        if (!y) {
            y = (float *)scratch((size_t)T * out * sizeof(float), 5);
            if (!y) return k3d_status();
        }
        K3_TRY(gemm_bf16_tc(1, &W, &y, &out, x, in, T, 0, 0, s));
        launch_pdl(k_rows_argmax, dim3(T), dim3(1024), 0, s, key, (const float *)y, out);
        note_launch();
        return check_launch("lm head rows argmax");
    }
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) { allow_smem(k_gemv_bf16_argmax<2, 7>); init |= dev_bit(); }
    K3_TRY(cudaMemsetAsync(key, 0, (size_t)T * sizeof(unsigned long long), s) == cudaSuccess
               ? K3D_OK : fail(K3D_ECUDA, "argmax key reset"));
    if (g_gemv_stream && s == stream() && gemv_stream_argmax(y, key, x, W, in, out, T, s, ni))
        return check_launch("lm head argmax stream");
    if (ni) {
        x = norm_to_scratch(x, *ni, in, T, s);
        if (!x) return k3d_status();
    }
    launch_pdl(k_gemv_bf16_argmax<2, 7>, dim3(grid_for(out, 16)), dim3(256), (size_t)T * in * 4, s, y, key, x, W, in, out, T);
    note_launch();
    return check_launch("lm head argmax");
}

int argmax_finish(int *next, const unsigned long long *key, int T, cudaStream_t s)
{
    launch_pdl(k_argmax_finish, dim3((T + 255) / 256), dim3(256), 0, s, next, key, T);
    note_launch();
    return check_launch("argmax finish");
}

int key_offset(unsigned long long *key, int T, int v0, cudaStream_t s)
{
    if (T > 1024) return fail(K3D_EINVAL, "key offset: T=%d", T);
    k_key_offset<<<1, 1024, 0, s>>>(key, T, v0);
    note_launch();
    return check_launch("argmax key offset");
}

int gemv_bf16_argmax(float *y, unsigned long long *key, int *next, const float *x,
                     const uint16_t *W, int in, int out, int T, cudaStream_t s, const NormIn *ni)
{
    K3_TRY(lm_head_keys(y, key, x, W, in, out, T, s, ni));
    return argmax_finish(next, key, T, s);
}

int gemv_tagged(float *y, const float *x, const void *W, int wdt, int in, int out, cudaStream_t s)
{
    if (wdt == K3_WBF16) return gemv_ref_bf16(y, x, (const uint16_t *)W, in, out, 1, 0, s);
    if (wdt == K3_WF32) return gemv_ref_f32(y, x, (const float *)W, in, out, 1, 0, s);
    return fail(K3D_EUNSUPPORTED, "weight tag %d (the int8 draft format is not served here)", wdt);
}

int gemv_f32(float *y, const float *x, const float *W, int in, int out, cudaStream_t s)
{
    if (out <= 0) return K3D_OK;
    const bool fast = (in % 4) == 0 && al16(W) && (size_t)in * 4 <= 200 * 1024;
    if (!fast) {
        k_gemv_generic<float><<<grid_for(out, 8), 256, 0, s>>>(y, x, W, in, out, 0);
        note_launch();
        return check_launch("gemv f32 generic");
    }
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) { allow_smem(k_gemv_f32<2, 4>); init |= dev_bit(); }
    k_gemv_f32<2, 4><<<grid_for(out, 16), 256, (size_t)in * sizeof(float), s>>>(y, x, W, in, out);
    note_launch();
    return check_launch("gemv f32");
}

}  // namespace k3

using namespace k3;

extern "C" {

void k3_matmul(float *y, const float *x, const float *W, int in, int out)
{
    if (ensure_ctx()) return;
    if (in <= 0 || out <= 0) return;
    Stage st;
    const float *Wd = (const float *)st.weight(W, (size_t)in * out * sizeof(float));
    const float *X = (const float *)st.in(x, (size_t)in * sizeof(float));
    float *Y = (float *)st.out(y, (size_t)out * sizeof(float));
    if (st.err) return;
    if (gemv_ref_f32(Y, X, Wd, in, out, 1, 0, stream())) return;
    st.finish();
}

void k3_matmul_bf16(float *y, const float *x, const uint16_t *W, int in, int out)
{
    if (ensure_ctx()) return;
    if (in <= 0 || out <= 0) return;
    Stage st;
    const uint16_t *Wd = (const uint16_t *)st.weight(W, (size_t)in * out * sizeof(uint16_t));
    const float *X = (const float *)st.in(x, (size_t)in * sizeof(float));
    float *Y = (float *)st.out(y, (size_t)out * sizeof(float));
    if (st.err) return;
    if (gemv_ref_bf16(Y, X, Wd, in, out, 1, 0, stream())) return;
    st.finish();
}

void k3_matmul_q8(float *y, const float *x, const void *W, int in, int out)
{
    (void)y; (void)x; (void)W; (void)in; (void)out;
    if (ensure_ctx()) return;
    fail(K3D_EUNSUPPORTED, "k3_matmul_q8: the int8 draft-model format is not served here");
}

int k3d_gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out, int T,
                  int accumulate)
{
    K3_TRY(ensure_ctx());
    if (!y || !x || !W) return fail(K3D_EINVAL, "k3d_gemv_bf16 null pointer");
    return gemv_bf16(y, x, W, in, out, T, accumulate, stream());
}

}  // extern "C"
