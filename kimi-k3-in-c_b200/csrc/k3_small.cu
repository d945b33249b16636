// k3_small.cu -- the elementwise and reduction ops of the decode path:
//   k3_rmsnorm    k3_ops.c:94-102     (double sum of squares, eps inside the sqrt)
//   k3_situ_glu   k3_ops.c:110-123    (sigmoid takes the UNCAPPED gate)
//   k3_shortconv  k3_ops.c:133-165    (causal depthwise conv, SiLU fused, state in place)
//   k3_kda_decay  k3_ops.c:168-183    (A_log indexed per head)
//   k3_attn_res   k3_ops.c:481-512    (keys normalised, values raw)
//   k3d_silu_mul  SwiGLU activation of the benchmark shapes
#include "k3_common.cuh"
#include "k3_ops.cuh"

namespace k3 {

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ double block_sum_d(double v, double *red)
{
    v = warp_sum_d(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    double s = 0.0;
    if (threadIdx.x < 32) {
        s = (lane < nw) ? red[lane] : 0.0;
        s = warp_sum_d(s);
        if (lane == 0) red[0] = s;
    }
    __syncthreads();
    return red[0];
}

// one CTA per row, the row and the weights held in registers: x and w are loaded together
// up front (one memory round trip), the same per-thread order as k_rmsnorm below.
template <int PER>
__global__ void __launch_bounds__(1024) k_rmsnorm_reg(float *y, const float *x, const float *w,
                                                      int n, float eps)
{
    pdl_wait();
    pdl_trigger();
    __shared__ double red[32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *yr = y + (size_t)blockIdx.x * n;
    float xv[PER], wv[PER];
#pragma unroll
    for (int k = 0; k < PER; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        xv[k] = i < n ? xr[i] : 0.0f;
        wv[k] = i < n ? __ldg(w + i) : 0.0f;
    }
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < PER; k++) {
        const double v = (double)xv[k];
        ss = fma(v, v, ss);
    }
    ss = block_sum_d(ss, red);
    const float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
#pragma unroll
    for (int k = 0; k < PER; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < n) yr[i] = __fmul_rn(__fmul_rn(wv[k], xv[k]), inv);
    }
}

// one CTA per row (any n)
__global__ void k_rmsnorm(float *y, const float *x, const float *w, int n, float eps)
{
    pdl_wait();
    pdl_trigger();
    __shared__ double red[32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *yr = y + (size_t)blockIdx.x * n;
    double ss = 0.0;
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double v = (double)xr[i];
        ss = fma(v, v, ss);
    }
    ss = block_sum_d(ss, red);
    const float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        yr[i] = __fmul_rn(__fmul_rn(w[i], xr[i]), inv);
}

__global__ void k_situ_glu(float *y, const float *x, int n, int rows, float b1, float b2)
{
    const size_t total = (size_t)n * rows;
    for (size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x; k < total;
         k += (size_t)gridDim.x * blockDim.x) {
        const size_t r = k / n, i = k % n;
        const float g = x[r * 2 * n + i];
        const float up = x[r * 2 * n + n + i];
        const float a = b1 * tanhf(g / b1) * sigmoid_f(g);
        const float u = b2 * tanhf(up / b2);
        y[r * n + i] = a * u;
    }
}

__global__ void k_silu_mul(float *y, const float *gu, int n, int rows)
{
    const size_t total = (size_t)n * rows;
    for (size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x; k < total;
         k += (size_t)gridDim.x * blockDim.x) {
        const size_t r = k / n, i = k % n;
        const float g = gu[r * 2 * n + i];
        const float u = gu[r * 2 * n + n + i];
        y[r * n + i] = silu_f(g) * u;
    }
}

// thread per channel; history kept in registers-by-loop (k <= 16)
__global__ void k_shortconv(float *y, const float *x, const float *w, float *state,
                            int channels, int k, int T)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= channels) return;
    const int hist = k - 1;
    float buf[15];
    for (int j = 0; j < hist; j++) buf[j] = state ? state[(size_t)c * hist + j] : 0.f;
    for (int t = 0; t < T; t++) {
        const float cur = x[(size_t)t * channels + c];
        float acc = w[(size_t)c * k + hist] * cur;
        for (int j = 0; j < hist; j++) acc += w[(size_t)c * k + j] * buf[j];
        for (int j = 0; j + 1 < hist; j++) buf[j] = buf[j + 1];
        if (hist > 0) buf[hist - 1] = cur;
        y[(size_t)t * channels + c] = acc * sigmoid_f(acc);
    }
    if (state)
        for (int j = 0; j < hist; j++) state[(size_t)c * hist + j] = buf[j];
}

__global__ void k_kda_decay(float *g, float *alpha, const float *z, const float *A_log,
                            const float *dt_bias, int H, int D, float lb)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= H * D) return;
    const int h = i / D;
    const float a = expf(A_log[h]);
    const float u = a * (z[i] + dt_bias[i]);
    const float gi = lb * sigmoid_f(u);
    g[i] = gi;
    alpha[i] = expf(gi);
}

// single CTA: nsrc sources of width n
__global__ void k_attn_res(float *out, const float *src, const float *fold, int nsrc, int n,
                           float eps)
{
    extern __shared__ float sc[];   // [nsrc]
    __shared__ double red[32];
    for (int s = 0; s < nsrc; s++) {
        const float *v = src + (size_t)s * n;
        double ss = 0.0;
        for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fma((double)v[i], (double)v[i], ss);
        ss = block_sum_d(ss, red);
        const float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
        double acc = 0.0;
        for (int i = threadIdx.x; i < n; i += blockDim.x)
            acc = fma((double)__fmul_rn(v[i], inv), (double)fold[i], acc);
        acc = block_sum_d(acc, red);
        if (threadIdx.x == 0) sc[s] = (float)acc;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float m = sc[0];
        for (int s = 1; s < nsrc; s++) if (sc[s] > m) m = sc[s];
        double z = 0.0;
        for (int s = 0; s < nsrc; s++) { sc[s] = expf(sc[s] - m); z += sc[s]; }
        for (int s = 0; s < nsrc; s++) sc[s] = (float)(sc[s] / z);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float o = 0.f;
        for (int s = 0; s < nsrc; s++) o = __fadd_rn(o, __fmul_rn(sc[s], src[(size_t)s * n + i]));
        out[i] = o;
    }
}

static int blocks_for(size_t n, int threads)
{
    size_t b = (n + threads - 1) / threads;
    const size_t cap = (size_t)sm_count() * 16;
    if (b > cap) b = cap;
    return b < 1 ? 1 : (int)b;
}

int rmsnorm(float *y, const float *x, const float *w, int n, int rows, float eps, cudaStream_t s)
{
    if (rows <= 0 || n <= 0) return K3D_OK;
    if (n > 4096 && n <= 8192)
        launch_pdl(k_rmsnorm_reg<8>, dim3(rows), dim3(1024), 0, s, y, x, w, n, eps);
    else
        launch_pdl(k_rmsnorm, dim3(rows), dim3(n >= 1024 ? 1024 : 256), 0, s, y, x, w, n, eps);
    note_launch();
    return check_launch("rmsnorm");
}

int situ_glu(float *y, const float *x, int n, int rows, float b1, float b2, cudaStream_t s)
{
    if (rows <= 0 || n <= 0) return K3D_OK;
    k_situ_glu<<<blocks_for((size_t)n * rows, 256), 256, 0, s>>>(y, x, n, rows, b1, b2);
    note_launch();
    return check_launch("situ_glu");
}

int silu_mul(float *y, const float *gu, int n, int rows, cudaStream_t s)
{
    if (rows <= 0 || n <= 0) return K3D_OK;
    k_silu_mul<<<blocks_for((size_t)n * rows, 256), 256, 0, s>>>(y, gu, n, rows);
    note_launch();
    return check_launch("silu_mul");
}

int shortconv(float *y, const float *x, const float *w, float *state, int channels, int k,
              int T, cudaStream_t s)
{
    if (k < 1 || k > 16) return fail(K3D_EINVAL, "shortconv k=%d outside 1..16", k);
    if (channels <= 0 || T <= 0) return K3D_OK;
    k_shortconv<<<(channels + 127) / 128, 128, 0, s>>>(y, x, w, state, channels, k, T);
    note_launch();
    return check_launch("shortconv");
}

int kda_decay(float *g, float *alpha, const float *z, const float *A_log, const float *dt_bias,
              int H, int D, float lb, cudaStream_t s)
{
    if (H <= 0 || D <= 0) return K3D_OK;
    k_kda_decay<<<(H * D + 255) / 256, 256, 0, s>>>(g, alpha, z, A_log, dt_bias, H, D, lb);
    note_launch();
    return check_launch("kda_decay");
}

int attn_res(float *out, const float *src, const float *fold, int nsrc, int n, float eps,
             cudaStream_t s)
{
    if (nsrc <= 0 || n <= 0) return K3D_OK;
    k_attn_res<<<1, 1024, (size_t)nsrc * sizeof(float), s>>>(out, src, fold, nsrc, n, eps);
    note_launch();
    return check_launch("attn_res");
}

}  // namespace k3

using namespace k3;

extern "C" {

void k3_rmsnorm(float *y, const float *x, const float *w, int n, float eps)
{
    if (ensure_ctx() || n <= 0) return;
    Stage st;
    const float *W = (const float *)st.weight(w, (size_t)n * sizeof(float));
    const float *X = (const float *)st.in(x, (size_t)n * sizeof(float));
    // in-place use (y == x) is allowed, as on the CPU
    float *Y = (y == x && !is_device_ptr(y)) ? (float *)st.out(y, (size_t)n * sizeof(float))
                                            : (float *)st.out(y, (size_t)n * sizeof(float));
    if (st.err) return;
    if (rmsnorm(Y, X, W, n, 1, eps, stream())) return;
    st.finish();
}

void k3_situ_glu(float *y, const float *x, int n, float b1, float b2)
{
    if (ensure_ctx() || n <= 0) return;
    Stage st;
    const float *X = (const float *)st.in(x, (size_t)2 * n * sizeof(float));
    float *Y = (float *)st.out(y, (size_t)n * sizeof(float));
    if (st.err) return;
    if (situ_glu(Y, X, n, 1, b1, b2, stream())) return;
    st.finish();
}

void k3_shortconv(float *y, const float *x, const float *w, float *state, int channels, int k,
                  int T)
{
    if (ensure_ctx() || channels <= 0 || T <= 0) return;
    Stage st;
    const float *Wd = (const float *)st.weight(w, (size_t)channels * k * sizeof(float));
    const float *X = (const float *)st.in(x, (size_t)T * channels * sizeof(float));
    float *S = (state && k > 1) ? (float *)st.inout(state, (size_t)channels * (k - 1) * sizeof(float))
                                : nullptr;
    float *Y = (float *)st.out(y, (size_t)T * channels * sizeof(float));
    if (st.err) return;
    if (shortconv(Y, X, Wd, S, channels, k, T, stream())) return;
    st.finish();
}

void k3_kda_decay(float *g, float *alpha, const float *z, const float *A_log,
                  const float *dt_bias, int H, int D, float lb)
{
    if (ensure_ctx() || H <= 0 || D <= 0) return;
    Stage st;
    const float *Z = (const float *)st.in(z, (size_t)H * D * sizeof(float));
    const float *A = (const float *)st.weight(A_log, (size_t)H * sizeof(float));
    const float *B = (const float *)st.weight(dt_bias, (size_t)H * D * sizeof(float));
    float *G = (float *)st.out(g, (size_t)H * D * sizeof(float));
    float *AL = (float *)st.out(alpha, (size_t)H * D * sizeof(float));
    if (st.err) return;
    if (kda_decay(G, AL, Z, A, B, H, D, lb, stream())) return;
    st.finish();
}

void k3_attn_res(float *out, const float *src, const float *fold, int nsrc, int n, float eps)
{
    if (ensure_ctx() || nsrc <= 0 || n <= 0) return;
    Stage st;
    const float *S = (const float *)st.in(src, (size_t)nsrc * n * sizeof(float));
    const float *F = (const float *)st.in(fold, (size_t)n * sizeof(float));
    float *O = (float *)st.out(out, (size_t)n * sizeof(float));
    if (st.err) return;
    if (attn_res(O, S, F, nsrc, n, eps, stream())) return;
    st.finish();
}

int k3d_rmsnorm(float *y, const float *x, const float *w, int n, int rows, float eps)
{
    K3_TRY(ensure_ctx());
    if (!y || !x || !w) return fail(K3D_EINVAL, "k3d_rmsnorm null pointer");
    return rmsnorm(y, x, w, n, rows, eps, stream());
}

int k3d_silu_mul(float *y, const float *gu, int n, int rows)
{
    K3_TRY(ensure_ctx());
    if (!y || !gu) return fail(K3D_EINVAL, "k3d_silu_mul null pointer");
    return silu_mul(y, gu, n, rows, stream());
}

}  // extern "C"
