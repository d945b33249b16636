// k3_router.cu -- MoE router with indices and weights bit-identical to k3_router
// (k3_ops.c:419-478).
//
// WHAT THE CPU COMPUTES, per expert e:
//     acc = 0.0; for i in 0..hidden-1: acc += (double)W[e][i] * (double)x[i]   (sequential)
//     score = 1.0f / (1.0f + expf(-(float)acc)),   choice = score + bias[e]
//   then top-k by repeated strict-greater max (lowest index wins ties, taken entries
//   become -inf), weights = unbiased scores, optional renorm in double, * routed_scale.
//
// HOW THE GPU MATCHES IT WITHOUT A 7168-LONG SERIAL CHAIN PER EXPERT
//   Every product W*x is exact in double (24 + 24 significant bits < 53), so the only
//   rounding in the CPU sum is in its additions. Let s_k be the exact prefix sums and
//   A = sum |p_i|. The sequential double sum differs from the exact sum by at most
//   u * sum_k |s^_k| <= u * (sum_k |s_k| + n * gamma_n * A), u = 2^-53.
//   A warp computes, in one coalesced pass over the row, (1) the exact sum to ~2^-100
//   relative (TwoSum accumulation per lane, then a TwoSum tree) and (2) sum_k |s_k| from
//   the prefix sums in the CPU's element order (a warp scan per round of 32 chunks gives
//   each chunk's starting prefix). If the whole interval [S - bound, S + bound] rounds
//   to one float, that float IS (float)acc of the CPU. Otherwise (about one expert in
//   10^5 at the benchmark shapes; k3d_router_fallbacks counts them) lane 0 runs the
//   CPU's exact sequential loop for that expert.
//   The sigmoid uses k3_expf (glibc's expf restated, bit-identical), and all float
//   operations use explicit round-to-nearest intrinsics so nothing is contracted.
#include "k3_common.cuh"
#include "k3_expf.h"
#include "k3_ops.cuh"

namespace k3 {

template <typename WT> __device__ __forceinline__ double wval(const WT *p, int i);
template <> __device__ __forceinline__ double wval<float>(const float *p, int i)
{
    return (double)__ldg(p + i);
}
template <> __device__ __forceinline__ double wval<uint16_t>(const uint16_t *p, int i)
{
    return (double)__uint_as_float((uint32_t)__ldg(p + i) << 16);
}

__device__ __forceinline__ void two_sum(double a, double b, double &s, double &e)
{
    s = __dadd_rn(a, b);
    const double bb = __dsub_rn(s, a);
    e = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
}

// Counts experts whose logit needed the sequential fallback (read by k3d_router_fallbacks).
__device__ unsigned long long k3_router_fallbacks;

template <typename WT> struct Chunk;
template <> struct Chunk<uint16_t> {   // 8 bf16 = 16 bytes
    __device__ static void load(const uint16_t *row, int c, double w[8])
    {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(row) + c);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[2 * i] = (double)__uint_as_float(u[i] << 16);
            w[2 * i + 1] = (double)__uint_as_float(u[i] & 0xffff0000u);
        }
    }
};
template <> struct Chunk<float> {      // 8 fp32 = 32 bytes
    __device__ static void load(const float *row, int c, double w[8])
    {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(row) + 2 * c);
        const float4 b = __ldg(reinterpret_cast<const float4 *>(row) + 2 * c + 1);
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    }
};

// One warp per (token, expert): writes score and choice. Lane l owns 8-element chunks
// l, l+32, ...; one pass computes (1) the exact total with TwoSum accumulation, (2)
// sum |p|, and (3) sum over k of |prefix sum k| in the CPU's element order, using a warp
// scan per round of 32 chunks for the prefix at each chunk start.
// Requires hidden % 8 == 0 and 16-byte aligned rows and x.
template <typename WT>
__global__ void __launch_bounds__(256) k_router_scores(float *score, float *choice,
                                                       const float *x, const WT *W,
                                                       const float *bias, int hidden,
                                                       int n_experts)
{
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int t = blockIdx.y;
    if (e >= n_experts) return;
    const float *xt = x + (size_t)t * hidden;
    const WT *row = W + (size_t)e * hidden;
    const int nchunk = hidden >> 3;
    double hs = 0.0, ls = 0.0, A = 0.0, absum = 0.0, run = 0.0;
    for (int base = 0; base < nchunk; base += 32) {
        const int c = base + lane;
        double p[8];
        if (c < nchunk) {
            double w[8];
            Chunk<WT>::load(row, c, w);
            const float4 xa = __ldg(reinterpret_cast<const float4 *>(xt) + 2 * c);
            const float4 xb = __ldg(reinterpret_cast<const float4 *>(xt) + 2 * c + 1);
            const double xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int i = 0; i < 8; i++) p[i] = __dmul_rn(w[i], xv[i]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) p[i] = 0.0;
        }
        double cs = 0.0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            // exact accumulation of the lane's products
            const double s1 = __dadd_rn(hs, p[i]);
            const double bb = __dsub_rn(s1, hs);
            ls = __dadd_rn(ls, __dadd_rn(__dsub_rn(hs, __dsub_rn(s1, bb)), __dsub_rn(p[i], bb)));
            hs = s1;
            A = __dadd_rn(A, fabs(p[i]));
            cs = __dadd_rn(cs, p[i]);
        }
        // prefix at this chunk's start: run + exclusive scan of chunk sums
        double incl = cs;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl = __dadd_rn(incl, v);
        }
        double pre = __dadd_rn(run, __dsub_rn(incl, cs));
#pragma unroll
        for (int i = 0; i < 8; i++) {
            pre = __dadd_rn(pre, p[i]);
            absum = __dadd_rn(absum, fabs(pre));
        }
        run = __dadd_rn(run, __shfl_sync(0xffffffffu, incl, 31));
    }
    // TwoSum tree over the lanes' (hs, ls)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const double oh = __shfl_xor_sync(0xffffffffu, hs, o);
        const double ol = __shfl_xor_sync(0xffffffffu, ls, o);
        double sum, err;
        two_sum(hs, oh, sum, err);
        const double low = __dadd_rn(__dadd_rn(ls, ol), err);
        double s2, e2;
        two_sum(sum, low, s2, e2);
        hs = s2;
        ls = e2;
    }
    const double total = hs;
    A = warp_sum_d(A);
    const double R = warp_sum_d(absum);

    if (lane == 0) {
        const double u = 0x1p-53;
        const double n = (double)hidden;
        const double gam = n * u / (1.0 - n * u);
        const double bound = (u * (R + 4.0 * n * gam * A) + 8.0 * u * fabs(total) +
                              64.0 * n * n * u * u * A) * (1.0 + 0x1p-20) + 0x1p-1074;
        const float flo = (float)(total - bound);
        const float fhi = (float)(total + bound);
        float logit;
        if (flo == fhi) {
            logit = flo;
        } else {
            // ambiguous: the CPU's exact sequential loop (k3_ops.c:449-450)
            double acc = 0.0;
            for (int i = 0; i < hidden; i++) {
                const double wv = (sizeof(WT) == 2)
                    ? (double)__uint_as_float((uint32_t)__ldg((const uint16_t *)row + i) << 16)
                    : (double)__ldg((const float *)row + i);
                acc = __dadd_rn(acc, __dmul_rn(wv, (double)__ldg(xt + i)));
            }
            logit = (float)acc;
            atomicAdd(&k3_router_fallbacks, 1ull);
        }
        const float sc = __fdiv_rn(1.0f, __fadd_rn(1.0f, k3_expf(-logit)));
        score[(size_t)t * n_experts + e] = sc;
        choice[(size_t)t * n_experts + e] = bias ? __fadd_rn(sc, __ldg(bias + e)) : sc;
    }
}

// Any shape: one warp per (token, expert), lanes over contiguous segments.
template <typename WT>
__global__ void __launch_bounds__(256) k_router_scores_generic(float *score, float *choice,
                                                               const float *x, const WT *W,
                                                               const float *bias, int hidden,
                                                               int n_experts)
{
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int t = blockIdx.y;
    if (e >= n_experts) return;
    const float *xt = x + (size_t)t * hidden;
    const WT *row = W + (size_t)e * hidden;
    const int seg = (hidden + 31) >> 5;
    const int lo = min(hidden, lane * seg);
    const int hi = min(hidden, lo + seg);
    double s = 0.0, c = 0.0, a = 0.0;
    for (int i = lo; i < hi; i++) {
        const double p = __dmul_rn(wval<WT>(row, i), (double)__ldg(xt + i));
        const double tt = __dadd_rn(s, p);
        if (fabs(s) >= fabs(p)) c = __dadd_rn(c, __dadd_rn(__dsub_rn(s, tt), p));
        else c = __dadd_rn(c, __dadd_rn(__dsub_rn(p, tt), s));
        s = tt;
        a = __dadd_rn(a, fabs(p));
    }
    const double lane_tot = __dadd_rn(s, c);
    double incl = lane_tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = __dadd_rn(incl, v);
    }
    const double excl = __dsub_rn(incl, lane_tot);
    double hs = s, ls = c;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const double oh = __shfl_xor_sync(0xffffffffu, hs, o);
        const double ol = __shfl_xor_sync(0xffffffffu, ls, o);
        double sum, err;
        two_sum(hs, oh, sum, err);
        const double low = __dadd_rn(__dadd_rn(ls, ol), err);
        double s2, e2;
        two_sum(sum, low, s2, e2);
        hs = s2;
        ls = e2;
    }
    const double total = hs;
    const double A = warp_sum_d(a);
    double run = excl, absum = 0.0;
    for (int i = lo; i < hi; i++) {
        const double p = __dmul_rn(wval<WT>(row, i), (double)__ldg(xt + i));
        run = __dadd_rn(run, p);
        absum = __dadd_rn(absum, fabs(run));
    }
    const double R = warp_sum_d(absum);
    if (lane == 0) {
        const double u = 0x1p-53;
        const double n = (double)hidden;
        const double gam = n * u / (1.0 - n * u);
        const double bound = (u * (R + 4.0 * n * gam * A) + 8.0 * u * fabs(total) +
                              64.0 * n * n * u * u * A) * (1.0 + 0x1p-20) + 0x1p-1074;
        const float flo = (float)(total - bound);
        const float fhi = (float)(total + bound);
        float logit;
        if (flo == fhi) {
            logit = flo;
        } else {
            double acc = 0.0;
            for (int i = 0; i < hidden; i++)
                acc = __dadd_rn(acc, __dmul_rn(wval<WT>(row, i), (double)__ldg(xt + i)));
            logit = (float)acc;
            atomicAdd(&k3_router_fallbacks, 1ull);
        }
        const float sc = __fdiv_rn(1.0f, __fadd_rn(1.0f, k3_expf(-logit)));
        score[(size_t)t * n_experts + e] = sc;
        choice[(size_t)t * n_experts + e] = bias ? __fadd_rn(sc, __ldg(bias + e)) : sc;
    }
}

// One warp per token: top-k by repeated max, renorm, scale (k3_ops.c:459-475).
__global__ void k_router_topk(int *idx, float *wout, float *choice, const float *score,
                              int n_experts, int topk, int renorm, float routed_scale,
                              int idx_stride)
{
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x;
    float *ch = choice + (size_t)t * n_experts;
    const float *scr = score + (size_t)t * n_experts;
    __shared__ float wsel[K3_MAX_TOPK];
    __shared__ int isel[K3_MAX_TOPK];
    for (int j = 0; j < topk; j++) {
        float bv = -INFINITY;
        int best = -1;
        for (int e = lane; e < n_experts; e += 32) {
            const float v = ch[e];
            if (v > bv) { bv = v; best = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int ob = __shfl_xor_sync(0xffffffffu, best, o);
            // larger value wins; on equal values the lower index (the one a forward
            // scan meets first) wins; -1 (nothing found) loses to anything found
            const bool take = (ob >= 0) && (best < 0 || ov > bv || (ov == bv && ob < best));
            if (take) { bv = ov; best = ob; }
        }
        if (lane == 0) {
            if (best < 0) { isel[j] = 0; wsel[j] = 0.0f; }
            else { isel[j] = best; wsel[j] = scr[best]; ch[best] = -INFINITY; }
        }
        __syncwarp();
    }
    if (lane == 0) {
        if (renorm && topk > 1) {
            double s = 0.0;
            for (int j = 0; j < topk; j++) s = __dadd_rn(s, (double)wsel[j]);
            const float inv = (float)__ddiv_rn(1.0, __dadd_rn(s, 1e-20));
            for (int j = 0; j < topk; j++) wsel[j] = __fmul_rn(wsel[j], inv);
        }
        for (int j = 0; j < topk; j++) {
            idx[(size_t)t * idx_stride + j] = isel[j];
            wout[(size_t)t * idx_stride + j] = __fmul_rn(wsel[j], routed_scale);
        }
    }
}

size_t router_ws_bytes(int T, int n_experts)
{
    return 2 * (size_t)T * n_experts * sizeof(float) + 256;
}

template <typename WT>
static int router_launch(int *idx, float *w, const float *x, const WT *W, const float *bias,
                         int T, int hidden, int n_experts, int topk, int renorm,
                         float routed_scale, void *ws, cudaStream_t s)
{
    if (topk < 1 || topk > K3_MAX_TOPK)
        return fail(K3D_EBOUND, "router topk=%d outside 1..%d", topk, K3_MAX_TOPK);
    if (n_experts < 1 || hidden < 1 || T < 1)
        return fail(K3D_EINVAL, "router hidden=%d n_experts=%d T=%d", hidden, n_experts, T);
    float *score = (float *)ws;
    float *choice = score + (size_t)T * n_experts;
    dim3 grid((n_experts + 7) / 8, T);
    const bool vec = (hidden % 8) == 0 && (((uintptr_t)W | (uintptr_t)x) & 15u) == 0;
    if (vec) k_router_scores<WT><<<grid, 256, 0, s>>>(score, choice, x, W, bias, hidden, n_experts);
    else k_router_scores_generic<WT><<<grid, 256, 0, s>>>(score, choice, x, W, bias, hidden, n_experts);
    k_router_topk<<<T, 32, 0, s>>>(idx, w, choice, score, n_experts, topk, renorm,
                                   routed_scale, topk);
    note_launch(2);
    return check_launch("router");
}

int router_f32(int *idx, float *w, const float *x, const float *W, const float *bias,
               int T, int hidden, int n_experts, int topk, int renorm, float routed_scale,
               void *ws, cudaStream_t s)
{
    return router_launch<float>(idx, w, x, W, bias, T, hidden, n_experts, topk, renorm,
                                routed_scale, ws, s);
}

int router_bf16(int *idx, float *w, const float *x, const uint16_t *W, const float *bias,
                int T, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                void *ws, cudaStream_t s)
{
    return router_launch<uint16_t>(idx, w, x, W, bias, T, hidden, n_experts, topk, renorm,
                                   routed_scale, ws, s);
}

// Fixed scratch of k3d_router_bf16_noalloc: scores then choice keys, each up to
// K3D_ROUTER_NOALLOC_MAX floats. Every element a call reads it has first written, so
// nothing needs clearing between calls.
static __device__ __align__(256) float g_router_noalloc_ws[2 * K3D_ROUTER_NOALLOC_MAX];
static const int kMaxDevices = 64;

}  // namespace k3

using namespace k3;

extern "C" {

void k3_router(int *idx, float *w, const float *x, const float *W, const float *bias,
               int hidden, int n_experts, int topk, int renorm, float routed_scale)
{
    if (ensure_ctx()) return;
    if (topk < 1 || topk > K3_MAX_TOPK) {
        fail(K3D_EBOUND, "k3_router topk=%d outside 1..%d", topk, K3_MAX_TOPK);
        return;
    }
    Stage st;
    const float *Wd = (const float *)st.weight(W, (size_t)n_experts * hidden * sizeof(float));
    const float *Bd = bias ? (const float *)st.weight(bias, (size_t)n_experts * sizeof(float))
                           : nullptr;
    const float *X = (const float *)st.in(x, (size_t)hidden * sizeof(float));
    int *I = (int *)st.out(idx, (size_t)topk * sizeof(int));
    float *Wt = (float *)st.out(w, (size_t)topk * sizeof(float));
    if (st.err) return;
    void *ws = scratch(router_ws_bytes(1, n_experts), 1);
    if (!ws) return;
    if (router_f32(I, Wt, X, Wd, Bd, 1, hidden, n_experts, topk, renorm, routed_scale, ws,
                   stream()))
        return;
    st.finish();
}

long long k3d_router_fallbacks(void)
{
    if (ensure_ctx()) return -1;
    unsigned long long v = 0;
    cudaMemcpyFromSymbol(&v, k3_router_fallbacks, sizeof v);
    return (long long)v;
}

int k3d_router_bf16(int *idx, float *w, const float *x, const uint16_t *W, const float *bias,
                    int T, int hidden, int n_experts, int topk, int renorm, float routed_scale)
{
    K3_TRY(ensure_ctx());
    if (!idx || !w || !x || !W) return fail(K3D_EINVAL, "k3d_router_bf16 null pointer");
    void *ws = scratch(router_ws_bytes(T, n_experts), 1);
    if (!ws) return k3d_status();
    return router_bf16(idx, w, x, W, bias, T, hidden, n_experts, topk, renorm, routed_scale,
                       ws, stream());
}

int k3d_router_bf16_noalloc(int *idx, float *w, const float *x, const uint16_t *W,
                            const float *bias, int T, int hidden, int n_experts, int topk,
                            int renorm, float routed_scale)
{
    K3_TRY(ensure_ctx());
    if (!idx || !w || !x || !W) return fail(K3D_EINVAL, "k3d_router_bf16_noalloc null pointer");
    if (T < 1 || n_experts < 1 || (long long)T * n_experts > K3D_ROUTER_NOALLOC_MAX)
        return fail(K3D_EBOUND, "k3d_router_bf16_noalloc: T=%d x n_experts=%d scores exceed "
                    "the fixed scratch of %d", T, n_experts, K3D_ROUTER_NOALLOC_MAX);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(K3D_ECUDA, "k3d_router_bf16_noalloc: device %d: %s", dev, cudaGetErrorString(e));
    // set-up once per device: the address of the scratch array in this device's module
    static void *ws_of[kMaxDevices];
    if (!ws_of[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_router_noalloc_ws);
        if (e != cudaSuccess || !p)
            return fail(K3D_ECUDA, "k3d_router_bf16_noalloc: scratch address: %s",
                        cudaGetErrorString(e));
        ws_of[dev] = p;
    }
    return router_bf16(idx, w, x, W, bias, T, hidden, n_experts, topk, renorm, routed_scale,
                       ws_of[dev], stream());
}

}  // extern "C"
