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
//   A warp computes (1) the exact sum to ~2^-100 relative with compensated lane sums
//   and a TwoSum tree, and (2) sum_k |s_k| from a second pass over prefix sums. If the
//   whole interval [S - bound, S + bound] rounds to one float, that float IS
//   (float)acc of the CPU. Otherwise (about one expert in 10^5 at the benchmark shapes)
//   lane 0 runs the CPU's exact sequential loop for that expert.
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

// One warp per (token, expert): writes score and choice.
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
    const int seg = (hidden + 31) >> 5;
    const int lo = min(hidden, lane * seg);
    const int hi = min(hidden, lo + seg);

    // pass 1: compensated lane sum (Neumaier) and sum of |p|
    double s = 0.0, c = 0.0, a = 0.0;
    for (int i = lo; i < hi; i++) {
        const double p = __dmul_rn(wval<WT>(row, i), (double)__ldg(xt + i));
        const double tt = __dadd_rn(s, p);
        if (fabs(s) >= fabs(p)) c = __dadd_rn(c, __dadd_rn(__dsub_rn(s, tt), p));
        else c = __dadd_rn(c, __dadd_rn(__dsub_rn(p, tt), s));
        s = tt;
        a = __dadd_rn(a, fabs(p));
    }
    // lane total for the prefix pass
    const double lane_tot = __dadd_rn(s, c);
    // exclusive prefix of lane totals
    double incl = lane_tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = __dadd_rn(incl, v);
    }
    const double excl = __dsub_rn(incl, lane_tot);

    // exact-ish total: TwoSum tree over (s, c) pairs
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
    const double total = hs;  // |ls| <= u |hs|
    const double A = warp_sum_d(a);

    // pass 2: sum over k of |prefix sum|
    double run = excl, absum = 0.0;
    for (int i = lo; i < hi; i++) {
        const double p = __dmul_rn(wval<WT>(row, i), (double)__ldg(xt + i));
        run = __dadd_rn(run, p);
        absum = __dadd_rn(absum, fabs(run));
    }
    const double R = warp_sum_d(absum);

    float logit = 0.f;
    if (lane == 0) {
        const double u = 0x1p-53;
        const double n = (double)hidden;
        const double gam = n * u / (1.0 - n * u);
        // sequential-sum bound + error of our own total + slack for the arithmetic here
        const double bound = (u * (R + 4.0 * n * gam * A) + 8.0 * u * fabs(total) +
                              64.0 * n * n * u * u * A) * (1.0 + 0x1p-20) + 0x1p-1074;
        const float flo = (float)(total - bound);
        const float fhi = (float)(total + bound);
        if (flo == fhi) {
            logit = flo;
        } else {
            // ambiguous: reproduce the CPU loop exactly
            double acc = 0.0;
            for (int i = 0; i < hidden; i++)
                acc = __dadd_rn(acc, __dmul_rn(wval<WT>(row, i), (double)__ldg(xt + i)));
            logit = (float)acc;
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
    k_router_scores<WT><<<grid, 256, 0, s>>>(score, choice, x, W, bias, hidden, n_experts);
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

}  // extern "C"
