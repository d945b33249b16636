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
//   Every product W*x is exact in double (at most 24 + 24 significant bits), so the only
//   rounding in the CPU sum is in its additions. A warp computes the exact sum S (TwoSum
//   accumulation, ~2^-100 relative) and a rigorous bound B on |CPU sum - S|. If the whole
//   interval [S - B, S + B] rounds to one float, that float IS (float)acc of the CPU;
//   otherwise lane 0 runs the CPU's sequential loop for that expert (k3d_router_fallbacks
//   counts these).
//   The bound counts only additions that can round: fl(s + p) is exact when s and p are
//   both multiples of the ulp of the largest possible result, which the warp decides from
//   the exact p and a running prefix known to within a margin M = 4 n u sum|p|. With bf16
//   weights a product has at most 32 significant bits, so only additions of tiny products
//   and additions that move the running sum into a higher binade can round; B is a few
//   ulps of the running sum instead of the classical u * sum |prefix|, and the fallback,
//   which that classical bound needed about once per 800 experts, becomes rare.
//   The sigmoid uses k3_expf (glibc's expf restated, bit-identical), and all float
//   operations use explicit round-to-nearest intrinsics so nothing is contracted.
#include "k3_bulk.cuh"
#include "k3_common.cuh"
#include "k3_expf.h"
#include "k3_moe.cuh"
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

// Binary exponent of a positive normal double, and of its lowest set bit ("quantum":
// p is an odd multiple of 2^quantum_exp(p)). Zero has no quantum (a large sentinel).
__device__ __forceinline__ int exp_of(double v)
{
    return (int)((__double_as_longlong(v) >> 52) & 0x7ff) - 1023;
}

__device__ __forceinline__ int quantum_exp(double p)
{
    const unsigned long long b = (unsigned long long)__double_as_longlong(p) & 0x7fffffffffffffffull;
    if (b == 0) return 4096;
    const int be = (int)(b >> 52);
    const unsigned long long m = (b & ((1ull << 52) - 1)) | (be ? (1ull << 52) : 0ull);
    return (be ? be : 1) - 1075 + (__ffsll((long long)m) - 1);
}

// Counts experts whose logit needed the sequential fallback (read by k3d_router_fallbacks).
__device__ unsigned long long k3_router_fallbacks;

template <typename WT> struct Chunk;
template <> struct Chunk<uint16_t> {   // 8 bf16 = 16 bytes
    __device__ static void load_smem_f32(const unsigned char *seg, int c, float w[8])
    {
        const uint4 v = *reinterpret_cast<const uint4 *>(seg + 16 * c);
        const uint32_t uu[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[2 * i] = __uint_as_float(uu[i] << 16);
            w[2 * i + 1] = __uint_as_float(uu[i] & 0xffff0000u);
        }
    }
    __device__ static void load_smem(const unsigned char *seg, int c, double w[8])
    {
        const uint4 v = *reinterpret_cast<const uint4 *>(seg + 16 * c);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[2 * i] = (double)__uint_as_float(u[i] << 16);
            w[2 * i + 1] = (double)__uint_as_float(u[i] & 0xffff0000u);
        }
    }
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
    __device__ static void load_smem_f32(const unsigned char *seg, int c, float w[8])
    {
        const float4 a = *reinterpret_cast<const float4 *>(seg + 32 * c);
        const float4 b = *reinterpret_cast<const float4 *>(seg + 32 * c + 16);
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    }
    __device__ static void load_smem(const unsigned char *seg, int c, double w[8])
    {
        const float4 a = *reinterpret_cast<const float4 *>(seg + 32 * c);
        const float4 b = *reinterpret_cast<const float4 *>(seg + 32 * c + 16);
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    }
    __device__ static void load(const float *row, int c, double w[8])
    {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(row) + 2 * c);
        const float4 b = __ldg(reinterpret_cast<const float4 *>(row) + 2 * c + 1);
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    }
};

// The logit of one expert from the warp's pieces: total (exact sum, double-double), A =
// sum |p|, R = sum over k of |computed prefix k| in the CPU's order; returns the float the
// CPU's sequential double loop produces, running that loop itself only when the error
// bound does not settle the rounding.
template <typename WT>
__device__ __forceinline__ float settle_logit(double total, double A, double R, const WT *row,
                                              const float *xt, int hidden)
{
    const double u = 0x1p-53;
    const double n = (double)hidden;
    const double gam = n * u / (1.0 - n * u);
    const double bound = (u * (R + 4.0 * n * gam * A) + 8.0 * u * fabs(total) +
                          64.0 * n * n * u * u * A) * (1.0 + 0x1p-20) + 0x1p-1074;
    const float flo = (float)(total - bound);
    const float fhi = (float)(total + bound);
    if (flo == fhi) return flo;
    // ambiguous: the CPU's exact sequential loop (k3_ops.c:449-450)
    double acc = 0.0;
    for (int i = 0; i < hidden; i++) acc = __dadd_rn(acc, __dmul_rn(wval<WT>(row, i), (double)__ldg(xt + i)));
    atomicAdd(&k3_router_fallbacks, 1ull);
    return (float)acc;
}

// 2-adic valuation (exponent of the lowest set bit) of a bf16 or fp32 value, and of a
// product: v(w * x) = v(w) + v(x). Zero has none (a large sentinel).
__device__ __forceinline__ int val_f32(float f)
{
    const uint32_t b = __float_as_uint(f) & 0x7fffffffu;
    if (b == 0) return 4096;
    const int be = (int)(b >> 23);
    const uint32_t m = (b & 0x7fffffu) | (be ? 0x800000u : 0u);
    return (be ? be : 1) - 150 + (__ffs((int)m) - 1);
}

// ---------------------------------------------------------------- the exact path
// For the rare expert whose logit the fast pass cannot settle and that can change the
// selection. x and the expert's row are staged in shared memory as 128 contiguous segments
// of se = hidden/128 elements in the CPU's order (segment g at g * pitch, padded so that
// the lanes' 16-byte reads hit distinct banks). All 128 threads of the CTA call
// exact_logit; lane l of warp q owns segment 32q + l.
//
// Exact pass: the exact sum S of the products (TwoSum accumulation per lane, then exact
// combination of lanes and quarters) and A = sum |p|. Any summation order of n terms is
// within gamma_n * A of S (gamma_n = n u / (1 - n u)), so if [S - gamma_n A, S + gamma_n A]
// rounds to one float, that float is the CPU's logit.
//
// Tight pass: a rigorous bound that counts only additions that can round. Step k computes
// fl(s^_{k-1} + p_k), exact when the result is a multiple of U = ulp of the largest
// |s^_{k-1} + p_k| possible. Two sufficient tests:
//   granularity: every CPU prefix s^_k is a multiple of 2^G_k, G_k = the lowest 2-adic
//     valuation among p_1..p_k (an exact sum keeps it; a rounded one is a multiple of
//     its ulp, itself a multiple of 2^G_k), so G_k >= log2 U suffices;
//   alignment: p_k is a multiple of U and the smallest possible |s^_{k-1}| lies in a
//     binade no lower than U's.
// `run` tracks the prefix to within M = 4 n u A of both the exact prefix and the CPU's.
// Each step that may round adds U/2. If the bound is zero and S is a double, the CPU sum
// is S; otherwise the interval test is repeated with the tight bound, and if that still
// straddles a float rounding boundary thread 0 runs the CPU's sequential loop
// (k3d_router_fallbacks counts these).
struct ExactShared {
    double th[4], tl[4], A[4], bt[4];
    int q[4];
    float logit;
};

__host__ __device__ __forceinline__ int seg_xpitch(int hidden) { return (hidden >> 10) * 32 + 16; }
template <typename WT>
__host__ __device__ __forceinline__ int seg_wpitch(int hidden)
{
    return (hidden >> 10) * 8 * (int)sizeof(WT) + (sizeof(WT) == 2 ? 32 : 16);
}

// Copies hidden elements of elem_bytes each as 128 segments, segment g at dst + g * pitch.
__device__ __forceinline__ void stage_segments(unsigned char *dst, const void *src, int hidden,
                                               int elem_bytes, int pitch)
{
    const int per = (hidden >> 7) * elem_bytes / 16;      // 16-byte pieces per segment
    const int n16 = hidden * elem_bytes / 16;
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    const unsigned char *s = static_cast<const unsigned char *>(src);
    for (int c = threadIdx.x; c < n16; c += blockDim.x)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                     :: "r"(d + (uint32_t)((c / per) * pitch + (c % per) * 16)), "l"(s + 16 * (size_t)c)
                     : "memory");
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
}

template <typename WT>
__device__ float exact_logit(const unsigned char *xs, const unsigned char *wr, int hidden,
                             ExactShared &X)
{
    const int lane = threadIdx.x & 31, q = threadIdx.x >> 5;
    const int se = hidden >> 7;               // elements per segment
    const int nc = se >> 3;                   // 8-element chunks per segment
    const int xpitch = seg_xpitch(hidden);
    const int wpitch = seg_wpitch<WT>(hidden);
    const int seg = q * 32 + lane;
    const unsigned char *xl = xs + seg * xpitch;
    const unsigned char *wl = wr + seg * wpitch;

    // ---- exact pass: exact segment total, sum |p|
    double hs[4] = {0.0, 0.0, 0.0, 0.0}, ls[4] = {0.0, 0.0, 0.0, 0.0};
    double A0 = 0.0, A1 = 0.0;
    for (int c = 0; c < nc; c++) {
        double w[8];
        Chunk<WT>::load_smem(wl, c, w);
        const float4 xa = *reinterpret_cast<const float4 *>(xl + 32 * c);
        const float4 xb = *reinterpret_cast<const float4 *>(xl + 32 * c + 16);
        const double xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const double pi = __dmul_rn(w[i], xv[i]);
            const int k = i & 3;
            const double s1 = __dadd_rn(hs[k], pi);
            const double bb = __dsub_rn(s1, hs[k]);
            ls[k] = __dadd_rn(ls[k], __dadd_rn(__dsub_rn(hs[k], __dsub_rn(s1, bb)), __dsub_rn(pi, bb)));
            hs[k] = s1;
            if (i & 1) A1 = __dadd_rn(A1, fabs(pi)); else A0 = __dadd_rn(A0, fabs(pi));
        }
    }
    // the lane's exact total as a double-double
    double lh = hs[0], ll = ls[0];
#pragma unroll
    for (int k = 1; k < 4; k++) {
        double sum, err;
        two_sum(lh, hs[k], sum, err);
        const double low = __dadd_rn(__dadd_rn(ll, ls[k]), err);
        two_sum(sum, low, lh, ll);
    }
    // the quarter's exact total: TwoSum tree over the lanes
    double h = lh, l = ll;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const double oh = __shfl_xor_sync(0xffffffffu, h, o);
        const double ol = __shfl_xor_sync(0xffffffffu, l, o);
        double sum, err;
        two_sum(h, oh, sum, err);
        const double low = __dadd_rn(__dadd_rn(l, ol), err);
        two_sum(sum, low, h, l);
    }
    const double Aq = warp_sum_d(__dadd_rn(A0, A1));
    if (lane == 0) { X.th[q] = h; X.tl[q] = l; X.A[q] = Aq; }
    __syncthreads();
    // the row's exact total and sum |p| (same arithmetic in every thread)
    double Sh = X.th[0], Sl = X.tl[0];
    double A = X.A[0];
    for (int k = 1; k < 4; k++) {
        double sum, err;
        two_sum(Sh, X.th[k], sum, err);
        const double low = __dadd_rn(__dadd_rn(Sl, X.tl[k]), err);
        two_sum(sum, low, Sh, Sl);
        A = __dadd_rn(A, X.A[k]);
    }
    const double u = 0x1p-53;
    const double n = (double)hidden;
    const double slack = 8.0 * u * fabs(Sh) + fabs(Sl);
    {
        const double gam = n * u / (1.0 - n * u);
        const double bound = (gam * A * (1.0 + 0x1p-20) + slack) * (1.0 + 0x1p-20) + 0x1p-1074;
        const float flo = (float)__dsub_rn(Sh, bound), fhi = (float)__dadd_rn(Sh, bound);
        if (flo == fhi) return flo;          // uniform: every thread computed the same values
    }
    // ---- tight pass
    const double M = 4.0 * n * u * A + 0x1p-1000;
    // the lane's lowest product valuation (integer work on the raw bits only)
    int qmin = 4096;
    for (int c = 0; c < nc; c++) {
        float wf[8];
        Chunk<WT>::load_smem_f32(wl, c, wf);
        const float4 xa = *reinterpret_cast<const float4 *>(xl + 32 * c);
        const float4 xb = *reinterpret_cast<const float4 *>(xl + 32 * c + 16);
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int i = 0; i < 8; i++) qmin = min(qmin, val_f32(wf[i]) + val_f32(xv[i]));
    }
    int wq = qmin;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wq = min(wq, __shfl_xor_sync(0xffffffffu, wq, o));
    if (lane == 0) X.q[q] = wq;
    __syncthreads();
    // offsets: previous quarters' totals + the exclusive prefix of this warp's lane totals
    double off = 0.0;
    int G = 4096;
    for (int k = 0; k < q; k++) { off = __dadd_rn(off, __dadd_rn(X.th[k], X.tl[k])); G = min(G, X.q[k]); }
    const double lt = __dadd_rn(lh, ll);
    double incl = lt;
    int gq = qmin;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double v = __shfl_up_sync(0xffffffffu, incl, o);
        const int vq = __shfl_up_sync(0xffffffffu, gq, o);
        if (lane >= o) { incl = __dadd_rn(incl, v); gq = min(gq, vq); }
    }
    const int gprev = __shfl_up_sync(0xffffffffu, gq, 1);
    if (lane > 0) G = min(G, gprev);
    double run = __dadd_rn(off, __dsub_rn(incl, lt)), bt = 0.0;
    for (int c = 0; c < nc; c++) {
        float wf[8];
        Chunk<WT>::load_smem_f32(wl, c, wf);
        const float4 xa = *reinterpret_cast<const float4 *>(xl + 32 * c);
        const float4 xb = *reinterpret_cast<const float4 *>(xl + 32 * c + 16);
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const double pi = __dmul_rn((double)wf[i], (double)xv[i]);
            // valuation of p (4096 for zero, so a zero product never lowers G)
            const int qe = val_f32(wf[i]) + val_f32(xv[i]);
            G = min(G, qe);
            const double prev_lo = __dsub_rn(fabs(run), M);      // <= |s^_{k-1}|
            run = __dadd_rn(run, pi);
            const int E = exp_of(__dadd_rn(fabs(run), M));       // binade of max |s^_{k-1} + p_k|
            const int Ep = prev_lo > 0.0 ? exp_of(prev_lo) : -4096;
            const bool exact = (G >= E - 52) || (qe >= E - 52 && Ep >= E);
            // branch-free: + U/2 = 2^(E-53) when the step may round
            bt = __dadd_rn(bt, exact ? 0.0 : __longlong_as_double((long long)(E - 53 + 1023) << 52));
        }
    }
    bt = warp_sum_d(bt);
    if (lane == 0) X.bt[q] = bt;
    __syncthreads();
    if (threadIdx.x == 0) {
        const double B = __dadd_rn(__dadd_rn(X.bt[0], X.bt[1]), __dadd_rn(X.bt[2], X.bt[3]));
        float flo, fhi;
        if (B == 0.0 && Sl == 0.0) {
            flo = fhi = (float)Sh;       // no addition can have rounded: the CPU sum is S
        } else {
            const double bound = (B + slack) * (1.0 + 0x1p-20) + 0x1p-1074;
            flo = (float)__dsub_rn(Sh, bound);
            fhi = (float)__dadd_rn(Sh, bound);
        }
        float logit = flo;
        if (flo != fhi) {
            // still ambiguous: the CPU's sequential loop (k3_ops.c:449-450), from shared memory
            double acc = 0.0;
            for (int i = 0; i < hidden; i++) {
                const int sg = i / se, k = i % se;
                const double wv = (sizeof(WT) == 2)
                    ? (double)__uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(wr + sg * wpitch)[k] << 16)
                    : (double)reinterpret_cast<const float *>(wr + sg * wpitch)[k];
                const double xv = (double)reinterpret_cast<const float *>(xs + sg * xpitch)[k];
                acc = __dadd_rn(acc, __dmul_rn(wv, xv));
            }
            atomicAdd(&k3_router_fallbacks, 1ull);
            logit = (float)acc;
        }
        X.logit = logit;
    }
    __syncthreads();
    return X.logit;
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
        const float logit = settle_logit<WT>(total, A, R, row, xt, hidden);
        const float sc = __fdiv_rn(1.0f, __fadd_rn(1.0f, k3_expf(-logit)));
        score[(size_t)t * n_experts + e] = sc;
        choice[(size_t)t * n_experts + e] = bias ? __fadd_rn(sc, __ldg(bias + e)) : sc;
    }
}

// Renorm and scale of the selected weights, then the stores (k3_ops.c:468-475).
__device__ __forceinline__ void topk_finish(int *idx, float *wout, const int *isel, float *wsel,
                                            int topk, int renorm, float routed_scale)
{
    if (renorm && topk > 1) {
        double s = 0.0;
        for (int j = 0; j < topk; j++) s = __dadd_rn(s, (double)wsel[j]);
        const float inv = (float)__ddiv_rn(1.0, __dadd_rn(s, 1e-20));
        for (int j = 0; j < topk; j++) wsel[j] = __fmul_rn(wsel[j], inv);
    }
    for (int j = 0; j < topk; j++) {
        idx[j] = isel[j];
        wout[j] = __fmul_rn(wsel[j], routed_scale);
    }
}

// Warp argmax step: larger value wins; on equal values the lower index (the one a forward
// scan meets first) wins; -1 (nothing found) loses to anything found.
__device__ __forceinline__ void warp_best(float &bv, int &best)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int ob = __shfl_xor_sync(0xffffffffu, best, o);
        const bool take = (ob >= 0) && (best < 0 || ov > bv || (ov == bv && ob < best));
        if (take) { bv = ov; best = ob; }
    }
}

// One warp per token, the choices held in registers (lane l: experts l, l+32, ...;
// n_experts <= 32*PER): top-k by repeated strict-greater max (k3_ops.c:459-466).
template <int PER>
__global__ void k_router_topk_reg(int *idx, float *wout, const float *choice, const float *score,
                                  int n_experts, int topk, int renorm, float routed_scale,
                                  int idx_stride)
{
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x;
    const float *ch = choice + (size_t)t * n_experts;
    const float *scr = score + (size_t)t * n_experts;
    float v[PER], sv[PER];
#pragma unroll
    for (int k = 0; k < PER; k++) {
        const int e = lane + 32 * k;
        v[k] = e < n_experts ? ch[e] : -INFINITY;
        sv[k] = e < n_experts ? scr[e] : 0.0f;
    }
    __shared__ float wsel[K3_MAX_TOPK];
    __shared__ int isel[K3_MAX_TOPK];
    for (int j = 0; j < topk; j++) {
        float bv = -INFINITY;
        int best = -1;
#pragma unroll
        for (int k = 0; k < PER; k++)
            if (v[k] > bv) { bv = v[k]; best = lane + 32 * k; }
        warp_best(bv, best);
        if (best >= 0 && (best & 31) == lane) {
            // the owning lane takes the entry out and publishes its unbiased score
#pragma unroll
            for (int k = 0; k < PER; k++)
                if (lane + 32 * k == best) { v[k] = -INFINITY; wsel[j] = sv[k]; }
            isel[j] = best;
        }
        if (best < 0 && lane == 0) { isel[j] = 0; wsel[j] = 0.0f; }
    }
    __syncwarp();
    if (lane == 0)
        topk_finish(idx + (size_t)t * idx_stride, wout + (size_t)t * idx_stride, isel, wsel,
                    topk, renorm, routed_scale);
}

// Any n_experts: the choices stay in global memory (taken entries become -inf there).
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
        warp_best(bv, best);
        if (lane == 0) {
            if (best < 0) { isel[j] = 0; wsel[j] = 0.0f; }
            else { isel[j] = best; wsel[j] = scr[best]; ch[best] = -INFINITY; }
        }
        __syncwarp();
    }
    if (lane == 0)
        topk_finish(idx + (size_t)t * idx_stride, wout + (size_t)t * idx_stride, isel, wsel,
                    topk, renorm, routed_scale);
}

// ------------------------------------------------------------------ fused router
// One launch for scores, top-k and (MoE) the grouping of assignments by expert.
//
// Phase 1, CTA = 2 experts x 128 threads; quarter q (a warp) takes a contiguous quarter of
// the row, lane l its 8-element chunks l, l+32, ... (coalesced). Per expert, in fp64, the
// sum s~ of the exact products in this order (summation depth d <= 128 for hidden <= 16384)
// and, in fp32, A~ = sum |w||x| (an upper bound after a relative 2^-15 and an absolute
// 2^-100 margin). The CPU's sequential sum is within gamma_{n-1} A of the exact sum S and
// s~ within gamma_d A, so [s~ - B, s~ + B] with B = gamma_{n+128} A~ (+ 4u|s~| for the
// rounding of the endpoints) holds the CPU's double; if both ends round to one float, that
// float is the CPU's logit ("settled", about 99% of experts). Otherwise the expert carries
// an interval [lo, hi] of its choice value (sigmoid + bias at both ends, widened by two
// float ulps for the last-bit behaviour of expf).
//
// Phase 2, the last CTA of token t (completion counter): top-k by repeated strict-greater
// max over keys = the exact choice of settled experts and lo of the others. If every
// selected expert is settled and every unsettled one has hi below the k-th selected key,
// the selection is the CPU's (each unsettled expert is below k settled ones). Otherwise
// the offending experts are settled exactly (the exact path above) and the selection is
// repeated. Then the weights (renorm in double) and, for the MoE, once the last token is
// done, the grouping by expert.
constexpr int kRouterMaxT = 4096;          // tokens per fused call
constexpr int kNeedMax = 16;               // exact settlements per selection round
// Completion counters: [t] counts the CTAs of token t that wrote their experts,
// [kRouterMaxT] the tokens whose top-k is written. The last CTA to arrive resets its
// counter, so every call starts from zero; calls are ordered on the library stream.
__device__ unsigned int g_router_ctr[kRouterMaxT + 1] = {0};

struct RouterJob {
    const float *x;
    const void *W;
    const float *bias;
    float *lo, *hi, *score;        // [T][n_experts] scratch
    int *idx;
    float *wts;
    int T, hidden, n_experts, topk, renorm;
    float routed_scale;
    // grouping of the assignments by expert (MoE), when n_active is set
    int *n_active, *act_expert, *act_off, *assign;
    int e_lo, e_hi;
    int *zero;                     // zeroed with the grouping (nzero ints)
    int nzero;
};

template <typename WT> struct WChunk;       // 8 weights held in registers
template <> struct WChunk<uint16_t> {
    uint4 v;
    __device__ __forceinline__ void load(const uint16_t *row, int c) { v = ldg_nc_v4(row + 8 * (size_t)c); }
    __device__ __forceinline__ void load_s(const uint16_t *row, int c) { v = *reinterpret_cast<const uint4 *>(row + 8 * (size_t)c); }
    __device__ __forceinline__ void get(float w[8]) const
    {
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w[2 * i] = __uint_as_float(u[i] << 16);
            w[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
        }
    }
};
template <> struct WChunk<float> {
    uint4 a, b;
    __device__ __forceinline__ void load(const float *row, int c)
    {
        a = ldg_nc_v4(row + 8 * (size_t)c);
        b = ldg_nc_v4(row + 8 * (size_t)c + 4);
    }
    __device__ __forceinline__ void load_s(const float *row, int c)
    {
        a = *reinterpret_cast<const uint4 *>(row + 8 * (size_t)c);
        b = *reinterpret_cast<const uint4 *>(row + 8 * (size_t)c + 4);
    }
    __device__ __forceinline__ void get(float w[8]) const
    {
        w[0] = __uint_as_float(a.x); w[1] = __uint_as_float(a.y);
        w[2] = __uint_as_float(a.z); w[3] = __uint_as_float(a.w);
        w[4] = __uint_as_float(b.x); w[5] = __uint_as_float(b.y);
        w[6] = __uint_as_float(b.z); w[7] = __uint_as_float(b.w);
    }
};

// atomic add with acquire-release semantics at GPU scope: it releases this thread's earlier
// stores and, for the CTA that arrives last, acquires the stores the others released
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned *p, unsigned v)
{
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Order-preserving code of a selection key: a larger float gives a larger code, -0 and +0
// the same; -inf and NaN give 0, which the top-k never selects (the CPU's strict-greater
// scan from -inf never selects them either).
__device__ __forceinline__ uint32_t order_code(float v)
{
    if (!(v > -INFINITY)) return 0u;
    const uint32_t u = __float_as_uint(__fadd_rn(v, 0.0f));
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// The largest of a lane's 16 codes (a max tree).
__device__ __forceinline__ uint32_t umax16(const uint32_t c[16])
{
    uint32_t v[8];
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = max(c[i], c[i + 8]);
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = max(v[i], v[i + 4]);
    v[0] = max(v[0], v[2]);
    v[1] = max(v[1], v[3]);
    return max(v[0], v[1]);
}

__device__ __forceinline__ float sigmoid_k(float v)
{
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, k3_expf(-v)));
}

// Dynamic shared memory: phase 1 holds the CTA's two weight rows and x (bulk copies);
// phase 2 (the last CTA only, after phase 1) reuses it for the keys and the exact path.
template <typename WT>
__host__ __device__ inline size_t fused_smem_bytes(int hidden, int n_experts)
{
    const size_t p2 = (size_t)128 * seg_xpitch(hidden) + (size_t)128 * seg_wpitch<WT>(hidden) +
                      (size_t)n_experts * (3 * sizeof(float) + 2 * sizeof(int) + 1) + 16;
    const size_t p1 = (size_t)2 * hidden * sizeof(WT) + (size_t)hidden * sizeof(float);
    return p1 > p2 ? p1 : p2;
}

template <typename WT>
__global__ void __launch_bounds__(128) k_router_fused(RouterJob J)
{
    extern __shared__ __align__(16) unsigned char rsm[];
    __shared__ double p_s[2][4];
    __shared__ float p_a[2][4];
    __shared__ ExactShared X;
    __shared__ int s_last, s_nneed;
    __shared__ int s_need[kNeedMax];
    __shared__ int s_isel[K3_MAX_TOPK];
    __shared__ int s_idx[K3_MAX_TOPK];
    __shared__ uint32_t s_qc[4][8];          // quarter top-k (K <= 8): codes, experts
    __shared__ int s_qi[4][8];
    __shared__ float s_m;
    const int lane = threadIdx.x & 31, q = threadIdx.x >> 5;
    const int t = blockIdx.y;
    const int E = J.n_experts, hidden = J.hidden;
    const int e0 = blockIdx.x * 2;
    const float *xt = J.x + (size_t)t * hidden;
    const WT *W = static_cast<const WT *>(J.W);
    const size_t tE = (size_t)t * E;
    if (threadIdx.x == 0) s_last = 0;
    // loads whose latency would otherwise sit on the tail of phase 1: the writers' biases,
    // and the expf table (constant memory) into this SM's constant cache
    const int ew = e0 + (int)threadIdx.x;
    const float bias_w = (threadIdx.x < 2 && ew < E && J.bias) ? __ldg(J.bias + ew) : 0.0f;
    if (q == 3 && k3_exp2_tab_d[lane] == 0ull) s_last = 0;   // never true: keeps the load

    // ---------------------------------------------------------------- phase 1
    {
        const int nj = hidden >> 10;                     // chunks per lane
        const int cbase = q * (hidden >> 5) + lane;
        const bool act0 = e0 < E, act1 = e0 + 1 < E;
        const int nrows = act1 ? 2 : 1;
        // the CTA's weight rows (adjacent: one copy) and x arrive by bulk copies into
        // shared memory, the rows before the programmatic wait (weights never depend on
        // the kernel before), x after it
        __shared__ __align__(8) unsigned long long p1_bar[2];
        __shared__ int p1_abort;
        WT *wsm = reinterpret_cast<WT *>(rsm);
        float *xsm = reinterpret_cast<float *>(rsm + (size_t)2 * hidden * sizeof(WT));
        const uint32_t b_w = bulk::saddr(&p1_bar[0]), b_x = bulk::saddr(&p1_bar[1]);
        if (threadIdx.x == 0) {
            bulk::mbar_init(b_w, 1);
            bulk::mbar_init(b_x, 1);
            p1_abort = 0;
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            const uint32_t wbytes = (uint32_t)((size_t)nrows * hidden * sizeof(WT));
            bulk::mbar_expect_tx(b_w, wbytes);
            bulk::g2s(bulk::saddr(wsm), W + (size_t)e0 * hidden, wbytes, b_w);
        }
        pdl_wait();
        pdl_trigger();
        if (threadIdx.x == 0) {
            bulk::mbar_expect_tx(b_x, (uint32_t)(hidden * sizeof(float)));
            bulk::g2s(bulk::saddr(xsm), xt, (uint32_t)(hidden * sizeof(float)), b_x);
        }
        __syncthreads();                                  // the barriers are initialised
        // bounded waits: on a time-out the error flag is raised and the (stale) contents are
        // used, so that the completion count still finishes and resets
        bulk::mbar_wait(b_w, 0, &p1_abort, K3_SITE_ROUTER, 1);
        bulk::mbar_wait(b_x, 0, &p1_abort, K3_SITE_ROUTER, 2);
        const WT *row0 = wsm;
        const WT *row1 = wsm + hidden;
        double s0[2] = {0.0, 0.0}, s1[2] = {0.0, 0.0};
        float a[2] = {0.0f, 0.0f};
        WChunk<WT> wv[2][8];
        for (int j0 = 0; j0 < nj; j0 += 8) {
            float4 xv[8][2];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j0 + j < nj) {
                    const int c = cbase + 32 * (j0 + j);
                    xv[j][0] = reinterpret_cast<const float4 *>(xsm)[2 * c];
                    xv[j][1] = reinterpret_cast<const float4 *>(xsm)[2 * c + 1];
                    if (act0) wv[0][j].load_s(row0, c);
                    if (act1) wv[1][j].load_s(row1, c);
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j0 + j < nj) {
                    const float xf[8] = {xv[j][0].x, xv[j][0].y, xv[j][0].z, xv[j][0].w,
                                         xv[j][1].x, xv[j][1].y, xv[j][1].z, xv[j][1].w};
#pragma unroll
                    for (int k = 0; k < 2; k++) {
                        if (!(k == 0 ? act0 : act1)) continue;
                        float wf[8];
                        wv[k][j].get(wf);
#pragma unroll
                        for (int i = 0; i < 8; i += 2) {
                            // products are exact in double, so the fma rounds only the sum
                            s0[k] = __fma_rn((double)wf[i], (double)xf[i], s0[k]);
                            s1[k] = __fma_rn((double)wf[i + 1], (double)xf[i + 1], s1[k]);
                            a[k] = __fmaf_rn(fabsf(wf[i]), fabsf(xf[i]), a[k]);
                            a[k] = __fmaf_rn(fabsf(wf[i + 1]), fabsf(xf[i + 1]), a[k]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const double sk = warp_sum_d(__dadd_rn(s0[k], s1[k]));
            const float ak = warp_sum(a[k]);
            if (lane == 0) { p_s[k][q] = sk; p_a[k][q] = ak; }
        }
        __syncthreads();
        if (threadIdx.x < 2 && e0 + (int)threadIdx.x < E) {
            const int k = threadIdx.x, e = e0 + k;
            const double S = __dadd_rn(__dadd_rn(__dadd_rn(p_s[k][0], p_s[k][1]), p_s[k][2]), p_s[k][3]);
            const float A32 = __fadd_rn(__fadd_rn(__fadd_rn(p_a[k][0], p_a[k][1]), p_a[k][2]), p_a[k][3]);
            const double u = 0x1p-53, n = (double)hidden + 128.0;
            const double Aup = __fma_rn((double)A32, 1.0 + 0x1p-15, 0x1p-100);   // +inf stays +inf
            const double gam = n * u / (1.0 - n * u) * (1.0 + 0x1p-20);
            const double bound = __fma_rn(gam, Aup, 4.0 * u * fabs(S)) * (1.0 + 0x1p-20) + 0x1p-1074;
            const float flo = (float)__dsub_rn(S, bound), fhi = (float)__dadd_rn(S, bound);
            const float b = bias_w;
            float lo, hi, sc = 0.0f;
            if (flo == fhi) {
                sc = sigmoid_k(flo);
                lo = hi = J.bias ? __fadd_rn(sc, b) : sc;
            } else if (isnan(flo) || isnan(fhi)) {
                lo = hi = __int_as_float(0x7fc00000);
            } else {
                const float c1 = sigmoid_k(flo), c2 = sigmoid_k(fhi);
                lo = J.bias ? __fadd_rd(fminf(c1, c2), b) : fminf(c1, c2);
                hi = J.bias ? __fadd_ru(fmaxf(c1, c2), b) : fmaxf(c1, c2);
                lo = __fsub_rd(lo, __fmaf_ru(fabsf(lo), 0x1p-21f, 0x1p-120f));
                hi = __fadd_ru(hi, __fmaf_ru(fabsf(hi), 0x1p-21f, 0x1p-120f));
            }
            J.lo[tE + e] = lo;
            J.hi[tE + e] = hi;
            J.score[tE + e] = sc;
        }
        __syncthreads();
        // one arrival per CTA: after the barrier, thread 0's gpu-scope fence (cumulative over
        // the stores the barrier ordered before it) publishes both writers' stores, then the
        // count; the CTA that completes it acquires every other CTA's stores
        if (threadIdx.x == 0) __threadfence();
        if (threadIdx.x == 0 && atom_add_acq_rel(&g_router_ctr[t], 1u) == gridDim.x - 1) {
            g_router_ctr[t] = 0;
            s_last = 1;
        }
        __syncthreads();
        if (!s_last) return;
    }

    // ---------------------------------------------------------------- phase 2
    unsigned char *xs = rsm;
    unsigned char *wr = xs + 128 * seg_xpitch(hidden);
    float *key = reinterpret_cast<float *>(wr + 128 * seg_wpitch<WT>(hidden));
    float *hv = key + E;
    float *sv = hv + E;
    int *gsm = reinterpret_cast<int *>(sv + E);                 // 2 * E ints for the grouping
    unsigned char *settled = reinterpret_cast<unsigned char *>(gsm + 2 * E);
    {
        // every value in flight at once (E <= 512, 128 threads)
        float l4[4], h4[4], s4[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int e = threadIdx.x + 128 * k;
            if (e < E) {
                l4[k] = __ldcg(J.lo + tE + e);
                h4[k] = __ldcg(J.hi + tE + e);
                s4[k] = __ldcg(J.score + tE + e);
            }
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int e = threadIdx.x + 128 * k;
            if (e < E) {
                key[e] = l4[k];
                hv[e] = h4[k];
                sv[e] = s4[k];
                settled[e] = (l4[k] == h4[k]);
            }
        }
    }
    __syncthreads();
    const int K = J.topk;
    bool x_staged = false;
    for (int iter = 0; iter <= E; iter++) {
        if (K <= 8) {
            // top-k by repeated strict-greater max over the keys, lowest index on ties
            // (k3_ops.c:459-466), in two steps: warp q selects the top K of experts
            // [128 q, 128 q + 128) (lane l holds 128 q + l + 32 k, k < 4) by the rounds of
            // the single-warp scan below, then warp 0 selects the top K of the 4 K
            // candidates (one a lane) the same way. Every expert of the overall top K is in
            // its quarter's top K (fewer than K keys, in the order (key desc, index asc),
            // precede it there too), so the selection and its order are the same.
            uint32_t c[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int e = 128 * q + lane + 32 * k;
                c[k] = e < E ? order_code(key[e]) : 0u;
            }
            uint32_t bc = max(max(c[0], c[1]), max(c[2], c[3]));
            for (int j = 0; j < K; j++) {
                const uint32_t m = __reduce_max_sync(0xffffffffu, bc);
                int best = -1;
                if (m != 0u) {
                    uint32_t mask = 0u;
#pragma unroll
                    for (int k = 0; k < 4; k++) mask |= (c[k] == m ? 1u : 0u) << k;
                    const uint32_t cand = mask ? (uint32_t)(128 * q + lane + 32 * (__ffs(mask) - 1)) : 0xffffffffu;
                    best = (int)__reduce_min_sync(0xffffffffu, cand);
                }
                if (best >= 0 && (best & 31) == lane) {
                    const int kb = (best - 128 * q) >> 5;
#pragma unroll
                    for (int k = 0; k < 4; k++) c[k] = (k == kb) ? 0u : c[k];
                    bc = max(max(c[0], c[1]), max(c[2], c[3]));
                }
                if (lane == 0) {
                    s_qc[q][j] = best >= 0 ? m : 0u;
                    s_qi[q][j] = best;
                }
            }
            __syncthreads();
            if (q == 0) {
                uint32_t cc = 0u;
                int ci = -1;
                if (lane < 4 * K) {
                    cc = s_qc[lane / K][lane % K];
                    ci = s_qi[lane / K][lane % K];
                }
                for (int j = 0; j < K; j++) {
                    const uint32_t m = __reduce_max_sync(0xffffffffu, cc);
                    int best = -1;
                    if (m != 0u)
                        best = (int)__reduce_min_sync(0xffffffffu, cc == m ? (uint32_t)ci : 0xffffffffu);
                    if (best >= 0 && cc == m && ci == best) cc = 0u;
                    if (lane == 0) s_isel[j] = best;
                }
                if (lane == 0) {
                    const int b = s_isel[K - 1];
                    s_m = b >= 0 ? key[b] : -INFINITY;
                    s_nneed = 0;
                }
            }
        } else if (q == 0) {
            // top-k by repeated strict-greater max over the keys, lowest index on ties
            // (k3_ops.c:459-466): per round one redux for the largest key and one for the
            // lowest index holding it; lane l holds experts l + 32k, its lowest k holding
            // the round's maximum found from a bit mask
            uint32_t c[16];
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const int e = lane + 32 * k;
                c[k] = e < E ? order_code(key[e]) : 0u;
            }
            uint32_t bc = umax16(c);
            for (int j = 0; j < K; j++) {
                const uint32_t m = __reduce_max_sync(0xffffffffu, bc);
                int best = -1;
                if (m != 0u) {
                    uint32_t mask = 0u;
#pragma unroll
                    for (int k = 0; k < 16; k++) mask |= (c[k] == m ? 1u : 0u) << k;
                    const uint32_t cand = mask ? (uint32_t)(lane + 32 * (__ffs(mask) - 1)) : 0xffffffffu;
                    best = (int)__reduce_min_sync(0xffffffffu, cand);
                }
                if (best >= 0 && (best & 31) == lane) {
                    // the owning lane takes the entry out
#pragma unroll
                    for (int k = 0; k < 16; k++) c[k] = (k == (best >> 5)) ? 0u : c[k];
                    bc = umax16(c);
                }
                if (lane == 0) s_isel[j] = best;
            }
            if (lane == 0) {
                const int b = s_isel[K - 1];
                s_m = b >= 0 ? key[b] : -INFINITY;
                s_nneed = 0;
            }
        }
        __syncthreads();
        for (int e = threadIdx.x; e < E; e += blockDim.x) {
            if (settled[e]) continue;
            bool need = !(hv[e] < s_m);
            for (int j = 0; j < K; j++) need |= (s_isel[j] == e);
            if (need) {
                const int slot = atomicAdd(&s_nneed, 1);
                if (slot < kNeedMax) s_need[slot] = e;
            }
        }
        __syncthreads();
        const int nn = min(s_nneed, kNeedMax);
        if (nn == 0) break;
        if (!x_staged) {
            stage_segments(xs, xt, hidden, 4, seg_xpitch(hidden));
            x_staged = true;
        }
        for (int i = 0; i < nn; i++) {
            const int e = s_need[i];
            stage_segments(wr, W + (size_t)e * hidden, hidden, (int)sizeof(WT), seg_wpitch<WT>(hidden));
            __syncthreads();
            const float logit = exact_logit<WT>(xs, wr, hidden, X);
            if (threadIdx.x == 0) {
                const float sc = sigmoid_k(logit);
                const float c = J.bias ? __fadd_rn(sc, __ldg(J.bias + e)) : sc;
                key[e] = c;
                hv[e] = c;
                sv[e] = sc;
                settled[e] = 1;
            }
            __syncthreads();
        }
    }
    if (q == 0) {
        // weights (k3_ops.c:468-475): lane j < K fetches slot j; lane 0 forms the double
        // sum in slot order and the reciprocal; lanes scale and store their slots
        const bool rn = J.renorm && K > 1;
        const int b0 = lane < K ? s_isel[lane] : -1;
        const int b1 = lane + 32 < K ? s_isel[lane + 32] : -1;
        float w0 = b0 >= 0 ? sv[b0] : 0.0f;
        float w1 = b1 >= 0 ? sv[b1] : 0.0f;
        float inv = 1.0f;
        if (rn) {
            double sum = 0.0;
            if (K <= 8) {
                // the shuffles first (independent of the sum), then the sum in slot order
                float wv[8];
#pragma unroll
                for (int j = 0; j < 8; j++) wv[j] = __shfl_sync(0xffffffffu, w0, j);
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (j < K) sum = __dadd_rn(sum, (double)wv[j]);
            } else {
                for (int j = 0; j < K; j++) {
                    const float wj = __shfl_sync(0xffffffffu, j < 32 ? w0 : w1, j & 31);
                    sum = __dadd_rn(sum, (double)wj);
                }
            }
            // every lane holds the same sum: each forms the reciprocal itself
            inv = (float)__ddiv_rn(1.0, __dadd_rn(sum, 1e-20));
            w0 = __fmul_rn(w0, inv);
            w1 = __fmul_rn(w1, inv);
        }
        if (lane < K) {
            J.idx[(size_t)t * K + lane] = b0 >= 0 ? b0 : 0;
            s_idx[lane] = b0 >= 0 ? b0 : 0;
            J.wts[(size_t)t * K + lane] = __fmul_rn(w0, J.routed_scale);
        }
        if (lane + 32 < K) {
            J.idx[(size_t)t * K + lane + 32] = b1 >= 0 ? b1 : 0;
            s_idx[lane + 32] = b1 >= 0 ? b1 : 0;
            J.wts[(size_t)t * K + lane + 32] = __fmul_rn(w1, J.routed_scale);
        }
        if (J.T > 1) __threadfence();
    }
    if (!J.n_active) return;
    // ---------------------------------------------------------------- grouping
    __syncthreads();
    if (J.T > 1) {
        if (threadIdx.x == 0) {
            const unsigned prev = atom_add_acq_rel(&g_router_ctr[kRouterMaxT], 1u);
            s_last = (prev == (unsigned)J.T - 1);
            if (s_last) g_router_ctr[kRouterMaxT] = 0;
        }
        __syncthreads();
        if (!s_last) return;
    }
    // one token: its selection is in this CTA's shared memory; more: every token's last CTA
    // published its row of idx (fenced) before the count
    if (J.T == 1 && K <= 32) {
        // one token's K distinct experts: warp 0 writes what group_assignments writes (active
        // experts in increasing id order, one assignment each, act_off[u] = u, assign[u] the
        // slot of the u-th expert) from each slot's rank among the slots, without the count
        // and scan passes; a token holding an expert twice (only when fewer than K experts
        // were selectable) takes the general grouping below
        __shared__ int s_dup;
        for (int i = threadIdx.x; i < J.nzero; i += blockDim.x) J.zero[i] = 0;
        if (q == 0) {
            const int e = lane < K ? s_idx[lane] : -1;
            const bool in = lane < K && e >= J.e_lo && e < J.e_hi && e >= 0 && e < E;
            const unsigned inm = __ballot_sync(0xffffffffu, in);
            const unsigned same = __match_any_sync(0xffffffffu, in ? e : -1 - lane);
            const bool dup = __any_sync(0xffffffffu, in && __popc(same) > 1);
            if (!dup) {
                int rank = 0;
                for (int j = 0; j < K; j++) {
                    const int ej = __shfl_sync(0xffffffffu, e, j);
                    rank += ((inm >> j) & 1u) && ej < e;
                }
                if (in) {
                    J.act_expert[rank] = e;
                    J.act_off[rank] = rank;
                    J.assign[rank] = lane;
                }
                if (lane == 0) {
                    const int n = __popc(inm);
                    J.n_active[0] = n;
                    J.n_active[1] = n;
                    J.act_off[n] = n;
                }
            }
            if (lane == 0) s_dup = dup;
        }
        __syncthreads();
        if (!s_dup) return;
    }
    if (J.T == 1)
        group_assignments(s_idx, K, E, J.e_lo, J.e_hi, J.n_active, J.act_expert, J.act_off,
                          J.assign, gsm, J.zero, J.nzero, true);
    else
        group_assignments(J.idx, J.T * K, E, J.e_lo, J.e_hi, J.n_active, J.act_expert, J.act_off,
                          J.assign, gsm, J.zero, J.nzero);
}

size_t router_ws_bytes(int T, int n_experts)
{
    return 3 * (size_t)T * n_experts * sizeof(float) + 256;
}

template <typename WT>
static int router_launch(int *idx, float *w, const float *x, const WT *W, const float *bias,
                         int T, int hidden, int n_experts, int topk, int renorm,
                         float routed_scale, void *ws, cudaStream_t s, RouterGroup *grp)
{
    if (topk < 1 || topk > K3_MAX_TOPK)
        return fail(K3D_EBOUND, "router topk=%d outside 1..%d", topk, K3_MAX_TOPK);
    if (n_experts < 1 || hidden < 1 || T < 1)
        return fail(K3D_EINVAL, "router hidden=%d n_experts=%d T=%d", hidden, n_experts, T);
    if (grp) grp->done = 0;
    float *score = (float *)ws;
    float *choice = score + (size_t)T * n_experts;
    // the fused kernel needs hidden % 1024 == 0 (<= 16384), 16-byte aligned rows and x,
    // at most 512 experts (the register scan) and kRouterMaxT tokens
    const bool fused = (hidden % 1024) == 0 && hidden <= 16384 &&
                       (((uintptr_t)W | (uintptr_t)x) & 15u) == 0 && n_experts <= 512 &&
                       T <= kRouterMaxT;
    if (fused) {
        RouterJob J;
        J.x = x;
        J.W = W;
        J.bias = bias;
        J.lo = score;
        J.hi = score + (size_t)T * n_experts;
        J.score = score + 2 * (size_t)T * n_experts;
        J.idx = idx;
        J.wts = w;
        J.T = T;
        J.hidden = hidden;
        J.n_experts = n_experts;
        J.topk = topk;
        J.renorm = renorm;
        J.routed_scale = routed_scale;
        J.n_active = grp ? grp->n_active : nullptr;
        J.act_expert = grp ? grp->act_expert : nullptr;
        J.act_off = grp ? grp->act_off : nullptr;
        J.assign = grp ? grp->assign : nullptr;
        J.e_lo = grp ? grp->lo : 0;
        J.e_hi = grp ? grp->hi : n_experts;
        J.zero = grp ? grp->zero : nullptr;
        J.nzero = grp ? grp->nzero : 0;
        const size_t smem = fused_smem_bytes<WT>(hidden, n_experts);
        static unsigned long long init = 0;   // one bit per device
        if (!(init & dev_bit())) { allow_smem_max(k_router_fused<WT>); init |= dev_bit(); }
        dim3 grid((n_experts + 1) / 2, T);
        launch_pdl(k_router_fused<WT>, dim3(grid), dim3(128), smem, s, J);
        note_launch();
        if (grp) grp->done = 1;
        return check_launch("router");
    }
    dim3 grid((n_experts + 7) / 8, T);
    k_router_scores_generic<WT><<<grid, 256, 0, s>>>(score, choice, x, W, bias, hidden, n_experts);
    if (n_experts <= 512)
        k_router_topk_reg<16><<<T, 32, 0, s>>>(idx, w, choice, score, n_experts, topk, renorm,
                                               routed_scale, topk);
    else
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
                                routed_scale, ws, s, nullptr);
}

int router_bf16(int *idx, float *w, const float *x, const uint16_t *W, const float *bias,
                int T, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                void *ws, cudaStream_t s, RouterGroup *grp)
{
    return router_launch<uint16_t>(idx, w, x, W, bias, T, hidden, n_experts, topk, renorm,
                                   routed_scale, ws, s, grp);
}

// Fixed scratch of k3d_router_bf16_noalloc: three score arrays, each up to
// K3D_ROUTER_NOALLOC_MAX floats. Every element a call reads it has first written, so
// nothing needs clearing between calls.
static __device__ __align__(256) float g_router_noalloc_ws[3 * K3D_ROUTER_NOALLOC_MAX];
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
    // set-up once per device: the address of the scratch array in this device's module,
    // looked up under the context lock so that first calls from two threads do not race
    static void *ws_of[kMaxDevices];
    void *ws = nullptr;
    {
        std::lock_guard<std::recursive_mutex> lk(g_mu);
        if (!ws_of[dev]) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_router_noalloc_ws);
            if (e != cudaSuccess || !p)
                return fail(K3D_ECUDA, "k3d_router_bf16_noalloc: scratch address: %s",
                            cudaGetErrorString(e));
            ws_of[dev] = p;
        }
        ws = ws_of[dev];
    }
    return router_bf16(idx, w, x, W, bias, T, hidden, n_experts, topk, renorm, routed_scale,
                       ws, stream());
}

}  // extern "C"
