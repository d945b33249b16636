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

// ------------------------------------------------------------------ scores kernel
// CTA = 2 experts x 4 warps (256 threads); warp w takes expert slot w/4 and quarter w%4
// of the row. The row is cut into 128 contiguous segments of se = hidden/128 elements in
// the CPU's order; lane l of quarter q owns segment 32q + l. x and both rows are staged in
// shared memory first (independent cp.async copies: the memory latency is paid once),
// each segment padded so that the lanes' 16-byte reads hit distinct banks.
//
// Fast pass (every expert): the exact sum S of the products (TwoSum accumulation per lane,
// then exact combination of lanes and quarters) and A = sum |p|. Any summation order of n
// terms is within gamma_n * A of S (gamma_n = n u / (1 - n u)), so if
// [S - gamma_n A, S + gamma_n A] rounds to one float, that float is the CPU's logit
// (about 99.4% of experts at the benchmark shapes).
//
// Tight pass (the rest; the expert's 4 warps, synchronised by a named barrier): a
// rigorous bound that counts only additions that can round. Step k computes
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
// straddles a float rounding boundary lane 0 runs the CPU's sequential loop.
template <typename WT>
__global__ void __launch_bounds__(256) k_router_scores(float *score, float *choice,
                                                       const float *x, const WT *W,
                                                       const float *bias, int hidden,
                                                       int n_experts)
{
    extern __shared__ __align__(16) unsigned char rsm[];
    __shared__ double s_th[2][4], s_tl[2][4], s_A[2][4], s_bt[2][4];
    __shared__ int s_q[2][4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int es = warp >> 2, q = warp & 3;
    const int e = blockIdx.x * 2 + es;
    const int t = blockIdx.y;
    const float *xt = x + (size_t)t * hidden;
    const int se = hidden >> 7;               // elements per segment
    const int nc = se >> 3;                   // 8-element chunks per segment
    const int xpitch = nc * 32 + 16;
    const int wpitch = nc * 8 * (int)sizeof(WT) + (sizeof(WT) == 2 ? 32 : 16);
    unsigned char *xs = rsm;
    unsigned char *wrow0 = rsm + 128 * xpitch;
    {
        const uint32_t xs_s = (uint32_t)__cvta_generic_to_shared(xs);
        const int x4 = se / 4;                // float4 chunks per segment
        for (int f = threadIdx.x; f < hidden / 4; f += blockDim.x)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                         :: "r"(xs_s + (uint32_t)((f / x4) * xpitch + (f % x4) * 16)), "l"(xt + 4 * f)
                         : "memory");
        const int per_seg = nc * (int)sizeof(WT) / 2;      // 16-byte chunks per segment
        const int wq = hidden * (int)sizeof(WT) / 16;
        for (int k = 0; k < 2; k++) {
            const int ek = blockIdx.x * 2 + k;
            if (ek >= n_experts) break;
            const unsigned char *row = reinterpret_cast<const unsigned char *>(W + (size_t)ek * hidden);
            const uint32_t w_s = (uint32_t)__cvta_generic_to_shared(wrow0 + k * 128 * wpitch);
            for (int c = threadIdx.x; c < wq; c += blockDim.x)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                             :: "r"(w_s + (uint32_t)((c / per_seg) * wpitch + (c % per_seg) * 16)),
                                "l"(row + 16 * (size_t)c) : "memory");
        }
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
    }
    __syncthreads();
    const bool active = e < n_experts;
    const int seg = q * 32 + lane;
    const unsigned char *xl = xs + seg * xpitch;
    const unsigned char *wl = wrow0 + es * 128 * wpitch + seg * wpitch;

    // ---- fast pass: exact segment total, sum |p|
    double hs[4] = {0.0, 0.0, 0.0, 0.0}, ls[4] = {0.0, 0.0, 0.0, 0.0};
    double A0 = 0.0, A1 = 0.0;
    if (active) {
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
    if (lane == 0) { s_th[es][q] = h; s_tl[es][q] = l; s_A[es][q] = Aq; }
    __syncthreads();
    if (!active) return;
    // the row's exact total and sum |p| (same arithmetic in all four warps)
    double Sh = s_th[es][0], Sl = s_tl[es][0];
    double A = s_A[es][0];
    for (int k = 1; k < 4; k++) {
        double sum, err;
        two_sum(Sh, s_th[es][k], sum, err);
        const double low = __dadd_rn(__dadd_rn(Sl, s_tl[es][k]), err);
        two_sum(sum, low, Sh, Sl);
        A = __dadd_rn(A, s_A[es][k]);
    }
    const double u = 0x1p-53;
    const double n = (double)hidden;
    const double slack = 8.0 * u * fabs(Sh) + fabs(Sl);
    {
        const double gam = n * u / (1.0 - n * u);
        const double bound = (gam * A * (1.0 + 0x1p-20) + slack) * (1.0 + 0x1p-20) + 0x1p-1074;
        const float flo = (float)__dsub_rn(Sh, bound), fhi = (float)__dadd_rn(Sh, bound);
        if (flo == fhi) {
            if (q == 0 && lane == 0) {
                const float sc = __fdiv_rn(1.0f, __fadd_rn(1.0f, k3_expf(-flo)));
                score[(size_t)t * n_experts + e] = sc;
                choice[(size_t)t * n_experts + e] = bias ? __fadd_rn(sc, __ldg(bias + e)) : sc;
            }
            return;
        }
    }
    // ---- tight pass (this expert's four warps; named barrier 1 + es, 128 threads)
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
    if (lane == 0) s_q[es][q] = wq;
    asm volatile("bar.sync %0, 128;" :: "r"(1 + es) : "memory");
    // offsets: previous quarters' totals + the exclusive prefix of this warp's lane totals
    double off = 0.0;
    int G = 4096;
    for (int k = 0; k < q; k++) { off = __dadd_rn(off, __dadd_rn(s_th[es][k], s_tl[es][k])); G = min(G, s_q[es][k]); }
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
    if (lane == 0) s_bt[es][q] = bt;
    asm volatile("bar.sync %0, 128;" :: "r"(1 + es) : "memory");
    if (q != 0 || lane != 0) return;
    const double B = __dadd_rn(__dadd_rn(s_bt[es][0], s_bt[es][1]), __dadd_rn(s_bt[es][2], s_bt[es][3]));
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
        const unsigned char *wr = wrow0 + es * 128 * wpitch;
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
    const float sc = __fdiv_rn(1.0f, __fadd_rn(1.0f, k3_expf(-logit)));
    score[(size_t)t * n_experts + e] = sc;
    choice[(size_t)t * n_experts + e] = bias ? __fadd_rn(sc, __ldg(bias + e)) : sc;
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
    // the staged kernel needs hidden % 1024 == 0, 16-byte aligned rows and x, and its
    // shared-memory image (x plus two rows, padded) within the opt-in limit
    const size_t need = (size_t)hidden * 4 + (size_t)2 * hidden * sizeof(WT) + 128 * 16 * 3;
    const bool vec = (hidden % 1024) == 0 && (((uintptr_t)W | (uintptr_t)x) & 15u) == 0 &&
                     need <= 200 * 1024;
    if (vec) {
        // four warps (experts) per CTA: 96 CTAs for 384 experts, one wave over the SMs
        dim3 grid((n_experts + 1) / 2, T);
        const int nc = hidden >> 10;
        const size_t smem = (size_t)128 * (nc * 32 + 16) +
                            (size_t)2 * 128 * (nc * 8 * sizeof(WT) + (sizeof(WT) == 2 ? 32 : 16));
        static bool init = false;
        if (!init) { allow_smem_max(k_router_scores<WT>); init = true; }
        k_router_scores<WT><<<grid, 256, smem, s>>>(score, choice, x, W, bias, hidden, n_experts);
    } else {
        dim3 grid((n_experts + 7) / 8, T);
        k_router_scores_generic<WT><<<grid, 256, 0, s>>>(score, choice, x, W, bias, hidden, n_experts);
    }
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
