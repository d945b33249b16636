// k3_kda_layer.cu -- one KDA decode layer for B sequences (one token each), following
// k3_kda_layer (k3_ops.c:850-937) at T = 1, with bf16 projection weights:
//
//   1. one multi-segment GEMV of the normed input: q, k, v, g [P], b [H], f_a [D]
//   2. f_b GEMV: z = f_b(f_a x)                                               [P]
//   3. k_kda_head, one CTA per (sequence, head), thread j = channel:
//        ShortConv + SiLU on q, k, v (conv history updated in place)  k3_ops.c:875-878
//        L2Norm q and k over the head (sum of squares, eps 1e-6)      k3_ops.c:881-885
//        beta = sigmoid(b);  g = lb*sigmoid(exp(A_log[h])*(z+dt_bias)); alpha = exp(g)
//        q *= D^-0.5; the delta-rule step on the head's state tile, staged in shared
//        memory, one column per thread in the CPU's order       k3_ops.c:186-243, 916-924
//        head RMSNorm with o_norm, THEN times sigmoid(g)         k3_ops.c:927-933
//   4. o_proj GEMV accumulated into the residual stream.
//
// State per sequence: S [H][D][D] fp32 followed by the conv history [3][P][conv_k-1]
// (q, k, v channels), the CPU engine's layout (k3.h:464-466).
#include "k3_common.cuh"
#include "k3_ops.cuh"

namespace k3 {

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ double block_sum_dd(double v, double *red, int nwarps)
{
    v = warp_sum_d(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
    for (int i = 0; i < nwarps; i++) s += red[i];
    return s;
}

struct KdaHeadArgs {
    const float *qp, *kp, *vp, *gp, *bp, *z;   // projections [B][P] / [B][H]
    const float *q_conv, *k_conv, *v_conv;     // [P][K]
    const float *A_log, *dt_bias, *o_norm;     // [H], [P], [D]
    float *state;                              // [B][state floats]
    float *heads;                              // [B][P]
    int H, D, K;
    float lb, eps;
    size_t state_stride;                       // floats per sequence
};

__device__ __forceinline__ float conv_silu(const float *w, float *hist, float cur, int K)
{
    const int hst = K - 1;
    float acc = __fmul_rn(w[hst], cur);
    for (int j = 0; j < hst; j++) acc = __fadd_rn(acc, __fmul_rn(w[j], hist[j]));
    for (int j = 0; j + 1 < hst; j++) hist[j] = hist[j + 1];
    if (hst > 0) hist[hst - 1] = cur;
    return __fmul_rn(acc, sigm(acc));
}

// grid (H, B), blockDim = D (<= 128, multiple of 32). Shared: D*D state + 3*D vectors.
// KC = conv_k when it is a compile-time constant (4 for the K3 model): every global load
// of the thread (projections, gates, conv weights and histories) is then issued before any
// arithmetic; KC = 0 handles any conv_k.
template <int KC>
__global__ void __launch_bounds__(128) k_kda_head(KdaHeadArgs A)
{
    extern __shared__ __align__(16) float sh[];
    __shared__ double red[8];
    __shared__ __align__(8) unsigned long long st_bar;
    const int h = blockIdx.x, b = blockIdx.y, j = threadIdx.x;
    const int D = A.D, H = A.H, K = KC > 0 ? KC : A.K, P = H * D, hst = K - 1;
    float *St = sh;
    float *qs = St + D * D, *ks = qs + D, *as = ks + D;
    float *S = A.state + (size_t)b * A.state_stride + (size_t)h * D * D;
    float *conv = A.state + (size_t)b * A.state_stride + (size_t)H * D * D;
    const int nw = blockDim.x >> 5;
    const int c = h * D + j;
    const size_t bp = (size_t)b * P + c;
    float qv, kv, vv, gpv, zv, dtb, bpv, alog, onw;
    float *hq = conv + (size_t)c * hst;
    float *hk = conv + (size_t)P * hst + (size_t)c * hst;
    float *hv = conv + (size_t)2 * P * hst + (size_t)c * hst;
    // The state tile (written by this layer's previous step, never by the kernels just
    // before) streams in as one bulk copy, requested before the programmatic wait.
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&st_bar);
    const bool bulk_ok = (((uintptr_t)S) & 15u) == 0;
    if (j == 0 && bulk_ok) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(bar));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint32_t bytes = (uint32_t)(D * D * 4);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     :: "r"((uint32_t)__cvta_generic_to_shared(St)), "l"(S), "r"(bytes), "r"(bar) : "memory");
    }
    if constexpr (KC > 0) {
        // every load of the thread is issued before any arithmetic; the weights, the conv
        // history and the per-head constants before the programmatic wait as well
        float wq[KC], wk[KC], wv[KC], xq[KC], xk[KC], xv[KC];
#pragma unroll
        for (int t = 0; t < KC; t++) {
            wq[t] = A.q_conv[(size_t)c * KC + t];
            wk[t] = A.k_conv[(size_t)c * KC + t];
            wv[t] = A.v_conv[(size_t)c * KC + t];
        }
#pragma unroll
        for (int t = 0; t < KC - 1; t++) { xq[t] = hq[t]; xk[t] = hk[t]; xv[t] = hv[t]; }
        dtb = A.dt_bias[c];
        alog = A.A_log[h];
        onw = A.o_norm[j];
        pdl_wait();
        pdl_trigger();
        xq[KC - 1] = A.qp[bp]; xk[KC - 1] = A.kp[bp]; xv[KC - 1] = A.vp[bp];
        gpv = A.gp[bp]; zv = A.z[bp];
        bpv = A.bp[(size_t)b * H + h];
        if (!bulk_ok) {
            const float4 *S4 = reinterpret_cast<const float4 *>(S);
            float4 *T4 = reinterpret_cast<float4 *>(St);
#pragma unroll 8
            for (int f = j; f < D * D / 4; f += blockDim.x) T4[f] = S4[f];
        }
        // ShortConv + SiLU in the CPU's order: the newest input times the last tap, then the
        // history oldest first (k3_ops.c:875-878); the history shifts in place
        float aq = __fmul_rn(wq[KC - 1], xq[KC - 1]);
        float ak = __fmul_rn(wk[KC - 1], xk[KC - 1]);
        float av = __fmul_rn(wv[KC - 1], xv[KC - 1]);
#pragma unroll
        for (int t = 0; t < KC - 1; t++) {
            aq = __fadd_rn(aq, __fmul_rn(wq[t], xq[t]));
            ak = __fadd_rn(ak, __fmul_rn(wk[t], xk[t]));
            av = __fadd_rn(av, __fmul_rn(wv[t], xv[t]));
        }
#pragma unroll
        for (int t = 0; t < KC - 1; t++) { hq[t] = xq[t + 1]; hk[t] = xk[t + 1]; hv[t] = xv[t + 1]; }
        qv = __fmul_rn(aq, sigm(aq));
        kv = __fmul_rn(ak, sigm(ak));
        vv = __fmul_rn(av, sigm(av));
    } else {
        pdl_wait();
        pdl_trigger();
        if (!bulk_ok) {
            const float4 *S4 = reinterpret_cast<const float4 *>(S);
            float4 *T4 = reinterpret_cast<float4 *>(St);
#pragma unroll 8
            for (int f = j; f < D * D / 4; f += blockDim.x) T4[f] = S4[f];
        }
        // ShortConv + SiLU (history in place)
        float hist[15];
        for (int t = 0; t < hst; t++) hist[t] = hq[t];
        qv = conv_silu(A.q_conv + (size_t)c * K, hist, A.qp[bp], K);
        for (int t = 0; t < hst; t++) hq[t] = hist[t];
        for (int t = 0; t < hst; t++) hist[t] = hk[t];
        kv = conv_silu(A.k_conv + (size_t)c * K, hist, A.kp[bp], K);
        for (int t = 0; t < hst; t++) hk[t] = hist[t];
        for (int t = 0; t < hst; t++) hist[t] = hv[t];
        vv = conv_silu(A.v_conv + (size_t)c * K, hist, A.vp[bp], K);
        for (int t = 0; t < hst; t++) hv[t] = hist[t];
        gpv = A.gp[bp]; zv = A.z[bp]; dtb = A.dt_bias[c];
        bpv = A.bp[(size_t)b * H + h]; alog = A.A_log[h]; onw = A.o_norm[j];
    }
    // L2Norm q and k over the head
    const double sq = block_sum_dd((double)qv * (double)qv, red, nw);
    const double sk = block_sum_dd((double)kv * (double)kv, red, nw);
    qv = __fmul_rn(qv, (float)(1.0 / sqrt(sq + (double)1e-6f)));
    kv = __fmul_rn(kv, (float)(1.0 / sqrt(sk + (double)1e-6f)));
    qv = __fmul_rn(qv, 1.0f / sqrtf((float)D));
    // beta and the decay chain
    const float beta = sigm(bpv);
    const float a = expf(alog);
    const float gdec = __fmul_rn(A.lb, sigm(__fmul_rn(a, __fadd_rn(zv, dtb))));
    qs[j] = qv;
    ks[j] = kv;
    as[j] = expf(gdec);
    if (bulk_ok) {
        // the state tile has landed (bounded wait: on a time-out the device error flag is
        // raised and the tile is read as it is)
        uint32_t ok = 0;
        const long long t0 = clock64();
        do {
            asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
                         "selp.b32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(bar) : "memory");
            if (!ok && clock64() - t0 > 4000000000LL) { k3_raise(K3D_ETIMEOUT, K3_SITE_KDA); break; }
        } while (!ok);
    }
    __syncthreads();
    // delta-rule step, column j (the CPU's order and roundings)
    float u = 0.0f;
    for (int i = 0; i < D; i++) {
        const float si = __fmul_rn(St[i * D + j], as[i]);
        St[i * D + j] = si;
        if (ks[i] != 0.0f) u = __fadd_rn(u, __fmul_rn(ks[i], si));
    }
    const float d = __fsub_rn(vv, u);
    float o = 0.0f;
    for (int i = 0; i < D; i++) {
        float si = St[i * D + j];
        if (ks[i] != 0.0f) si = __fadd_rn(si, __fmul_rn(__fmul_rn(ks[i], beta), d));
        if (qs[i] != 0.0f) o = __fadd_rn(o, __fmul_rn(qs[i], si));
        S[(size_t)i * D + j] = si;
    }
    // head RMSNorm, then the output gate
    const double so = block_sum_dd((double)o * (double)o, red, nw);
    const float inv = (float)(1.0 / sqrt(so / (double)D + (double)A.eps));
    o = __fmul_rn(__fmul_rn(onw, o), inv);
    o = __fmul_rn(o, sigm(gpv));
    A.heads[bp] = o;
}

// Column j of the step from the state still in memory, with the CPU's skips of zero keys
// and queries (k_kda_head's loops): the register kernel's fallback when its dot products
// came out non-finite. Writes the column back and returns o.
template <int DT>
__device__ __forceinline__ float kda_column_exact(float *S, int j, const float *as, const float *ks,
                                               const float *kbs, const float *qs, float vv)
{
    float u = 0.0f;
    for (int i = 0; i < DT; i++) {
        const float si = __fmul_rn(S[(size_t)i * DT + j], as[i]);
        if (ks[i] != 0.0f) u = __fadd_rn(u, __fmul_rn(ks[i], si));
    }
    const float d = __fsub_rn(vv, u);
    float o = 0.0f;
    for (int i = 0; i < DT; i++) {
        float si = __fmul_rn(S[(size_t)i * DT + j], as[i]);
        if (ks[i] != 0.0f) si = __fadd_rn(si, __fmul_rn(kbs[i], d));
        if (qs[i] != 0.0f) o = __fadd_rn(o, __fmul_rn(qs[i], si));
        S[(size_t)i * DT + j] = si;
    }
    return o;
}

// The same head with the state column in registers: thread j loads column j of the head's
// state (DT coalesced rows, all issued before the programmatic wait), runs both passes of
// the step on its registers and stores the column back. No shared-memory tile, no bulk
// copy, and the two dependent fadd chains (u, then o) are the only serial part: the
// shared-tile kernel paid a shared-memory round trip per row in each pass with four warps
// per SM to hide it. Same operations in the same order, so bit-identical to k_kda_head.
// The per-row operands come four rows at a time (16-byte shared loads), and the two dot
// products add every row's product without the zero test: u and o start at +0 and a sum
// in round-to-nearest is -0 only when both terms are, so adding the +-0 product of a zero
// key or query changes nothing while the state is finite; a non-finite u or o (the only
// way a skipped product could have mattered) recomputes the column with the skips
// (kda_column_exact). The state update keeps its test.
template <int KC, int DT>
__global__ void __launch_bounds__(DT) k_kda_head_reg(const __grid_constant__ KdaHeadArgs A)
{
    static_assert(KC > 0 && DT % 32 == 0 && DT <= 128, "register head: KC > 0, DT in 32..128");
    constexpr int NW = DT / 32;
    __shared__ __align__(16) float qs[DT], ks[DT], kbs[DT], as[DT];
    __shared__ double red[2][NW];
    const int h = blockIdx.x, b = blockIdx.y, j = threadIdx.x;
    const int H = A.H, P = H * DT, lane = j & 31, warp = j >> 5;
    float *S = A.state + (size_t)b * A.state_stride + (size_t)h * DT * DT;
    float *conv = A.state + (size_t)b * A.state_stride + (size_t)H * DT * DT;
    const int c = h * DT + j;
    const size_t bp = (size_t)b * P + c;
    float *hq = conv + (size_t)c * (KC - 1);
    float *hk = conv + (size_t)P * (KC - 1) + (size_t)c * (KC - 1);
    float *hv = conv + (size_t)2 * P * (KC - 1) + (size_t)c * (KC - 1);
    // this layer's previous step wrote the state and the conv history; no kernel since
    float s[DT];
#pragma unroll
    for (int i = 0; i < DT; i++) s[i] = S[(size_t)i * DT + j];
    float wq[KC], wk[KC], wv[KC], xq[KC], xk[KC], xv[KC];
#pragma unroll
    for (int t = 0; t < KC; t++) {
        wq[t] = A.q_conv[(size_t)c * KC + t];
        wk[t] = A.k_conv[(size_t)c * KC + t];
        wv[t] = A.v_conv[(size_t)c * KC + t];
    }
#pragma unroll
    for (int t = 0; t < KC - 1; t++) { xq[t] = hq[t]; xk[t] = hk[t]; xv[t] = hv[t]; }
    const float dtb = A.dt_bias[c], alog = A.A_log[h], onw = A.o_norm[j];
    pdl_wait();
    pdl_trigger();
    xq[KC - 1] = A.qp[bp]; xk[KC - 1] = A.kp[bp]; xv[KC - 1] = A.vp[bp];
    const float gpv = A.gp[bp], zv = A.z[bp], bpv = A.bp[(size_t)b * H + h];
    float aq = __fmul_rn(wq[KC - 1], xq[KC - 1]);
    float ak = __fmul_rn(wk[KC - 1], xk[KC - 1]);
    float av = __fmul_rn(wv[KC - 1], xv[KC - 1]);
#pragma unroll
    for (int t = 0; t < KC - 1; t++) {
        aq = __fadd_rn(aq, __fmul_rn(wq[t], xq[t]));
        ak = __fadd_rn(ak, __fmul_rn(wk[t], xk[t]));
        av = __fadd_rn(av, __fmul_rn(wv[t], xv[t]));
    }
#pragma unroll
    for (int t = 0; t < KC - 1; t++) { hq[t] = xq[t + 1]; hk[t] = xk[t + 1]; hv[t] = xv[t + 1]; }
    float qv = __fmul_rn(aq, sigm(aq));
    float kv = __fmul_rn(ak, sigm(ak));
    const float vv = __fmul_rn(av, sigm(av));
    // both L2 norms in one exchange, each summed as block_sum_dd sums it
    {
        const double q2 = warp_sum_d((double)qv * (double)qv), k2 = warp_sum_d((double)kv * (double)kv);
        if (lane == 0) { red[0][warp] = q2; red[1][warp] = k2; }
    }
    __syncthreads();
    double sq = 0.0, sk = 0.0;
#pragma unroll
    for (int i = 0; i < NW; i++) { sq += red[0][i]; sk += red[1][i]; }
    qv = __fmul_rn(qv, (float)(1.0 / sqrt(sq + (double)1e-6f)));
    kv = __fmul_rn(kv, (float)(1.0 / sqrt(sk + (double)1e-6f)));
    qv = __fmul_rn(qv, 1.0f / sqrtf((float)A.D));
    const float beta = sigm(bpv);
    const float a = expf(alog);
    const float gdec = __fmul_rn(A.lb, sigm(__fmul_rn(a, __fadd_rn(zv, dtb))));
    qs[j] = qv;
    ks[j] = kv;
    kbs[j] = __fmul_rn(kv, beta);
    as[j] = expf(gdec);
    __syncthreads();
    float u = 0.0f;
#pragma unroll
    for (int i4 = 0; i4 < DT / 4; i4++) {
        const float4 a4 = reinterpret_cast<const float4 *>(as)[i4];
        const float4 k4 = reinterpret_cast<const float4 *>(ks)[i4];
        const float ar[4] = {a4.x, a4.y, a4.z, a4.w}, kr[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int t = 0; t < 4; t++) {
            s[4 * i4 + t] = __fmul_rn(s[4 * i4 + t], ar[t]);
            u = __fadd_rn(u, __fmul_rn(kr[t], s[4 * i4 + t]));
        }
    }
    const float d = __fsub_rn(vv, u);
    float o = 0.0f;
#pragma unroll
    for (int i4 = 0; i4 < DT / 4; i4++) {
        const float4 k4 = reinterpret_cast<const float4 *>(ks)[i4];
        const float4 b4 = reinterpret_cast<const float4 *>(kbs)[i4];
        const float4 q4 = reinterpret_cast<const float4 *>(qs)[i4];
        const float kr[4] = {k4.x, k4.y, k4.z, k4.w}, br[4] = {b4.x, b4.y, b4.z, b4.w};
        const float qr[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
        for (int t = 0; t < 4; t++) {
            float si = s[4 * i4 + t];
            if (kr[t] != 0.0f) si = __fadd_rn(si, __fmul_rn(br[t], d));
            o = __fadd_rn(o, __fmul_rn(qr[t], si));
            s[4 * i4 + t] = si;
        }
    }
    // the column goes back after the loop: a store through a generic pointer between the
    // loop's shared-memory reads would order every later read after it
    if (isfinite(u) && isfinite(o)) {
#pragma unroll
        for (int i = 0; i < DT; i++) S[(size_t)i * DT + j] = s[i];
    } else {
        o = kda_column_exact<DT>(S, j, as, ks, kbs, qs, vv);
    }
    {
        const double o2 = warp_sum_d((double)o * (double)o);
        if (lane == 0) red[0][warp] = o2;            // red[0] was last read before the
    }                                                // barrier above
    __syncthreads();
    double so = 0.0;
#pragma unroll
    for (int i = 0; i < NW; i++) so += red[0][i];
    const float inv = (float)(1.0 / sqrt(so / (double)DT + (double)A.eps));
    o = __fmul_rn(__fmul_rn(onw, o), inv);
    o = __fmul_rn(o, sigm(gpv));
    A.heads[bp] = o;
}

// The same head split over a cluster of DT / 32 one-warp CTAs: CTA r of the cluster owns
// value columns [32 r, 32 r + 32) (lane = column), so a head's 64 KB state tile streams
// through DT / 32 SMs instead of one (at batch 1, 256 CTAs on 148 SMs instead of 64). Every
// CTA computes the conv, L2 norms, gates and decays of all DT key channels (lane l holds
// channels l + 32 g), which are cheap; the head RMSNorm's sum of o^2 is combined across the
// cluster through distributed shared memory. Each sum keeps the order of k_kda_head (a
// warp's butterfly over 32 consecutive channels, then the 32-channel groups in order), so
// the result is bit-identical to it. The q and k conv histories are written by CTA 0 of
// the cluster only (every CTA computes the same values); each CTA writes its own v
// channels.
__device__ __forceinline__ uint32_t cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ double ld_dsmem_f64(const double *local, uint32_t rank)
{
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(local);
    uint32_t ra;
    double v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(ra) : "memory");
    return v;
}

template <int KC, int DT>
__global__ void __launch_bounds__(32) k_kda_head_cl(const __grid_constant__ KdaHeadArgs A)
{
    static_assert(KC > 0 && DT % 32 == 0 && DT <= 128, "cluster head: KC > 0, DT in 32..128");
    constexpr int NG = DT / 32;                      // channel groups = CTAs per head
    __shared__ float qs[DT], ks[DT], kbs[DT], as[DT];
    __shared__ double s_o2;
    const int l = threadIdx.x;
    const int cr = (int)cluster_rank();
    const int h = blockIdx.x / NG, b = blockIdx.y;
    const int H = A.H, P = H * DT;
    const int j = cr * 32 + l;                       // this lane's value column
    float *S = A.state + (size_t)b * A.state_stride + (size_t)h * DT * DT;
    float *conv = A.state + (size_t)b * A.state_stride + (size_t)H * DT * DT;
    const size_t rowb = (size_t)b * P + (size_t)h * DT;
    float s[DT];
#pragma unroll
    for (int i = 0; i < DT; i++) s[i] = S[(size_t)i * DT + j];
    // key channels c_g = h * DT + l + 32 g: q and k conv taps and histories, the decay inputs
    float wq[NG][KC], wk[NG][KC], xq[NG][KC], xk[NG][KC], dtb[NG];
#pragma unroll
    for (int g = 0; g < NG; g++) {
        const int c = h * DT + l + 32 * g;
#pragma unroll
        for (int t = 0; t < KC; t++) {
            wq[g][t] = A.q_conv[(size_t)c * KC + t];
            wk[g][t] = A.k_conv[(size_t)c * KC + t];
        }
#pragma unroll
        for (int t = 0; t < KC - 1; t++) {
            xq[g][t] = conv[(size_t)c * (KC - 1) + t];
            xk[g][t] = conv[(size_t)P * (KC - 1) + (size_t)c * (KC - 1) + t];
        }
        dtb[g] = A.dt_bias[c];
    }
    // value channel j
    const int cj = h * DT + j;
    float wv[KC], xv[KC];
    float *hv = conv + (size_t)2 * P * (KC - 1) + (size_t)cj * (KC - 1);
#pragma unroll
    for (int t = 0; t < KC; t++) wv[t] = A.v_conv[(size_t)cj * KC + t];
#pragma unroll
    for (int t = 0; t < KC - 1; t++) xv[t] = hv[t];
    const float alog = A.A_log[h], onw = A.o_norm[j];
    pdl_wait();
    pdl_trigger();
    float zv[NG];
#pragma unroll
    for (int g = 0; g < NG; g++) {
        xq[g][KC - 1] = A.qp[rowb + l + 32 * g];
        xk[g][KC - 1] = A.kp[rowb + l + 32 * g];
        zv[g] = A.z[rowb + l + 32 * g];
    }
    xv[KC - 1] = A.vp[rowb + j];
    const float gpv = A.gp[rowb + j], bpv = A.bp[(size_t)b * H + h];
    // ShortConv + SiLU in the CPU's order (k3_ops.c:875-878)
    float qv[NG], kv[NG];
#pragma unroll
    for (int g = 0; g < NG; g++) {
        float aq = __fmul_rn(wq[g][KC - 1], xq[g][KC - 1]);
        float ak = __fmul_rn(wk[g][KC - 1], xk[g][KC - 1]);
#pragma unroll
        for (int t = 0; t < KC - 1; t++) {
            aq = __fadd_rn(aq, __fmul_rn(wq[g][t], xq[g][t]));
            ak = __fadd_rn(ak, __fmul_rn(wk[g][t], xk[g][t]));
        }
        qv[g] = __fmul_rn(aq, sigm(aq));
        kv[g] = __fmul_rn(ak, sigm(ak));
    }
    float av = __fmul_rn(wv[KC - 1], xv[KC - 1]);
#pragma unroll
    for (int t = 0; t < KC - 1; t++) av = __fadd_rn(av, __fmul_rn(wv[t], xv[t]));
    const float vv = __fmul_rn(av, sigm(av));
#pragma unroll
    for (int t = 0; t < KC - 1; t++) hv[t] = xv[t + 1];
    // L2 norms: warp sums per 32-channel group, the groups added in order (block_sum_dd's)
    double sq = 0.0, sk = 0.0;
#pragma unroll
    for (int g = 0; g < NG; g++) {
        sq += warp_sum_d((double)qv[g] * (double)qv[g]);
        sk += warp_sum_d((double)kv[g] * (double)kv[g]);
    }
    const float iq = (float)(1.0 / sqrt(sq + (double)1e-6f)), ik = (float)(1.0 / sqrt(sk + (double)1e-6f));
    const float qscale = 1.0f / sqrtf((float)A.D);
    const float beta = sigm(bpv);
    const float a = expf(alog);
#pragma unroll
    for (int g = 0; g < NG; g++) {
        const int i = l + 32 * g;
        const float qn = __fmul_rn(__fmul_rn(qv[g], iq), qscale);
        const float kn = __fmul_rn(kv[g], ik);
        qs[i] = qn;
        ks[i] = kn;
        kbs[i] = __fmul_rn(kn, beta);
        as[i] = expf(__fmul_rn(A.lb, sigm(__fmul_rn(a, __fadd_rn(zv[g], dtb[g])))));
    }
    __syncwarp();
    float u = 0.0f;
#pragma unroll
    for (int i = 0; i < DT; i++) {
        s[i] = __fmul_rn(s[i], as[i]);
        const float ki = ks[i];
        if (ki != 0.0f) u = __fadd_rn(u, __fmul_rn(ki, s[i]));
    }
    const float d = __fsub_rn(vv, u);
    float o = 0.0f;
#pragma unroll
    for (int i = 0; i < DT; i++) {
        float si = s[i];
        if (ks[i] != 0.0f) si = __fadd_rn(si, __fmul_rn(kbs[i], d));
        const float qi = qs[i];
        if (qi != 0.0f) o = __fadd_rn(o, __fmul_rn(qi, si));
        s[i] = si;
    }
    // the column goes back after the loop: a store through a generic pointer between the
    // loop's shared-memory reads would order every later read after it
#pragma unroll
    for (int i = 0; i < DT; i++) S[(size_t)i * DT + j] = s[i];
    // head RMSNorm: this CTA's 32 columns are one group; the cluster's groups in order
    const double o2 = warp_sum_d((double)o * (double)o);
    if (l == 0) s_o2 = o2;
    cluster_sync_all();
    // every CTA of the cluster has read the q and k histories by now
    if (cr == 0) {
#pragma unroll
        for (int g = 0; g < NG; g++) {
            const int c = h * DT + l + 32 * g;
#pragma unroll
            for (int t = 0; t < KC - 1; t++) {
                conv[(size_t)c * (KC - 1) + t] = xq[g][t + 1];
                conv[(size_t)P * (KC - 1) + (size_t)c * (KC - 1) + t] = xk[g][t + 1];
            }
        }
    }
    double so = 0.0;
#pragma unroll
    for (int g = 0; g < NG; g++) so += ld_dsmem_f64(&s_o2, (uint32_t)g);
    cluster_sync_all();                              // every CTA has read every s_o2
    const float inv = (float)(1.0 / sqrt(so / (double)DT + (double)A.eps));
    o = __fmul_rn(__fmul_rn(onw, o), inv);
    o = __fmul_rn(o, sigm(gpv));
    A.heads[rowb + j] = o;
}

static size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace k3

using namespace k3;

extern "C" {

size_t k3d_kda_layer_ws_bytes(const K3dKdaShape *s, int B)
{
    if (!s || B < 1) return 0;
    const size_t P = (size_t)s->heads * s->head_dim;
    return 6 * al256((size_t)B * P * 4) + al256((size_t)B * s->heads * 4) +
           al256((size_t)B * s->head_dim * 4) + 256;
}

size_t k3d_kda_state_floats(const K3dKdaShape *s)
{
    const size_t P = (size_t)s->heads * s->head_dim;
    return (size_t)s->heads * s->head_dim * s->head_dim + 3 * P * (size_t)(s->conv_k - 1);
}

}  // extern "C"

// Which head kernel runs (k3d_set_kda_head_kernel): 0 chooses (the register-column kernel
// for up to four sequences, else the shared-tile kernel); 1 the shared-tile kernel; 2 the
// register-column kernel (one CTA per head); 3 the cluster kernel (head_dim / 32 one-warp
// CTAs per head). 2 and 3 apply where head_dim is 32, 64 or 128 and conv_k is 4 (else 1).
static int g_kda_head_kernel = 0;

// The layer; with ni, xn is the raw residual and the projection GEMV normalises it.
static int kda_layer_decode(float *h, const float *xn, const NormIn *ni, const K3dKdaW *w,
                            const K3dKdaShape *s, int B, float *state, void *ws, size_t ws_bytes,
                            int accumulate = 1)
{
    K3_TRY(ensure_ctx());
    if (!h || !xn || !w || !s || !state || !ws) return fail(K3D_EINVAL, "kda layer null pointer");
    if (!w->q || !w->k || !w->v || !w->g || !w->b || !w->f_a || !w->f_b || !w->o ||
        !w->q_conv || !w->k_conv || !w->v_conv || !w->A_log || !w->dt_bias || !w->o_norm)
        return fail(K3D_EINVAL, "kda layer weight missing");
    const int H = s->heads, D = s->head_dim, P = H * D;
    if (D < 32 || D > 128 || D % 32 || s->conv_k < 1 || s->conv_k > 16 || B < 1 || B > 256)
        return fail(K3D_EINVAL, "kda layer: head_dim %d (32..128, multiple of 32), conv_k %d, B %d (1..256)",
                    D, s->conv_k, B);
    if (ws_bytes < k3d_kda_layer_ws_bytes(s, B)) return fail(K3D_EINVAL, "kda layer workspace");
    char *p = (char *)ws;
    auto take = [&](size_t bytes) { char *r = p; p += al256(bytes); return (float *)r; };
    float *qp = take((size_t)B * P * 4), *kp = take((size_t)B * P * 4), *vp = take((size_t)B * P * 4);
    float *gp = take((size_t)B * P * 4), *z = take((size_t)B * P * 4), *heads = take((size_t)B * P * 4);
    float *bp = take((size_t)B * H * 4), *fa = take((size_t)B * D * 4);
    cudaStream_t st = stream();
    prof_begin("kda.proj_in");
    const uint16_t *Ws[6] = {w->q, w->k, w->v, w->g, w->b, w->f_a};
    float *Ys[6] = {qp, kp, vp, gp, bp, fa};
    const int rows[6] = {P, P, P, P, H, D};
    K3_TRY(gemv_bf16_multi(6, Ws, Ys, rows, xn, s->hidden, B, st, ni));
    K3_TRY(gemv_bf16(z, fa, w->f_b, D, P, B, 0, st));
    prof_end("kda.proj_in");
    prof_begin("kda.core");
    KdaHeadArgs A;
    A.qp = qp; A.kp = kp; A.vp = vp; A.gp = gp; A.bp = bp; A.z = z;
    A.q_conv = w->q_conv; A.k_conv = w->k_conv; A.v_conv = w->v_conv;
    A.A_log = w->A_log; A.dt_bias = w->dt_bias; A.o_norm = w->o_norm;
    A.state = state; A.heads = heads;
    A.H = H; A.D = D; A.K = s->conv_k; A.lb = s->gate_lb; A.eps = s->eps;
    A.state_stride = k3d_kda_state_floats(s);
    const size_t smem = ((size_t)D * D + 3 * (size_t)D) * 4;
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) {
        allow_smem_max(k_kda_head<4>);
        allow_smem_max(k_kda_head<0>);
        init |= dev_bit();
    }
    // default: the register-column kernel for up to four sequences (64 to 256 CTAs), the
    // shared-tile kernel above (the register kernel's 186 registers per thread cost it
    // occupancy when there are thousands of CTAs)
    const int kind = g_kda_head_kernel == 0 ? (B <= 4 ? 2 : 1) : g_kda_head_kernel;
    const bool cl = kind == 3 && s->conv_k == 4;
    const bool reg = kind == 2 && s->conv_k == 4;
    if (cl && D == 128) launch_pdl_cluster(k_kda_head_cl<4, 128>, dim3(H * 4, B), dim3(32), 0, st, 4, A);
    else if (cl && D == 64) launch_pdl_cluster(k_kda_head_cl<4, 64>, dim3(H * 2, B), dim3(32), 0, st, 2, A);
    else if (cl && D == 32) launch_pdl_cluster(k_kda_head_cl<4, 32>, dim3(H, B), dim3(32), 0, st, 1, A);
    else if (reg && D == 128) launch_pdl(k_kda_head_reg<4, 128>, dim3(H, B), dim3(D), 0, st, A);
    else if (reg && D == 64) launch_pdl(k_kda_head_reg<4, 64>, dim3(H, B), dim3(D), 0, st, A);
    else if (reg && D == 32) launch_pdl(k_kda_head_reg<4, 32>, dim3(H, B), dim3(D), 0, st, A);
    else if (s->conv_k == 4) launch_pdl(k_kda_head<4>, dim3(H, B), dim3(D), smem, st, A);
    else launch_pdl(k_kda_head<0>, dim3(H, B), dim3(D), smem, st, A);
    note_launch();
    K3_TRY(check_launch("kda head"));
    prof_end("kda.core");
    prof_begin("kda.proj_out");
    K3_TRY(gemv_bf16(h, heads, w->o, P, s->hidden, B, accumulate, st));
    prof_end("kda.proj_out");
    return K3D_OK;
}

extern "C" {

int k3d_set_kda_head_kernel(int kind)
{
    if (kind < 0 || kind > 3) return fail(K3D_EINVAL, "k3d_set_kda_head_kernel(%d): 0 to 3", kind);
    g_kda_head_kernel = kind;
    return K3D_OK;
}

int k3d_kda_layer_decode(float *h, const float *xn, const K3dKdaW *w, const K3dKdaShape *s,
                         int B, float *state, void *ws, size_t ws_bytes)
{
    return kda_layer_decode(h, xn, nullptr, w, s, B, state, ws, ws_bytes);
}

int k3d_kda_layer_decode_normed(float *h, const float *norm_w, float eps, const K3dKdaW *w,
                                const K3dKdaShape *s, int B, float *state, void *ws,
                                size_t ws_bytes)
{
    if (!norm_w) return fail(K3D_EINVAL, "kda layer: null norm weights");
    const NormIn ni{norm_w, eps};
    return kda_layer_decode(h, h, &ni, w, s, B, state, ws, ws_bytes);
}

int k3d_kda_layer_decode_normed_out(float *out, const float *h, const float *norm_w, float eps,
                                    const K3dKdaW *w, const K3dKdaShape *s, int B, float *state,
                                    void *ws, size_t ws_bytes, int accumulate)
{
    if (!norm_w || !out) return fail(K3D_EINVAL, "kda layer: null norm weights or output");
    const NormIn ni{norm_w, eps};
    return kda_layer_decode(out, h, &ni, w, s, B, state, ws, ws_bytes, accumulate ? 1 : 0);
}

}  // extern "C"
