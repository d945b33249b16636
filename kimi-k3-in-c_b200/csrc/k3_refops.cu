// k3_refops.cu -- the composite operators of include/k3/k3.h with the CPU engine's own
// semantics (latent MoE with SiTU-GLU, NoPE MLA over an expanded fp32 KV cache, the full
// KDA layer, the decoder layer with Attention Residuals), on the device.
//
//   k3_mla_cached / k3_mla       k3_ops.c:321-416
//   k3_moe / k3_moe_prefill      k3_ops.c:556-825
//   k3_kda_layer                 k3_ops.c:850-937
//   k3_decoder_layer[_inc]       k3_ops.c:964-1062
//   k3_*_scratch                 the reference sizers (k3_ops.c:519-535, 658-666, 839-848,
//                                940-953); returned for API compatibility
//
// These run the reference's order of operations with the sm_100a building blocks
// (GEMVs, router, KDA recurrence, norms); they serve drop-in callers and the reference's
// own fixtures. Host arguments are staged (k3.h, POINTERS). The caller's `scratch` is not
// needed: the library keeps its own device workspace. The decode hot path at the
// benchmark shapes is the k3d_* family in k3_cuda.h.
#include <cstdio>
#include <cstring>
#include <vector>

#include "k3_common.cuh"
#include "k3_ops.cuh"

namespace k3 {

int kda_seq(float *S, float *o, const float *q, const float *k, const float *v,
            const float *alpha, const float *beta, int T, int H, int dk, int dv, cudaStream_t st);
int shortconv(float *y, const float *x, const float *w, float *state, int channels, int k,
              int T, cudaStream_t s);
int kda_decay(float *g, float *alpha, const float *z, const float *A_log, const float *dt_bias,
              int H, int D, float lb, cudaStream_t s);
int attn_res(float *out, const float *src, const float *fold, int nsrc, int n, float eps,
             cudaStream_t s);

__device__ __forceinline__ float sgm(float x) { return 1.0f / (1.0f + expf(-x)); }

// rows of n: v *= 1/sqrt(sum v^2 + eps)  (l2norm_, k3_ops.c:831-837)
__global__ void k_l2norm_rows(float *v, int n, float eps)
{
    __shared__ double red[32];
    float *r = v + (size_t)blockIdx.x * n;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fma((double)r[i], (double)r[i], ss);
    ss = warp_sum_d(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += red[i];
    const float inv = (float)(1.0 / sqrt(t + (double)eps));
    for (int i = threadIdx.x; i < n; i += blockDim.x) r[i] = __fmul_rn(r[i], inv);
}

// elementwise helpers
__global__ void k_sigmoid(float *v, size_t n)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        v[i] = sgm(v[i]);
}
__global__ void k_scale(float *v, size_t n, float s)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        v[i] = __fmul_rn(v[i], s);
}
__global__ void k_gate_mul(float *v, const float *g, size_t n)   // v *= sigmoid(g)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        v[i] = __fmul_rn(v[i], sgm(g[i]));
}
__global__ void k_axpy_ordered(float *acc, const float *w, int j, const float *x, size_t n)
{   // acc += w[j] * x with a separate multiply and add (k3_ops.c:642)
    const float wj = w[j];
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        acc[i] = __fadd_rn(acc[i], __fmul_rn(wj, x[i]));
}
__global__ void k_add(float *y, const float *x, size_t n)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], x[i]);
}
__global__ void k_mul2(float *y, const float *a, const float *b, size_t n)   // y = a * b
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __fmul_rn(a[i], b[i]);
}

static int nb(size_t n)
{
    size_t b = (n + 255) / 256;
    const size_t cap = (size_t)sm_count() * 8;
    if (b > cap) b = cap;
    return b < 1 ? 1 : (int)b;
}

#define EW(kernel, n, ...) do { kernel<<<nb(n), 256, 0, stream()>>>(__VA_ARGS__); note_launch(); \
    K3_TRY(check_launch(#kernel)); } while (0)

// One token's attention for T queries at positions cached..cached+T-1, per (t, h) CTA.
// scores go to sc [T][H][last+1]; exactly the CPU's sequential double dot per score.
__global__ void k_mla_ref_attn(float *acc, float *sc, const float *q, const float *kvc,
                               const float *ropec, int H, int qn, int qr, int vh, int cached,
                               int nscore, float scale)
{
    __shared__ double red[32];
    __shared__ float redf[32];
    const int t = blockIdx.y, h = blockIdx.x;
    const int p = cached + t;
    const int qh = qn + qr, kvd = qn + vh;
    const float *qt = q + ((size_t)t * H + h) * qh;
    float *s = sc + ((size_t)t * H + h) * nscore;
    for (int j = threadIdx.x; j <= p; j += blockDim.x) {
        const float *ks = kvc + ((size_t)j * H + h) * kvd;
        const float *kr = ropec + (size_t)j * qr;
        double d = 0.0;
        for (int i = 0; i < qn; i++) d += (double)qt[i] * (double)ks[i];
        for (int i = 0; i < qr; i++) d += (double)qt[qn + i] * (double)kr[i];
        s[j] = __fmul_rn((float)d, scale);
    }
    __syncthreads();
    float m = -INFINITY;
    for (int j = threadIdx.x; j <= p; j += blockDim.x) m = fmaxf(m, s[j]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) redf[threadIdx.x >> 5] = m;
    __syncthreads();
    m = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, redf[i]);
    double z = 0.0;
    for (int j = threadIdx.x; j <= p; j += blockDim.x) {
        const float e = expf(__fsub_rn(s[j], m));
        s[j] = e;
        z += e;
    }
    z = warp_sum_d(z);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = z;
    __syncthreads();
    z = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) z += red[i];
    for (int jj = threadIdx.x; jj < vh; jj += blockDim.x) {
        float o = 0.0f;
        for (int j = 0; j <= p; j++) {
            const float pr = (float)((double)s[j] / z);
            o = __fadd_rn(o, __fmul_rn(pr, kvc[((size_t)j * H + h) * kvd + qn + jj]));
        }
        acc[((size_t)t * H + h) * vh + jj] = o;
    }
}

// rmsnorm of the first n of a row, leaving the rest
static int rms(float *y, const float *x, const float *w, int n, float eps)
{
    return rmsnorm(y, x, w, n, 1, eps, stream());
}

// ------------------------------------------------------------------ device bodies ----
static int mla_dev(float *out, const float *x, const K3MlaW *w, const K3Cfg *c, int T,
                   float *kvc, float *ropec, int cached)
{
    const int E = c->hidden, H = c->n_heads, qn = c->qk_nope, qr = c->qk_rope, vh = c->v_head;
    const int qh = qn + qr, kvw = c->kv_lora + qr, kvd = qn + vh;
    const float scale = 1.0f / sqrtf((float)qh);
    const int last = cached + T - 1;
    cudaStream_t st = stream();
    std::vector<size_t> sz = {(size_t)T * H * qh, (size_t)kvw, (size_t)c->q_lora, (size_t)T * H * vh,
                              (size_t)H * vh, (size_t)T * H * (last + 1),
                              kvc ? 0 : (size_t)T * H * kvd, ropec ? 0 : (size_t)T * qr};
    size_t tot = 0;
    for (size_t v : sz) tot += (v + 63) & ~(size_t)63;
    float *base = (float *)scratch(tot * sizeof(float), 2);
    if (!base) return k3d_status();
    float *ptrs[8];
    size_t off = 0;
    for (int i = 0; i < 8; i++) { ptrs[i] = base + off; off += (sz[i] + 63) & ~(size_t)63; }
    float *q = ptrs[0], *ct = ptrs[1], *ql = ptrs[2], *acc = ptrs[3], *gbuf = ptrs[4], *sc = ptrs[5];
    float *KV = kvc ? kvc : ptrs[6];
    float *RP = ropec ? ropec : ptrs[7];
    const int base_pos = kvc ? 0 : cached;       // self-contained buffers start at position cached
    for (int t = 0; t < T; t++) {
        const int p = cached + t;
        const float *xt = x + (size_t)t * E;
        K3_TRY(gemv_tagged(ql, xt, w->q_a, w->wdt, E, c->q_lora, st));
        K3_TRY(rms(ql, ql, w->q_a_norm, c->q_lora, c->rms_eps));
        K3_TRY(gemv_tagged(q + (size_t)t * H * qh, ql, w->q_b, w->wdt, c->q_lora, H * qh, st));
        K3_TRY(gemv_tagged(ct, xt, w->kv_a, w->wdt, E, kvw, st));
        K3_TRY(rms(ct, ct, w->kv_a_norm, c->kv_lora, c->rms_eps));
        if (cudaMemcpyAsync(RP + (size_t)(p - base_pos) * qr, ct + c->kv_lora, (size_t)qr * 4,
                            cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return fail(K3D_ECUDA, "mla rope slot copy");
        K3_TRY(gemv_tagged(KV + (size_t)(p - base_pos) * H * kvd, ct, w->kv_b, w->wdt, c->kv_lora,
                           H * kvd, st));
    }
    // without a cache the positions before `cached` do not exist: attend from base_pos
    k_mla_ref_attn<<<dim3(H, T), 256, 0, st>>>(acc, sc, q, KV, RP, H, qn, qr, vh, cached - base_pos,
                                               last + 1, scale);
    note_launch();
    K3_TRY(check_launch("mla ref attn"));
    for (int t = 0; t < T; t++) {
        float *at = acc + (size_t)t * H * vh;
        if (w->g) {
            K3_TRY(gemv_tagged(gbuf, x + (size_t)t * E, w->g, w->wdt, E, H * vh, st));
            EW(k_gate_mul, (size_t)H * vh, at, gbuf, (size_t)H * vh);
        }
        K3_TRY(gemv_tagged(out + (size_t)t * E, at, w->o, w->wdt, H * vh, E, st));
    }
    return K3D_OK;
}

static int kda_dev(float *out, const float *x, const K3KdaW *w, const K3Cfg *c, int T, float *state)
{
    const int E = c->hidden, H = c->kda_heads, D = c->kda_head_dim, P = H * D, K = c->conv_k;
    const int hist = K - 1;
    cudaStream_t st = stream();
    const size_t n_tp = (size_t)T * P;
    const size_t need = 6 * n_tp + (size_t)T * H + 2 * (size_t)P + D + (state ? 0 : (size_t)H * D * D) + 64;
    float *s = (float *)scratch(need * sizeof(float), 2);
    if (!s) return k3d_status();
    float *q = s, *k = q + n_tp, *v = k + n_tp, *z = v + n_tp, *al = z + n_tp, *o = al + n_tp;
    float *bt = o + n_tp, *gb = bt + (size_t)T * H, *fa = gb + P;
    float *S = state;
    if (!S) {
        S = fa + D + 16;
        if (cudaMemsetAsync(S, 0, (size_t)H * D * D * 4, st) != cudaSuccess)
            return fail(K3D_ECUDA, "kda zero state");
    }
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * E;
        K3_TRY(gemv_tagged(q + (size_t)t * P, xt, w->q, w->wdt, E, P, st));
        K3_TRY(gemv_tagged(k + (size_t)t * P, xt, w->k, w->wdt, E, P, st));
        K3_TRY(gemv_tagged(v + (size_t)t * P, xt, w->v, w->wdt, E, P, st));
        K3_TRY(gemv_tagged(bt + (size_t)t * H, xt, w->b, w->wdt, E, H, st));
        K3_TRY(gemv_tagged(fa, xt, w->f_a, w->wdt, E, D, st));
        K3_TRY(gemv_tagged(z + (size_t)t * P, fa, w->f_b, w->wdt, D, P, st));
    }
    float *cs = state ? state + (size_t)H * D * D : nullptr;
    K3_TRY(shortconv(q, q, w->q_conv, cs, P, K, T, st));
    K3_TRY(shortconv(k, k, w->k_conv, cs ? cs + (size_t)P * hist : nullptr, P, K, T, st));
    K3_TRY(shortconv(v, v, w->v_conv, cs ? cs + (size_t)2 * P * hist : nullptr, P, K, T, st));
    k_l2norm_rows<<<T * H, 128, 0, st>>>(q, D, 1e-6f);
    k_l2norm_rows<<<T * H, 128, 0, st>>>(k, D, 1e-6f);
    note_launch(2);
    K3_TRY(check_launch("kda l2norm"));
    EW(k_sigmoid, (size_t)T * H, bt, (size_t)T * H);
    for (int t = 0; t < T; t++)
        K3_TRY(kda_decay(z + (size_t)t * P, al + (size_t)t * P, z + (size_t)t * P, w->A_log,
                         w->dt_bias, H, D, c->gate_lb, st));
    EW(k_scale, n_tp, q, n_tp, 1.0f / sqrtf((float)D));
    K3_TRY(kda_seq(S, o, q, k, v, al, bt, T, H, D, D, st));
    K3_TRY(rmsnorm(o, o, w->o_norm, D, T * H, c->rms_eps, st));
    for (int t = 0; t < T; t++) {
        K3_TRY(gemv_tagged(gb, x + (size_t)t * E, w->g, w->wdt, E, P, st));
        EW(k_gate_mul, (size_t)P, o + (size_t)t * P, gb, (size_t)P);
        K3_TRY(gemv_tagged(out + (size_t)t * E, o + (size_t)t * P, w->o, w->wdt, P, E, st));
    }
    return K3D_OK;
}

// experts: per token, route (device), then the host walks the top-k like k3_moe.
static int moe_dev(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T,
                   int *idx_host, float *wt_host, const K3MoeW *w_host)
{
    const int E = c->hidden, L = c->latent, I = c->moe_inter, SI = I * c->n_shared, K = c->topk;
    cudaStream_t st = stream();
    const size_t need = (size_t)2 * L + 3 * (size_t)I + L + 3 * (size_t)SI + E + 2 * (size_t)K + 64;
    float *s = (float *)scratch(need * sizeof(float), 2);
    if (!s) return k3d_status();
    float *z = s, *accL = z + L, *gu = accL + L, *act = gu + 2 * I, *edn = act + I;
    float *sgu = edn + L, *sact = sgu + 2 * SI, *sdn = sact + SI;
    int *didx = (int *)(sdn + E);
    float *dwt = (float *)(didx + K);
    void *rws = scratch(router_ws_bytes(1, c->n_experts), 1);
    if (!rws) return k3d_status();
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * E;
        float *ot = out + (size_t)t * E;
        K3_TRY(router_f32(didx, dwt, xt, w->gate, w->bias, 1, E, c->n_experts, K, c->moe_renorm,
                          c->routed_scale, rws, st));
        if (cudaMemcpyAsync(idx_host, didx, K * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(wt_host, dwt, K * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            return fail(K3D_ECUDA, "router read-back");
        int nk = K;
        if (w_host->cache_only && w_host->src && w_host->src->resident) {
            int m = 0;
            float wsum = 0.0f;
            for (int j = 0; j < K; j++)
                if (w_host->src->resident(w_host->src, w_host->layer, idx_host[j], NULL)) {
                    idx_host[m] = idx_host[j]; wt_host[m] = wt_host[j]; wsum += wt_host[j]; m++;
                }
            nk = m;
            if (wsum > 0.0f) for (int j = 0; j < nk; j++) wt_host[j] /= wsum;
            if (cudaMemcpyAsync(dwt, wt_host, K * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
                return fail(K3D_ECUDA, "weights upload");
        }
        K3_TRY(gemv_tagged(z, xt, w->down, w->wdt, E, L, st));
        if (cudaMemsetAsync(accL, 0, (size_t)L * 4, st) != cudaSuccess) return fail(K3D_ECUDA, "memset");
        if (!w_host->cache_only && w_host->src && w_host->src->getmany)
            w_host->src->getmany(w_host->src, w_host->layer, idx_host, nk);
        for (int j = 0; j < nk; j++) {
            if (w_host->src) {
                K3ExpertQ q;
                const int miss = w_host->cache_only
                    ? !w_host->src->resident(w_host->src, w_host->layer, idx_host[j], &q)
                    : (w_host->src->get(w_host->src, w_host->layer, idx_host[j], &q) != 0);
                if (miss) {
                    if (w_host->cache_only) continue;
                    k3_expert_drops++;
                    fprintf(stderr, "EXPERT DROP: layer %d expert %d failed to load; this token is CORRUPT\n",
                            w_host->layer, idx_host[j]);
                    continue;
                }
                // per-call expert bytes: staged as inputs (a cache slot may be reused)
                Stage es;
                const size_t pb = (size_t)I * L / 2, sb = (size_t)I * L / 32;
                const unsigned char *p1 = (const unsigned char *)es.in(q.p1, pb);
                const unsigned char *s1 = (const unsigned char *)es.in(q.s1, sb);
                const unsigned char *p3 = (const unsigned char *)es.in(q.p3, pb);
                const unsigned char *s3 = (const unsigned char *)es.in(q.s3, sb);
                const unsigned char *p2 = (const unsigned char *)es.in(q.p2, pb);
                const unsigned char *s2 = (const unsigned char *)es.in(q.s2, sb);
                if (es.err) return es.err;
                K3_TRY(mxfp4_gemv(gu, z, p1, s1, L, I, K3_MXFP4_GROUP, st));
                K3_TRY(mxfp4_gemv(gu + I, z, p3, s3, L, I, K3_MXFP4_GROUP, st));
                K3_TRY(situ_glu(act, gu, I, 1, c->situ_b1, c->situ_b2, st));
                K3_TRY(mxfp4_gemv(edn, act, p2, s2, I, L, K3_MXFP4_GROUP, st));
                K3_TRY(es.finish());
            } else {
                const size_t e = (size_t)idx_host[j];
                K3_TRY(gemv_ref_f32(gu, z, w->w1 + e * I * L, L, I, 1, 0, st));
                K3_TRY(gemv_ref_f32(gu + I, z, w->w3 + e * I * L, L, I, 1, 0, st));
                K3_TRY(situ_glu(act, gu, I, 1, c->situ_b1, c->situ_b2, st));
                K3_TRY(gemv_ref_f32(edn, act, w->w2 + e * L * I, I, L, 1, 0, st));
            }
            EW(k_axpy_ordered, (size_t)L, accL, dwt, j, edn, (size_t)L);
        }
        if (c->latent_norm) K3_TRY(rmsnorm(accL, accL, w->latent_norm, L, 1, c->rms_eps, st));
        K3_TRY(gemv_tagged(ot, accL, w->up, w->wdt, L, E, st));
        K3_TRY(gemv_tagged(sgu, xt, w->sh1, w->wdt, E, SI, st));
        K3_TRY(gemv_tagged(sgu + SI, xt, w->sh3, w->wdt, E, SI, st));
        K3_TRY(situ_glu(sact, sgu, SI, 1, c->situ_b1, c->situ_b2, st));
        K3_TRY(gemv_tagged(sdn, sact, w->sh2, w->wdt, SI, E, st));
        EW(k_add, (size_t)E, ot, sdn, (size_t)E);
    }
    return K3D_OK;
}

// ---------------------------------------------------------------- staging of structs ----
static size_t wbytes(int wdt, size_t n) { return n * (wdt == K3_WBF16 ? 2 : 4); }

static bool stage_mla(Stage &st, const K3MlaW *w, const K3Cfg *c, K3MlaW *d)
{
    const size_t E = c->hidden, H = c->n_heads, qh = c->qk_nope + c->qk_rope;
    const size_t kvw = c->kv_lora + c->qk_rope, kvd = c->qk_nope + c->v_head, vh = c->v_head;
    *d = *w;
    d->q_a = st.weight(w->q_a, wbytes(w->wdt, c->q_lora * E));
    d->q_b = st.weight(w->q_b, wbytes(w->wdt, H * qh * c->q_lora));
    d->kv_a = st.weight(w->kv_a, wbytes(w->wdt, kvw * E));
    d->kv_b = st.weight(w->kv_b, wbytes(w->wdt, H * kvd * c->kv_lora));
    d->o = st.weight(w->o, wbytes(w->wdt, E * H * vh));
    d->g = w->g ? st.weight(w->g, wbytes(w->wdt, H * vh * E)) : nullptr;
    d->q_a_norm = (const float *)st.weight(w->q_a_norm, (size_t)c->q_lora * 4);
    d->kv_a_norm = (const float *)st.weight(w->kv_a_norm, (size_t)c->kv_lora * 4);
    return !st.err;
}

static bool stage_kda(Stage &st, const K3KdaW *w, const K3Cfg *c, K3KdaW *d)
{
    const size_t E = c->hidden, H = c->kda_heads, D = c->kda_head_dim, P = H * D, K = c->conv_k;
    *d = *w;
    d->q = st.weight(w->q, wbytes(w->wdt, P * E));
    d->k = st.weight(w->k, wbytes(w->wdt, P * E));
    d->v = st.weight(w->v, wbytes(w->wdt, P * E));
    d->q_conv = (const float *)st.weight(w->q_conv, P * K * 4);
    d->k_conv = (const float *)st.weight(w->k_conv, P * K * 4);
    d->v_conv = (const float *)st.weight(w->v_conv, P * K * 4);
    d->f_a = st.weight(w->f_a, wbytes(w->wdt, D * E));
    d->f_b = st.weight(w->f_b, wbytes(w->wdt, P * D));
    d->A_log = (const float *)st.weight(w->A_log, H * 4);
    d->dt_bias = (const float *)st.weight(w->dt_bias, P * 4);
    d->b = st.weight(w->b, wbytes(w->wdt, H * E));
    d->g = st.weight(w->g, wbytes(w->wdt, P * E));
    d->o_norm = (const float *)st.weight(w->o_norm, D * 4);
    d->o = st.weight(w->o, wbytes(w->wdt, E * P));
    return !st.err;
}

static bool stage_moe(Stage &st, const K3MoeW *w, const K3Cfg *c, K3MoeW *d)
{
    const size_t E = c->hidden, L = c->latent, I = c->moe_inter, SI = I * c->n_shared;
    const size_t NE = c->n_experts;
    *d = *w;
    d->gate = (const float *)st.weight(w->gate, NE * E * 4);
    d->bias = w->bias ? (const float *)st.weight(w->bias, NE * 4) : nullptr;
    if (!w->src) {
        d->w1 = (const float *)st.weight(w->w1, NE * I * L * 4);
        d->w3 = (const float *)st.weight(w->w3, NE * I * L * 4);
        d->w2 = (const float *)st.weight(w->w2, NE * L * I * 4);
    }
    d->latent_norm = c->latent_norm ? (const float *)st.weight(w->latent_norm, L * 4) : nullptr;
    d->down = st.weight(w->down, wbytes(w->wdt, L * E));
    d->up = st.weight(w->up, wbytes(w->wdt, E * L));
    d->sh1 = st.weight(w->sh1, wbytes(w->wdt, SI * E));
    d->sh3 = st.weight(w->sh3, wbytes(w->wdt, SI * E));
    d->sh2 = st.weight(w->sh2, wbytes(w->wdt, E * SI));
    return !st.err;
}

}  // namespace k3

using namespace k3;

extern "C" {

// ------------------------------------------------------------------- sizers ----
size_t k3_mla_scratch_cached(const K3Cfg *c, int T, int cap, int cached_mode)
{
    const int H = c->n_heads, qh = c->qk_nope + c->qk_rope, vh = c->v_head;
    const size_t kvd = (size_t)(c->qk_nope + vh);
    size_t n = (size_t)T * H * qh + (size_t)(c->kv_lora + c->qk_rope) + (size_t)c->q_lora +
               (size_t)2 * H * vh + (size_t)(cap > T ? cap : T);
    if (!cached_mode) n += (size_t)T * H * kvd + (size_t)T * c->qk_rope;
    return n;
}

size_t k3_mla_scratch(const K3Cfg *c, int T) { return k3_mla_scratch_cached(c, T, T, 0); }

size_t k3_moe_scratch(const K3Cfg *c)
{
    const int SI = c->moe_inter * c->n_shared;
    return (size_t)2 * c->latent + (size_t)3 * c->moe_inter + (size_t)c->latent +
           (size_t)3 * SI + (size_t)c->hidden;
}

size_t k3_kda_scratch(const K3Cfg *c, int T)
{
    const size_t P = (size_t)c->kda_heads * c->kda_head_dim;
    return 3 * (size_t)T * P + 2 * (size_t)T * P + (size_t)T * c->kda_heads + (size_t)T * P +
           2 * P + (size_t)c->kda_head_dim;
}

size_t k3_layer_scratch(const K3Cfg *c, int T)
{
    size_t a = k3_mla_scratch(c, T), b = k3_kda_scratch(c, T), m = k3_moe_scratch(c);
    size_t sub = a > b ? a : b;
    if (m > sub) sub = m;
    return (size_t)3 * T * c->hidden + (size_t)2 * c->hidden +
           (size_t)(c->n_layers / c->attn_res_block + 2) * c->hidden +
           (size_t)2 * c->dense_inter + sub;
}

// ---------------------------------------------------------------------- MLA ----
void k3_mla_cached(float *out, const float *x, const K3MlaW *w, const K3Cfg *c, int T,
                   float *scratch_unused, float *kvc, float *ropec, int cached, int cap)
{
    (void)scratch_unused;
    if (ensure_ctx() || !w || !c || T < 1) return;
    if (!kvc) { cached = 0; ropec = nullptr; }
    const int last = cached + T - 1;
    if (kvc && last >= cap) {
        fail(K3D_EBOUND, "MLA KV cache position %d exceeds capacity %d", last, cap - 1);
        return;
    }
    const int E = c->hidden, H = c->n_heads, kvd = c->qk_nope + c->v_head;
    Stage st;
    K3MlaW dw;
    if (!stage_mla(st, w, c, &dw)) return;
    const float *X = (const float *)st.in(x, (size_t)T * E * 4);
    float *KV = kvc ? (float *)st.inout(kvc, (size_t)cap * H * kvd * 4) : nullptr;
    float *RP = kvc ? (float *)st.inout(ropec, (size_t)cap * c->qk_rope * 4) : nullptr;
    float *O = (float *)st.out(out, (size_t)T * E * 4);
    if (st.err) return;
    if (mla_dev(O, X, &dw, c, T, KV, RP, cached)) return;
    st.finish();
}

void k3_mla(float *out, const float *x, const K3MlaW *w, const K3Cfg *c, int T, float *scratch)
{
    k3_mla_cached(out, x, w, c, T, scratch, NULL, NULL, 0, 0);
}

// ---------------------------------------------------------------------- MoE ----
void k3_moe(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T, int *idx,
            float *wt, float *scratch_unused)
{
    (void)scratch_unused;
    if (ensure_ctx() || !w || !c || T < 1) return;
    if (c->topk < 1 || c->topk > K3_MAX_TOPK) {
        fail(K3D_EBOUND, "k3_moe topk=%d", c->topk);
        return;
    }
    Stage st;
    K3MoeW dw;
    if (!stage_moe(st, w, c, &dw)) return;
    const float *X = (const float *)st.in(x, (size_t)T * c->hidden * 4);
    float *O = (float *)st.out(out, (size_t)T * c->hidden * 4);
    if (st.err) return;
    std::vector<int> ih(c->topk);
    std::vector<float> wh(c->topk);
    if (moe_dev(O, X, &dw, c, T, ih.data(), wh.data(), w)) return;
    if (st.finish()) return;
    if (idx) memcpy(idx, ih.data(), c->topk * sizeof(int));
    if (wt) memcpy(wt, wh.data(), c->topk * sizeof(float));
}

void k3_moe_prefill(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T, int *idx,
                    float *wt, float *scratch)
{
    // per-token results are identical to k3_moe (k3_ops.c:677-682); the order in which
    // experts are fetched is the only difference, and experts here are resident
    k3_moe(out, x, w, c, T, idx, wt, scratch);
}

// ---------------------------------------------------------------------- KDA ----
void k3_kda_layer(float *out, const float *x, const K3KdaW *w, const K3Cfg *c, int T,
                  float *state, float *scratch_unused)
{
    (void)scratch_unused;
    if (ensure_ctx() || !w || !c || T < 1) return;
    const int H = c->kda_heads, D = c->kda_head_dim, P = H * D;
    Stage st;
    K3KdaW dw;
    if (!stage_kda(st, w, c, &dw)) return;
    const float *X = (const float *)st.in(x, (size_t)T * c->hidden * 4);
    const size_t sfl = (size_t)H * D * D + 3 * (size_t)P * (c->conv_k - 1);
    float *S = state ? (float *)st.inout(state, sfl * 4) : nullptr;
    float *O = (float *)st.out(out, (size_t)T * c->hidden * 4);
    if (st.err) return;
    if (kda_dev(O, X, &dw, c, T, S)) return;
    st.finish();
}

// ------------------------------------------------------------- decoder layer ----
void k3_decoder_layer_inc(float *h, float *block_residual, int *n_blocks, const K3LayerW *w,
                          const K3Cfg *c, int layer_idx, int T, float *state, float *scratch_unused,
                          float *kvc, float *ropec, int cached, int cap)
{
    (void)scratch_unused;
    if (ensure_ctx() || !w || !c || !n_blocks || T < 1) return;
    const int E = c->hidden;
    const int maxb = c->n_layers / c->attn_res_block + 2;
    if (!w->attn_res_norm || !w->attn_res_proj || !w->mlp_res_norm || !w->mlp_res_proj) {
        fail(K3D_EINVAL, "k3_decoder_layer_inc: AttnRes weights are required (k3d_model_* runs "
                         "plain residual stacks)");
        return;
    }
    if (!kvc) { cached = 0; ropec = nullptr; }
    if (w->mla && kvc && cached + T - 1 >= cap) {
        fail(K3D_EBOUND, "MLA KV cache position %d exceeds capacity %d", cached + T - 1, cap - 1);
        return;
    }
    Stage st;
    float *H_ = (float *)st.inout(h, (size_t)T * E * 4);
    float *BR = (float *)st.inout(block_residual, (size_t)T * maxb * E * 4);
    const float *in_norm = (const float *)st.weight(w->in_norm, E * 4);
    const float *post_norm = (const float *)st.weight(w->post_norm, E * 4);
    const float *arn = (const float *)st.weight(w->attn_res_norm, E * 4);
    const float *arp = (const float *)st.weight(w->attn_res_proj, E * 4);
    const float *mrn = (const float *)st.weight(w->mlp_res_norm, E * 4);
    const float *mrp = (const float *)st.weight(w->mlp_res_proj, E * 4);
    K3KdaW kw;
    K3MlaW mw;
    K3MoeW ow;
    float *S = nullptr, *KV = nullptr, *RP = nullptr;
    if (w->kda) {
        if (!stage_kda(st, w->kda, c, &kw)) return;
        const size_t sfl = (size_t)c->kda_heads * c->kda_head_dim * c->kda_head_dim +
                           3 * (size_t)c->kda_heads * c->kda_head_dim * (c->conv_k - 1);
        S = state ? (float *)st.inout(state, sfl * 4) : nullptr;
    } else if (w->mla) {
        if (!stage_mla(st, w->mla, c, &mw)) return;
        const int kvd = c->qk_nope + c->v_head;
        if (kvc) {
            KV = (float *)st.inout(kvc, (size_t)cap * c->n_heads * kvd * 4);
            RP = (float *)st.inout(ropec, (size_t)cap * c->qk_rope * 4);
        }
    } else {
        fail(K3D_EINVAL, "k3_decoder_layer_inc: neither KDA nor MLA weights");
        return;
    }
    const void *dg = nullptr, *du = nullptr, *dd = nullptr;
    if (w->moe) {
        if (!stage_moe(st, w->moe, c, &ow)) return;
    } else {
        dg = st.weight(w->dense_gate, wbytes(w->wdt, (size_t)c->dense_inter * E));
        du = st.weight(w->dense_up, wbytes(w->wdt, (size_t)c->dense_inter * E));
        dd = st.weight(w->dense_down, wbytes(w->wdt, (size_t)E * c->dense_inter));
    }
    if (st.err) return;
    cudaStream_t s = stream();
    const size_t TE = (size_t)T * E;
    float *buf = (float *)scratch((4 * TE + 2 * (size_t)E + (size_t)(maxb + 1) * E +
                                   2 * (size_t)c->dense_inter + 64) * 4, 0);
    if (!buf) return;
    float *pref = buf, *tmp = pref + TE, *hin = tmp + TE, *foldA = hin + TE, *foldM = foldA + E;
    float *src = foldM + E, *dgu = src + (size_t)(maxb + 1) * E, *act = dgu + 2 * (size_t)c->dense_inter;
    // fold the AttnRes norm and projection vectors (k3_ops.c:983-986)
    k_mul2<<<nb(E), 256, 0, s>>>(foldA, arn, arp, (size_t)E);
    k_mul2<<<nb(E), 256, 0, s>>>(foldM, mrn, mrp, (size_t)E);
    note_launch(2);
    cudaMemcpyAsync(pref, H_, TE * 4, cudaMemcpyDeviceToDevice, s);
    int have_prefix = 1;
    const int nb0 = *n_blocks;
    if (nb0 > 0) {
        for (int t = 0; t < T; t++) {
            cudaMemcpyAsync(src, BR + (size_t)t * maxb * E, (size_t)nb0 * E * 4, cudaMemcpyDeviceToDevice, s);
            cudaMemcpyAsync(src + (size_t)nb0 * E, pref + (size_t)t * E, (size_t)E * 4, cudaMemcpyDeviceToDevice, s);
            if (attn_res(H_ + (size_t)t * E, src, foldA, nb0 + 1, E, c->rms_eps, s)) return;
        }
    }
    if (layer_idx % c->attn_res_block == 0) {
        for (int t = 0; t < T; t++)
            cudaMemcpyAsync(BR + ((size_t)t * maxb + nb0) * E, pref + (size_t)t * E, (size_t)E * 4,
                            cudaMemcpyDeviceToDevice, s);
        (*n_blocks)++;
        have_prefix = 0;
    }
    if (rmsnorm(hin, H_, in_norm, E, T, c->rms_eps, s)) return;
    if (w->kda) { if (kda_dev(tmp, hin, &kw, c, T, S)) return; }
    else if (mla_dev(tmp, hin, &mw, c, T, KV, RP, cached)) return;
    if (have_prefix) { k_add<<<nb(TE), 256, 0, s>>>(pref, tmp, TE); note_launch(); }
    else cudaMemcpyAsync(pref, tmp, TE * 4, cudaMemcpyDeviceToDevice, s);
    const int nb1 = *n_blocks;
    for (int t = 0; t < T; t++) {
        cudaMemcpyAsync(src, BR + (size_t)t * maxb * E, (size_t)nb1 * E * 4, cudaMemcpyDeviceToDevice, s);
        cudaMemcpyAsync(src + (size_t)nb1 * E, pref + (size_t)t * E, (size_t)E * 4, cudaMemcpyDeviceToDevice, s);
        if (attn_res(H_ + (size_t)t * E, src, foldM, nb1 + 1, E, c->rms_eps, s)) return;
    }
    if (rmsnorm(hin, H_, post_norm, E, T, c->rms_eps, s)) return;
    if (w->moe) {
        std::vector<int> ih(c->topk);
        std::vector<float> wh(c->topk);
        if (moe_dev(tmp, hin, &ow, c, T, ih.data(), wh.data(), w->moe)) return;
    } else {
        for (int t = 0; t < T; t++) {
            if (gemv_tagged(dgu, hin + (size_t)t * E, dg, w->wdt, E, c->dense_inter, s)) return;
            if (gemv_tagged(dgu + c->dense_inter, hin + (size_t)t * E, du, w->wdt, E, c->dense_inter, s))
                return;
            if (situ_glu(act, dgu, c->dense_inter, 1, c->situ_b1, c->situ_b2, s)) return;
            if (gemv_tagged(tmp + (size_t)t * E, act, dd, w->wdt, c->dense_inter, E, s)) return;
        }
    }
    k_add<<<nb(TE), 256, 0, s>>>(pref, tmp, TE);
    note_launch();
    cudaMemcpyAsync(H_, pref, TE * 4, cudaMemcpyDeviceToDevice, s);
    if (check_launch("decoder layer")) return;
    st.finish();
}

void k3_decoder_layer(float *h, float *block_residual, int *n_blocks, const K3LayerW *w,
                      const K3Cfg *c, int layer_idx, int T, float *state, float *scratch)
{
    k3_decoder_layer_inc(h, block_residual, n_blocks, w, c, layer_idx, T, state, scratch, NULL,
                         NULL, 0, 0);
}

}  // extern "C"
