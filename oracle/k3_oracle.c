/* k3_oracle.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * CPU restatement of the decode-path arithmetic of libxsmm/kimi-k3-in-c
 * (src/core/k3_ops.c), the checker for libk3cuda's parity tests. Build with
 * -ffp-contract=off (oracle/Makefile does) so that the order of every multiply and add
 * below is the order that executes, as in the reference build.
 */
#include "k3_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

float orc_bf16f(uint16_t h)
{
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)h << 16;
    return v.f;
}

uint16_t orc_f2bf(float f)
{
    union { uint32_t u; float f; } v;
    v.f = f;
    uint32_t u = v.u;
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static void *xmalloc(size_t n)
{
    void *p = malloc(n ? n : 1);
    if (!p) { fprintf(stderr, "oracle: out of memory (%zu bytes)\n", n); abort(); }
    return p;
}

static float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

/* k3_ops.c:84-89: full_attn is one-based */
int orc_is_mla(const K3Cfg *c, int layer)
{
    for (int i = 0; i < c->n_full_attn; i++)
        if (c->full_attn[i] == layer + 1) return 1;
    return 0;
}

/* k3_ops.c:94-102 */
void orc_rmsnorm(float *y, const float *x, const float *w, int n, float eps)
{
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    const float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
    for (int i = 0; i < n; i++) y[i] = w[i] * x[i] * inv;
}

/* k3_ops.c:110-123: the sigmoid takes the uncapped gate */
void orc_situ_glu(float *y, const float *x, int n, float b1, float b2)
{
    for (int i = 0; i < n; i++) {
        const float g = x[i], u = x[n + i];
        const float a = b1 * tanhf(g / b1) * sigm(g);
        const float c = b2 * tanhf(u / b2);
        y[i] = a * c;
    }
}

/* k3_ops.c:133-165: taps oldest..newest, w[k-1] multiplies the current input */
void orc_shortconv(float *y, const float *x, const float *w, float *state,
                   int channels, int k, int T)
{
    const int hist = k - 1;
    float buf[64];
    if (hist > 64) { fprintf(stderr, "oracle: shortconv k too large\n"); abort(); }
    for (int c = 0; c < channels; c++) {
        for (int j = 0; j < hist; j++) buf[j] = state ? state[(size_t)c * hist + j] : 0.0f;
        for (int t = 0; t < T; t++) {
            const float cur = x[(size_t)t * channels + c];
            float acc = w[(size_t)c * k + hist] * cur;
            for (int j = 0; j < hist; j++) acc += w[(size_t)c * k + j] * buf[j];
            for (int j = 0; j + 1 < hist; j++) buf[j] = buf[j + 1];
            if (hist > 0) buf[hist - 1] = cur;
            y[(size_t)t * channels + c] = acc * sigm(acc);
        }
        if (state)
            for (int j = 0; j < hist; j++) state[(size_t)c * hist + j] = buf[j];
    }
}

/* k3_ops.c:168-183: A_log indexed per head */
void orc_kda_decay(float *g, float *alpha, const float *z, const float *A_log,
                   const float *dt_bias, int H, int D, float lb)
{
    for (int h = 0; h < H; h++) {
        const float a = expf(A_log[h]);
        for (int d = 0; d < D; d++) {
            const int i = h * D + d;
            const float gi = lb * sigm(a * (z[i] + dt_bias[i]));
            g[i] = gi;
            alpha[i] = expf(gi);
        }
    }
}

/* k3_ops.c:186-243: decay rows, read u = S^T k, delta write, read o from updated S */
void orc_kda_step(float *S, float *o, const float *q, const float *k, const float *v,
                  const float *alpha, float beta, int dk, int dv)
{
    float *u = (float *)xmalloc((size_t)dv * sizeof(float));
    for (int i = 0; i < dk; i++)
        for (int j = 0; j < dv; j++) S[(size_t)i * dv + j] *= alpha[i];
    for (int j = 0; j < dv; j++) u[j] = 0.0f;
    for (int i = 0; i < dk; i++) {
        if (k[i] == 0.0f) continue;
        for (int j = 0; j < dv; j++) u[j] += k[i] * S[(size_t)i * dv + j];
    }
    for (int i = 0; i < dk; i++) {
        if (k[i] == 0.0f) continue;
        for (int j = 0; j < dv; j++) S[(size_t)i * dv + j] += k[i] * beta * (v[j] - u[j]);
    }
    for (int j = 0; j < dv; j++) o[j] = 0.0f;
    for (int i = 0; i < dk; i++) {
        if (q[i] == 0.0f) continue;
        for (int j = 0; j < dv; j++) o[j] += q[i] * S[(size_t)i * dv + j];
    }
    free(u);
}

/* k3_ops.c:265-291: sixteen double accumulators, fixed reduction tree */
static double dot16(const float *row, const float *x, int in, const uint16_t *brow)
{
    double a[16] = {0};
    int i = 0;
    for (; i + 15 < in; i += 16)
        for (int l = 0; l < 16; l++) {
            const double w = brow ? (double)orc_bf16f(brow[i + l]) : (double)row[i + l];
            a[l] = fma(w, (double)x[i + l], a[l]);
        }
    const double b0 = (a[0] + a[4]) + (a[8] + a[12]);
    const double b1 = (a[1] + a[5]) + (a[9] + a[13]);
    const double b2 = (a[2] + a[6]) + (a[10] + a[14]);
    const double b3 = (a[3] + a[7]) + (a[11] + a[15]);
    double acc = (b0 + b1) + (b2 + b3);
    for (; i < in; i++) {
        const double w = brow ? (double)orc_bf16f(brow[i]) : (double)row[i];
        acc = fma(w, (double)x[i], acc);
    }
    return acc;
}

void orc_matmul(float *y, const float *x, const float *W, int in, int out)
{
    #pragma omp parallel for schedule(static) if ((long)in * out > 262144)
    for (int o = 0; o < out; o++) y[o] = (float)dot16(W + (size_t)o * in, x, in, NULL);
}

/* k3_ops.c:1108-1213 (scalar path): bit-identical to orc_matmul on widened weights */
void orc_matmul_bf16(float *y, const float *x, const uint16_t *W, int in, int out)
{
    #pragma omp parallel for schedule(static) if ((long)in * out > 262144)
    for (int o = 0; o < out; o++) y[o] = (float)dot16(NULL, x, in, W + (size_t)o * in);
}

/* k3.h:289-295 */
void orc_mmw(float *y, const float *x, const void *W, int wdt, int in, int out)
{
    if (wdt == K3_WBF16) orc_matmul_bf16(y, x, (const uint16_t *)W, in, out);
    else orc_matmul(y, x, (const float *)W, in, out);
}

/* k3_ops.c:419-478. wb selects a bf16 gate matrix (widened exactly) */
static void router_any(int *idx, float *w, const float *x, const float *W, const uint16_t *Wb,
                       const float *bias, int hidden, int n_experts, int topk, int renorm,
                       float routed_scale)
{
    float *score = (float *)xmalloc((size_t)n_experts * sizeof(float));
    float *choice = (float *)xmalloc((size_t)n_experts * sizeof(float));
    for (int e = 0; e < n_experts; e++) {
        double acc = 0.0;
        for (int i = 0; i < hidden; i++) {
            const double wv = Wb ? (double)orc_bf16f(Wb[(size_t)e * hidden + i])
                                 : (double)W[(size_t)e * hidden + i];
            acc += wv * (double)x[i];
        }
        score[e] = 1.0f / (1.0f + expf(-(float)acc));
        choice[e] = score[e] + (bias ? bias[e] : 0.0f);
    }
    for (int j = 0; j < topk; j++) {
        int best = -1;
        float bv = -INFINITY;
        for (int e = 0; e < n_experts; e++)
            if (choice[e] > bv) { bv = choice[e]; best = e; }
        if (best < 0) { idx[j] = 0; w[j] = 0.0f; continue; }
        idx[j] = best;
        w[j] = score[best];
        choice[best] = -INFINITY;
    }
    if (renorm && topk > 1) {
        double s = 0.0;
        for (int j = 0; j < topk; j++) s += (double)w[j];
        const float inv = (float)(1.0 / (s + 1e-20));
        for (int j = 0; j < topk; j++) w[j] *= inv;
    }
    for (int j = 0; j < topk; j++) w[j] *= routed_scale;
    free(score);
    free(choice);
}

void orc_router(int *idx, float *w, const float *x, const float *W, const float *bias,
                int hidden, int n_experts, int topk, int renorm, float routed_scale)
{
    router_any(idx, w, x, W, NULL, bias, hidden, n_experts, topk, renorm, routed_scale);
}

void orc_router_bf16(int *idx, float *w, const float *x, const uint16_t *W, const float *bias,
                     int hidden, int n_experts, int topk, int renorm, float routed_scale)
{
    router_any(idx, w, x, NULL, W, bias, hidden, n_experts, topk, renorm, routed_scale);
}

/* k3_ops.c:481-512: keys normalised, values raw */
void orc_attn_res(float *out, const float *src, const float *fold, int nsrc, int n, float eps)
{
    float *score = (float *)xmalloc((size_t)nsrc * sizeof(float));
    for (int s = 0; s < nsrc; s++) {
        const float *v = src + (size_t)s * n;
        double ss = 0.0;
        for (int i = 0; i < n; i++) ss += (double)v[i] * (double)v[i];
        const float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
        double acc = 0.0;
        for (int i = 0; i < n; i++) acc += (double)(v[i] * inv) * (double)fold[i];
        score[s] = (float)acc;
    }
    float m = score[0];
    for (int s = 1; s < nsrc; s++) if (score[s] > m) m = score[s];
    double z = 0.0;
    for (int s = 0; s < nsrc; s++) { score[s] = expf(score[s] - m); z += score[s]; }
    for (int i = 0; i < n; i++) out[i] = 0.0f;
    for (int s = 0; s < nsrc; s++) {
        const float p = (float)(score[s] / z);
        for (int i = 0; i < n; i++) out[i] += p * src[(size_t)s * n + i];
    }
    free(score);
}

/* k3_ops.c:519-530 */
size_t orc_mla_scratch_cached(const K3Cfg *c, int T, int cap, int cached_mode)
{
    const int H = c->n_heads, qh = c->qk_nope + c->qk_rope, vh = c->v_head;
    const size_t kvd = (size_t)(c->qk_nope + vh);
    size_t n = (size_t)T * H * qh + (size_t)(c->kv_lora + c->qk_rope) + (size_t)c->q_lora +
               (size_t)2 * H * vh + (size_t)(cap > T ? cap : T);
    if (!cached_mode) n += (size_t)T * H * kvd + (size_t)T * c->qk_rope;
    return n;
}

/* k3_ops.c:321-410: NoPE, expanded per-head cache, shared rope slot, scale over the full
 * head width, causal, gate before o_proj */
void orc_mla_cached(float *out, const float *x, const K3MlaW *w, const K3Cfg *c, int T,
                    float *scratch, float *kvc, float *ropec, int cached, int cap)
{
    const int E = c->hidden, H = c->n_heads;
    const int qn = c->qk_nope, qr = c->qk_rope, vh = c->v_head;
    const int qh = qn + qr, kvw = c->kv_lora + qr, kvd = qn + vh;
    const float scale = 1.0f / sqrtf((float)qh);
    if (!kvc) cached = 0;
    const int last = cached + T - 1;
    if (kvc && last >= cap) { fprintf(stderr, "oracle: MLA cache overflow\n"); abort(); }
    float *q = scratch;
    float *ct = q + (size_t)T * H * qh;
    float *ql = ct + kvw;
    float *acc = ql + c->q_lora;
    float *gbuf = acc + (size_t)H * vh;
    float *sc = gbuf + (size_t)H * vh;
    float *kvs = sc + (last + 1);
    float *rps = kvs + (kvc ? 0 : (size_t)T * H * kvd);
#define KV_AT(p) (kvc ? kvc + (size_t)(p) * H * kvd : kvs + (size_t)(p) * H * kvd)
#define RP_AT(p) (ropec ? ropec + (size_t)(p) * qr : rps + (size_t)(p) * qr)
    for (int t = 0; t < T; t++) {
        const int p = cached + t;
        const float *xt = x + (size_t)t * E;
        orc_mmw(ql, xt, w->q_a, w->wdt, E, c->q_lora);
        orc_rmsnorm(ql, ql, w->q_a_norm, c->q_lora, c->rms_eps);
        orc_mmw(q + (size_t)t * H * qh, ql, w->q_b, w->wdt, c->q_lora, H * qh);
        orc_mmw(ct, xt, w->kv_a, w->wdt, E, kvw);
        orc_rmsnorm(ct, ct, w->kv_a_norm, c->kv_lora, c->rms_eps);
        memcpy(RP_AT(p), ct + c->kv_lora, (size_t)qr * sizeof(float));
        orc_mmw(KV_AT(p), ct, w->kv_b, w->wdt, c->kv_lora, H * kvd);
    }
    for (int t = 0; t < T; t++) {
        const int p = cached + t;
        for (int h = 0; h < H; h++) {
            const float *qt = q + ((size_t)t * H + h) * qh;
            float m = -INFINITY;
            for (int s = 0; s <= p; s++) {
                const float *ks = KV_AT(s) + (size_t)h * kvd;
                const float *kr = RP_AT(s);
                double d = 0.0;
                for (int i = 0; i < qn; i++) d += (double)qt[i] * (double)ks[i];
                for (int i = 0; i < qr; i++) d += (double)qt[qn + i] * (double)kr[i];
                sc[s] = (float)d * scale;
                if (sc[s] > m) m = sc[s];
            }
            double z = 0.0;
            for (int s = 0; s <= p; s++) { sc[s] = expf(sc[s] - m); z += sc[s]; }
            float *o = acc + (size_t)h * vh;
            for (int j = 0; j < vh; j++) o[j] = 0.0f;
            for (int s = 0; s <= p; s++) {
                const float pr = (float)(sc[s] / z);
                const float *vs = KV_AT(s) + (size_t)h * kvd + qn;
                for (int j = 0; j < vh; j++) o[j] += pr * vs[j];
            }
        }
        if (w->g) {
            orc_mmw(gbuf, x + (size_t)t * E, w->g, w->wdt, E, H * vh);
            for (int i = 0; i < H * vh; i++) acc[i] *= 1.0f / (1.0f + expf(-gbuf[i]));
        }
        orc_mmw(out + (size_t)t * E, acc, w->o, w->wdt, H * vh, E);
    }
#undef KV_AT
#undef RP_AT
}

/* k3_ops.c:658-666 */
size_t orc_moe_scratch(const K3Cfg *c)
{
    const int SI = c->moe_inter * c->n_shared;
    return (size_t)2 * c->latent + (size_t)3 * c->moe_inter + (size_t)c->latent +
           (size_t)3 * SI + (size_t)c->hidden;
}

/* k3_ops.c:1787-1817 */
static const float E2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                               -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

void orc_mxfp4_dequant(float *out, const unsigned char *packed, const unsigned char *scales,
                       int rows, int pcols, int group)
{
    const int width = pcols * 2;
    const int ngrp = (width + group - 1) / group;
    for (int r = 0; r < rows; r++) {
        for (int g = 0; g < ngrp; g++) {
            const unsigned char sb = scales[(size_t)r * ngrp + g];
            const float mult = (sb == 255) ? 0.0f : ldexpf(1.0f, (int)sb - 127);
            const int lo = g * group;
            int hi = lo + group;
            if (hi > width) hi = width;
            for (int i = lo; i < hi; i++) {
                const unsigned char byte = packed[(size_t)r * pcols + (i >> 1)];
                const unsigned char nib = (i & 1) ? (byte >> 4) : (byte & 0x0F);
                out[(size_t)r * width + i] = E2M1[nib] * mult;
            }
        }
    }
}

/* k3_ops.c:1380-1785, portable grouped path (1534-1780 without AVX2/NEON): per group,
 * expand to floats, eight double lanes reduced as ((s0+s4)+(s1+s5))+((s2+s6)+(s3+s7)),
 * then acc += sub * 2^(scale-127); a scale byte of 255 skips the group. */
void orc_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                      const unsigned char *scales, int in, int rows, int group)
{
    if ((in & 1) || group > 64 || group < 1) {
        fprintf(stderr, "oracle: matmul_mxfp4 in=%d group=%d\n", in, group);
        abort();
    }
    const int pcols = in / 2, ngrp = (in + group - 1) / group;
    #pragma omp parallel for schedule(static) if ((long)in * rows > 262144)
    for (int r = 0; r < rows; r++) {
        const unsigned char *pr = packed + (size_t)r * pcols;
        const unsigned char *sr = scales + (size_t)r * ngrp;
        double acc = 0.0;
        for (int g = 0; g < ngrp; g++) {
            const unsigned char sb = sr[g];
            if (sb == 255) continue;
            int n = in - g * group;
            if (n > group) n = group;
            float wf[64];
            for (int i = 0; i < n; i++) {
                const int ii = g * group + i;
                const unsigned char by = pr[ii >> 1];
                wf[i] = E2M1[(ii & 1) ? (by >> 4) : (by & 0x0F)];
            }
            const float *xg = x + (size_t)g * group;
            double s[8] = {0};
            int i = 0;
            for (; i + 7 < n; i += 8)
                for (int l = 0; l < 8; l++) s[l] = fma((double)wf[i + l], (double)xg[i + l], s[l]);
            double sub = ((s[0] + s[4]) + (s[1] + s[5])) + ((s[2] + s[6]) + (s[3] + s[7]));
            for (; i < n; i++) sub = fma((double)wf[i], (double)xg[i], sub);
            acc += sub * (double)ldexpf(1.0f, (int)sb - 127);
        }
        y[r] = (float)acc;
    }
}

/* k3_ops.c:556-656: route on the full width, down-project, experts in latent space
 * summed in top-k order, RMSNorm of the aggregate, up-project, + unweighted shared */
void orc_moe(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T, int *idx,
             float *wt, float *scratch, const K3ExpertQ *experts)
{
    const int E = c->hidden, L = c->latent, I = c->moe_inter, SI = I * c->n_shared;
    float *z = scratch, *accL = z + L, *gu = accL + L, *act = gu + 2 * I, *edn = act + I;
    float *sgu = edn + L, *sact = sgu + 2 * SI, *sdn = sact + SI;
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * E;
        float *ot = out + (size_t)t * E;
        orc_router(idx, wt, xt, w->gate, w->bias, E, c->n_experts, c->topk, c->moe_renorm,
                   c->routed_scale);
        orc_mmw(z, xt, w->down, w->wdt, E, L);
        for (int i = 0; i < L; i++) accL[i] = 0.0f;
        for (int j = 0; j < c->topk; j++) {
            if (experts) {
                const K3ExpertQ *q = &experts[idx[j]];
                orc_matmul_mxfp4(gu, z, q->p1, q->s1, L, I, K3_MXFP4_GROUP);
                orc_matmul_mxfp4(gu + I, z, q->p3, q->s3, L, I, K3_MXFP4_GROUP);
                orc_situ_glu(act, gu, I, c->situ_b1, c->situ_b2);
                orc_matmul_mxfp4(edn, act, q->p2, q->s2, I, L, K3_MXFP4_GROUP);
            } else {
                orc_matmul(gu, z, w->w1 + (size_t)idx[j] * I * L, L, I);
                orc_matmul(gu + I, z, w->w3 + (size_t)idx[j] * I * L, L, I);
                orc_situ_glu(act, gu, I, c->situ_b1, c->situ_b2);
                orc_matmul(edn, act, w->w2 + (size_t)idx[j] * L * I, I, L);
            }
            for (int i = 0; i < L; i++) accL[i] += wt[j] * edn[i];
        }
        if (c->latent_norm) orc_rmsnorm(accL, accL, w->latent_norm, L, c->rms_eps);
        orc_mmw(ot, accL, w->up, w->wdt, L, E);
        orc_mmw(sgu, xt, w->sh1, w->wdt, E, SI);
        orc_mmw(sgu + SI, xt, w->sh3, w->wdt, E, SI);
        orc_situ_glu(sact, sgu, SI, c->situ_b1, c->situ_b2);
        orc_mmw(sdn, sact, w->sh2, w->wdt, SI, E);
        for (int i = 0; i < E; i++) ot[i] += sdn[i];
    }
}

/* k3_ops.c:839-848 */
size_t orc_kda_scratch(const K3Cfg *c, int T)
{
    const size_t P = (size_t)c->kda_heads * c->kda_head_dim;
    return 3 * (size_t)T * P + 2 * (size_t)T * P + (size_t)T * c->kda_heads + (size_t)T * P +
           2 * P + (size_t)c->kda_head_dim;
}

/* k3_ops.c:831-837: sum of squares (not the mean), eps inside */
static void l2norm(float *v, int n, float eps)
{
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)v[i] * (double)v[i];
    const float inv = (float)(1.0 / sqrt(ss + (double)eps));
    for (int i = 0; i < n; i++) v[i] *= inv;
}

/* k3_ops.c:850-937 */
void orc_kda_layer(float *out, const float *x, const K3KdaW *w, const K3Cfg *c, int T,
                   float *state, float *scratch)
{
    const int E = c->hidden, H = c->kda_heads, D = c->kda_head_dim, P = H * D;
    const int K = c->conv_k, hist = K - 1;
    float *q = scratch, *k = q + (size_t)T * P, *v = k + (size_t)T * P, *z = v + (size_t)T * P;
    float *al = z + (size_t)T * P, *bt = al + (size_t)T * P, *o = bt + (size_t)T * H;
    float *gb = o + (size_t)T * P, *wr = gb + P, *fa = wr + P;
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * E;
        orc_mmw(q + (size_t)t * P, xt, w->q, w->wdt, E, P);
        orc_mmw(k + (size_t)t * P, xt, w->k, w->wdt, E, P);
        orc_mmw(v + (size_t)t * P, xt, w->v, w->wdt, E, P);
        orc_mmw(bt + (size_t)t * H, xt, w->b, w->wdt, E, H);
        orc_mmw(fa, xt, w->f_a, w->wdt, E, D);
        orc_mmw(z + (size_t)t * P, fa, w->f_b, w->wdt, D, P);
    }
    float *cs = state ? state + (size_t)H * D * D : NULL;
    orc_shortconv(q, q, w->q_conv, cs, P, K, T);
    orc_shortconv(k, k, w->k_conv, cs ? cs + (size_t)P * hist : NULL, P, K, T);
    orc_shortconv(v, v, w->v_conv, cs ? cs + (size_t)2 * P * hist : NULL, P, K, T);
    for (int t = 0; t < T; t++)
        for (int h = 0; h < H; h++) {
            l2norm(q + (size_t)t * P + (size_t)h * D, D, 1e-6f);
            l2norm(k + (size_t)t * P + (size_t)h * D, D, 1e-6f);
        }
    for (int t = 0; t < T; t++) {
        for (int h = 0; h < H; h++) bt[(size_t)t * H + h] = sigm(bt[(size_t)t * H + h]);
        orc_kda_decay(z + (size_t)t * P, al + (size_t)t * P, z + (size_t)t * P, w->A_log,
                      w->dt_bias, H, D, c->gate_lb);
    }
    float *S = state, *Sown = NULL;
    if (!S) { Sown = (float *)calloc((size_t)H * D * D, sizeof(float)); S = Sown; }
    const float qscale = 1.0f / sqrtf((float)D);
    for (int h = 0; h < H; h++) {
        float *wh = wr + (size_t)h * D;
        for (int t = 0; t < T; t++) {
            const size_t off = (size_t)t * P + (size_t)h * D;
            for (int i = 0; i < D; i++) wh[i] = q[off + i] * qscale;
            orc_kda_step(S + (size_t)h * D * D, o + off, wh, k + off, v + off, al + off,
                         bt[(size_t)t * H + h], D, D);
        }
    }
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * E;
        float *ot = o + (size_t)t * P;
        for (int h = 0; h < H; h++)
            orc_rmsnorm(ot + (size_t)h * D, ot + (size_t)h * D, w->o_norm, D, c->rms_eps);
        orc_mmw(gb, xt, w->g, w->wdt, E, P);
        for (int i = 0; i < P; i++) ot[i] *= sigm(gb[i]);
        orc_mmw(out + (size_t)t * E, ot, w->o, w->wdt, P, E);
    }
    free(Sown);
}

/* k3_ops.c:940-953 */
size_t orc_layer_scratch(const K3Cfg *c, int T)
{
    size_t a = orc_mla_scratch_cached(c, T, T, 0), b = orc_kda_scratch(c, T), m = orc_moe_scratch(c);
    size_t sub = a > b ? a : b;
    if (m > sub) sub = m;
    return (size_t)3 * T * c->hidden + (size_t)2 * c->hidden +
           (size_t)(c->n_layers / c->attn_res_block + 2) * c->hidden +
           (size_t)2 * c->dense_inter + sub;
}

/* k3_ops.c:964-1054: AttnRes wiring, boundary push-and-clear, unconditional second
 * aggregation */
void orc_decoder_layer_inc(float *h, float *block_residual, int *n_blocks, const K3LayerW *w,
                           const K3Cfg *c, int layer_idx, int T, float *state, float *scratch,
                           float *kvc, float *ropec, int cached, int cap,
                           const K3ExpertQ *experts)
{
    const int E = c->hidden, maxb = c->n_layers / c->attn_res_block + 2;
    float *pref = scratch, *tmp = pref + (size_t)T * E, *hin = tmp + (size_t)T * E;
    float *foldA = hin + (size_t)T * E, *foldM = foldA + E, *src = foldM + E;
    float *dgu = src + (size_t)maxb * E, *sub = dgu + (size_t)2 * c->dense_inter;
    for (int i = 0; i < E; i++) {
        foldA[i] = w->attn_res_norm[i] * w->attn_res_proj[i];
        foldM[i] = w->mlp_res_norm[i] * w->mlp_res_proj[i];
    }
    memcpy(pref, h, (size_t)T * E * sizeof(float));
    int have_prefix = 1;
    if (*n_blocks > 0) {
        for (int t = 0; t < T; t++) {
            for (int b = 0; b < *n_blocks; b++)
                memcpy(src + (size_t)b * E, block_residual + ((size_t)t * maxb + b) * E,
                       (size_t)E * sizeof(float));
            memcpy(src + (size_t)(*n_blocks) * E, pref + (size_t)t * E, (size_t)E * sizeof(float));
            orc_attn_res(h + (size_t)t * E, src, foldA, *n_blocks + 1, E, c->rms_eps);
        }
    }
    if (layer_idx % c->attn_res_block == 0) {
        for (int t = 0; t < T; t++)
            memcpy(block_residual + ((size_t)t * maxb + *n_blocks) * E, pref + (size_t)t * E,
                   (size_t)E * sizeof(float));
        (*n_blocks)++;
        have_prefix = 0;
    }
    for (int t = 0; t < T; t++)
        orc_rmsnorm(hin + (size_t)t * E, h + (size_t)t * E, w->in_norm, E, c->rms_eps);
    if (w->kda) orc_kda_layer(tmp, hin, w->kda, c, T, state, sub);
    else orc_mla_cached(tmp, hin, w->mla, c, T, sub, kvc, ropec, cached, cap);
    if (have_prefix) for (size_t i = 0; i < (size_t)T * E; i++) pref[i] += tmp[i];
    else memcpy(pref, tmp, (size_t)T * E * sizeof(float));
    for (int t = 0; t < T; t++) {
        for (int b = 0; b < *n_blocks; b++)
            memcpy(src + (size_t)b * E, block_residual + ((size_t)t * maxb + b) * E,
                   (size_t)E * sizeof(float));
        memcpy(src + (size_t)(*n_blocks) * E, pref + (size_t)t * E, (size_t)E * sizeof(float));
        orc_attn_res(h + (size_t)t * E, src, foldM, *n_blocks + 1, E, c->rms_eps);
    }
    for (int t = 0; t < T; t++)
        orc_rmsnorm(hin + (size_t)t * E, h + (size_t)t * E, w->post_norm, E, c->rms_eps);
    if (w->moe) {
        int idx[K3_MAX_TOPK];
        float wt[K3_MAX_TOPK];
        orc_moe(tmp, hin, w->moe, c, T, idx, wt, sub, experts);
    } else {
        for (int t = 0; t < T; t++) {
            orc_mmw(dgu, hin + (size_t)t * E, w->dense_gate, w->wdt, E, c->dense_inter);
            orc_mmw(dgu + c->dense_inter, hin + (size_t)t * E, w->dense_up, w->wdt, E,
                    c->dense_inter);
            orc_situ_glu(sub, dgu, c->dense_inter, c->situ_b1, c->situ_b2);
            orc_mmw(tmp + (size_t)t * E, sub, w->dense_down, w->wdt, c->dense_inter, E);
        }
    }
    for (size_t i = 0; i < (size_t)T * E; i++) pref[i] += tmp[i];
    memcpy(h, pref, (size_t)T * E * sizeof(float));
}

/* ------------------------------------------------ benchmark-shape compositions ---- */

float orc_silu(float g) { return g / (1.0f + expf(-g)); }

/* config 0: the per-expert body of k3_moe (k3_ops.c:628-631) with SiLU(g) * u */
void orc_expert_swiglu(float *y, const float *x, const K3ExpertQ *e, int hidden, int inter)
{
    float *g = (float *)xmalloc((size_t)inter * sizeof(float));
    float *u = (float *)xmalloc((size_t)inter * sizeof(float));
    orc_matmul_mxfp4(g, x, e->p1, e->s1, hidden, inter, K3_MXFP4_GROUP);
    orc_matmul_mxfp4(u, x, e->p3, e->s3, hidden, inter, K3_MXFP4_GROUP);
    for (int i = 0; i < inter; i++) g[i] = orc_silu(g[i]) * u[i];
    orc_matmul_mxfp4(y, g, e->p2, e->s2, inter, hidden, K3_MXFP4_GROUP);
    free(g);
    free(u);
}

/* config 1: k3_moe's order (k3_ops.c:571-655) without the latent step: route, experts in
 * top-k order with acc += w_j * edn_j, then the unweighted shared expert. Experts outside
 * [expert_lo, expert_hi) contribute nothing (one expert-parallel rank's partial). */
void orc_moe_swiglu(float *out, const float *x, int T, int hidden, int inter, int n_experts,
                    int topk, int renorm, float routed_scale, const uint16_t *router_w,
                    const float *router_bias, const K3ExpertQ *experts, int shared_inter,
                    const uint16_t *sh_gate, const uint16_t *sh_up, const uint16_t *sh_down,
                    int expert_lo, int expert_hi, int add_shared, int *idx_out, float *w_out)
{
    int idx[K3_MAX_TOPK];
    float wt[K3_MAX_TOPK];
    float *edn = (float *)xmalloc((size_t)hidden * sizeof(float));
    const int SI = shared_inter > 0 ? shared_inter : 1;
    float *sg = (float *)xmalloc((size_t)SI * sizeof(float));
    float *su = (float *)xmalloc((size_t)SI * sizeof(float));
    float *sd = (float *)xmalloc((size_t)hidden * sizeof(float));
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * hidden;
        float *ot = out + (size_t)t * hidden;
        orc_router_bf16(idx, wt, xt, router_w, router_bias, hidden, n_experts, topk, renorm,
                        routed_scale);
        if (idx_out) memcpy(idx_out + (size_t)t * topk, idx, (size_t)topk * sizeof(int));
        if (w_out) memcpy(w_out + (size_t)t * topk, wt, (size_t)topk * sizeof(float));
        for (int i = 0; i < hidden; i++) ot[i] = 0.0f;
        for (int j = 0; j < topk; j++) {
            if (idx[j] < expert_lo || idx[j] >= expert_hi) continue;
            orc_expert_swiglu(edn, xt, &experts[idx[j]], hidden, inter);
            for (int i = 0; i < hidden; i++) ot[i] += wt[j] * edn[i];
        }
        if (shared_inter > 0 && add_shared) {
            orc_matmul_bf16(sg, xt, sh_gate, hidden, shared_inter);
            orc_matmul_bf16(su, xt, sh_up, hidden, shared_inter);
            for (int i = 0; i < shared_inter; i++) sg[i] = orc_silu(sg[i]) * su[i];
            orc_matmul_bf16(sd, sg, sh_down, shared_inter, hidden);
            for (int i = 0; i < hidden; i++) ot[i] += sd[i];
        }
    }
    free(edn);
    free(sg);
    free(su);
    free(sd);
}

/* config 3 decode: k3_kda_step (k3_ops.c:186-243) per (sequence, head) */
void orc_kda_decode(float *S, float *o, const float *q, const float *k, const float *v,
                    const float *alpha, const float *beta, int B, int H, int dk, int dv)
{
    for (int b = 0; b < B; b++)
        for (int h = 0; h < H; h++) {
            const size_t bh = (size_t)b * H + h;
            orc_kda_step(S + bh * dk * dv, o + bh * dv, q + bh * dk, k + bh * dk, v + bh * dv,
                         alpha + bh * dk, beta[bh], dk, dv);
        }
}

/* RoPE on interleaved pairs (x[2i], x[2i+1]) with frequency theta^(-2i/d): the convention
 * chosen for the benchmark (the reference is NoPE, k3.h:43-48). Angle in double. */
void orc_rope(float *x, int d, int pos, float theta)
{
    if (!(theta > 0.0f)) return;   /* theta 0: NoPE, the reference's behaviour */
    for (int i = 0; i < d / 2; i++) {
        const double f = pow((double)theta, -2.0 * (double)i / (double)d);
        const double a = (double)pos * f;
        const float c = (float)cos(a), s = (float)sin(a);
        const float x0 = x[2 * i], x1 = x[2 * i + 1];
        x[2 * i] = x0 * c - x1 * s;
        x[2 * i + 1] = x0 * s + x1 * c;
    }
}

/* config 2: one decode token per sequence over a bf16 latent cache, k3_mla_cached's
 * arithmetic (k3_ops.c:321-410) in the EXPANDED form: every cached latent is widened and
 * re-projected through kv_b to per-head keys and values, then scored exactly as the
 * reference scores its fp32 expanded cache. Differences from the reference: the rope slot
 * is rotated (q per head, k at write time) and the cache holds bf16 latents. The new
 * token's latent and rotated rope key are rounded to bf16 when written, and attention
 * reads them back from the cache. cache [B][cap][kv_lora + rope]; positions [0, pos) are
 * filled and the new token is written at pos. */
/* When set, the attention of orc_mla_decode reads the new token's latent and rope key in
 * fp32, as the reference's k3_mla_cached does with its fp32 cache; the cache still receives
 * the bf16 rounding. Only the test that pins this restatement against the compiled
 * reference sets it: with it, the two compute the same arithmetic. */
static int g_mla_new_entry_fp32 = 0;
void orc_set_mla_new_entry_fp32(int on) { g_mla_new_entry_fp32 = on != 0; }

void orc_mla_decode(float *out, const float *x, int B, int hidden, int H, int q_lora,
                    int kv_lora, int qn, int qr, int vh, float theta, float eps,
                    const uint16_t *q_a, const uint16_t *q_b, const uint16_t *kv_a,
                    const uint16_t *kv_b, const uint16_t *o, const uint16_t *g,
                    const float *q_a_norm, const float *kv_a_norm, uint16_t *cache, int cap,
                    int pos)
{
    const int qh = qn + qr, kvw = kv_lora + qr, kvd = qn + vh;
    const float scale = 1.0f / sqrtf((float)qh);
    float *ql = (float *)xmalloc((size_t)q_lora * sizeof(float));
    float *q = (float *)xmalloc((size_t)H * qh * sizeof(float));
    float *c = (float *)xmalloc((size_t)kvw * sizeof(float));
    float *cl = (float *)xmalloc((size_t)kv_lora * sizeof(float));
    float *kv = (float *)xmalloc((size_t)(pos + 1) * H * kvd * sizeof(float));
    float *kr = (float *)xmalloc((size_t)(pos + 1) * qr * sizeof(float));
    float *sc = (float *)xmalloc((size_t)(pos + 1) * sizeof(float));
    float *acc = (float *)xmalloc((size_t)H * vh * sizeof(float));
    float *gb = (float *)xmalloc((size_t)H * vh * sizeof(float));
    for (int b = 0; b < B; b++) {
        const float *xb = x + (size_t)b * hidden;
        uint16_t *cb = cache + (size_t)b * cap * kvw;
        orc_matmul_bf16(ql, xb, q_a, hidden, q_lora);
        orc_rmsnorm(ql, ql, q_a_norm, q_lora, eps);
        orc_matmul_bf16(q, ql, q_b, q_lora, H * qh);
        for (int h = 0; h < H; h++) orc_rope(q + (size_t)h * qh + qn, qr, pos, theta);
        orc_matmul_bf16(c, xb, kv_a, hidden, kvw);
        orc_rmsnorm(c, c, kv_a_norm, kv_lora, eps);
        orc_rope(c + kv_lora, qr, pos, theta);
        for (int i = 0; i < kvw; i++) cb[(size_t)pos * kvw + i] = orc_f2bf(c[i]);
        for (int s = 0; s <= pos; s++) {
            const int wide = g_mla_new_entry_fp32 && s == pos;
            for (int i = 0; i < kv_lora; i++) cl[i] = wide ? c[i] : orc_bf16f(cb[(size_t)s * kvw + i]);
            for (int i = 0; i < qr; i++)
                kr[(size_t)s * qr + i] = wide ? c[kv_lora + i] : orc_bf16f(cb[(size_t)s * kvw + kv_lora + i]);
            orc_matmul_bf16(kv + (size_t)s * H * kvd, cl, kv_b, kv_lora, H * kvd);
        }
        for (int h = 0; h < H; h++) {
            const float *qt = q + (size_t)h * qh;
            float m = -INFINITY;
            for (int s = 0; s <= pos; s++) {
                const float *ks = kv + ((size_t)s * H + h) * kvd;
                double d = 0.0;
                for (int i = 0; i < qn; i++) d += (double)qt[i] * (double)ks[i];
                for (int i = 0; i < qr; i++) d += (double)qt[qn + i] * (double)kr[(size_t)s * qr + i];
                sc[s] = (float)d * scale;
                if (sc[s] > m) m = sc[s];
            }
            double z = 0.0;
            for (int s = 0; s <= pos; s++) { sc[s] = expf(sc[s] - m); z += sc[s]; }
            float *oh = acc + (size_t)h * vh;
            for (int j = 0; j < vh; j++) oh[j] = 0.0f;
            for (int s = 0; s <= pos; s++) {
                const float pr = (float)(sc[s] / z);
                const float *vs = kv + ((size_t)s * H + h) * kvd + qn;
                for (int j = 0; j < vh; j++) oh[j] += pr * vs[j];
            }
        }
        if (g) {
            orc_matmul_bf16(gb, xb, g, hidden, H * vh);
            for (int i = 0; i < H * vh; i++) acc[i] *= 1.0f / (1.0f + expf(-gb[i]));
        }
        orc_matmul_bf16(out + (size_t)b * hidden, acc, o, H * vh, hidden);
    }
    free(ql); free(q); free(c); free(cl); free(kv); free(kr); free(sc); free(acc); free(gb);
}

/* config 2 in the ABSORBED form: the same attention as orc_mla_decode (k3_ops.c:321-410's
 * arithmetic with this file's RoPE and bf16 latent cache), with kv_b folded into the query
 * and the output instead of expanding every cached latent. Per head h, with W_uk[h] the
 * qn rows of kv_b that make the keys and W_uv[h] the vh rows that make the values:
 *   q_lat = W_uk[h]^T q_nope,  score_s = (q_lat . c_s + q_rope . kr_s) * scale,
 *   p = softmax(score) (float exp, double sum, as the reference),
 *   ctx = sum_s p_s c_s,  o_h = W_uv[h] ctx.
 * Every sum runs in double, so the only roundings are the float score, the float exp and
 * the float probability, as in the expanded form; the expanded form's fp32 rounding of each
 * expanded key and value is absent here, a difference of a few fp32 ulps. O(L (2 kv_lora +
 * rope)) per head instead of O(L kv_lora (qn + vh)), which makes config 2's L = 32768 and
 * B = 32 checkable. OpenMP runs heads in parallel; each head's arithmetic is fixed. */
void orc_mla_decode_absorbed(float *out, const float *x, int B, int hidden, int H, int q_lora,
                             int kv_lora, int qn, int qr, int vh, float theta, float eps,
                             const uint16_t *q_a, const uint16_t *q_b, const uint16_t *kv_a,
                             const uint16_t *kv_b, const uint16_t *o, const uint16_t *g,
                             const float *q_a_norm, const float *kv_a_norm, uint16_t *cache,
                             int cap, int pos)
{
    const int qh = qn + qr, kvw = kv_lora + qr, kvd = qn + vh;
    const float scale = 1.0f / sqrtf((float)qh);
    const int L = pos + 1;
    float *ql = (float *)xmalloc((size_t)q_lora * sizeof(float));
    float *q = (float *)xmalloc((size_t)H * qh * sizeof(float));
    float *c = (float *)xmalloc((size_t)kvw * sizeof(float));
    float *cf = (float *)xmalloc((size_t)L * kvw * sizeof(float));
    float *acc = (float *)xmalloc((size_t)H * vh * sizeof(float));
    float *gb = (float *)xmalloc((size_t)H * vh * sizeof(float));
    for (int b = 0; b < B; b++) {
        const float *xb = x + (size_t)b * hidden;
        uint16_t *cb = cache + (size_t)b * cap * kvw;
        orc_matmul_bf16(ql, xb, q_a, hidden, q_lora);
        orc_rmsnorm(ql, ql, q_a_norm, q_lora, eps);
        orc_matmul_bf16(q, ql, q_b, q_lora, H * qh);
        for (int h = 0; h < H; h++) orc_rope(q + (size_t)h * qh + qn, qr, pos, theta);
        orc_matmul_bf16(c, xb, kv_a, hidden, kvw);
        orc_rmsnorm(c, c, kv_a_norm, kv_lora, eps);
        orc_rope(c + kv_lora, qr, pos, theta);
        for (int i = 0; i < kvw; i++) cb[(size_t)pos * kvw + i] = orc_f2bf(c[i]);
        #pragma omp parallel for schedule(static)
        for (long i = 0; i < (long)L * kvw; i++) cf[i] = orc_bf16f(cb[i]);
        #pragma omp parallel for schedule(dynamic, 1)
        for (int h = 0; h < H; h++) {
            const float *qt = q + (size_t)h * qh;
            double *qlat = (double *)xmalloc((size_t)kv_lora * sizeof(double));
            double *ctx = (double *)xmalloc((size_t)kv_lora * sizeof(double));
            float *sc = (float *)xmalloc((size_t)L * sizeof(float));
            for (int i = 0; i < kv_lora; i++) { qlat[i] = 0.0; ctx[i] = 0.0; }
            for (int j = 0; j < qn; j++) {
                const uint16_t *wr = kv_b + ((size_t)h * kvd + j) * kv_lora;
                const double qj = (double)qt[j];
                for (int i = 0; i < kv_lora; i++) qlat[i] += qj * (double)orc_bf16f(wr[i]);
            }
            float m = -INFINITY;
            for (int s_ = 0; s_ < L; s_++) {
                const float *cs = cf + (size_t)s_ * kvw;
                double d = 0.0;
                for (int i = 0; i < kv_lora; i++) d += qlat[i] * (double)cs[i];
                for (int i = 0; i < qr; i++) d += (double)qt[qn + i] * (double)cs[kv_lora + i];
                sc[s_] = (float)d * scale;
                if (sc[s_] > m) m = sc[s_];
            }
            double z = 0.0;
            for (int s_ = 0; s_ < L; s_++) { sc[s_] = expf(sc[s_] - m); z += sc[s_]; }
            for (int s_ = 0; s_ < L; s_++) {
                const double pr = (double)(float)(sc[s_] / z);
                const float *cs = cf + (size_t)s_ * kvw;
                for (int i = 0; i < kv_lora; i++) ctx[i] += pr * (double)cs[i];
            }
            for (int j = 0; j < vh; j++) {
                const uint16_t *wr = kv_b + ((size_t)h * kvd + qn + j) * kv_lora;
                double d = 0.0;
                for (int i = 0; i < kv_lora; i++) d += (double)orc_bf16f(wr[i]) * ctx[i];
                acc[(size_t)h * vh + j] = (float)d;
            }
            free(qlat); free(ctx); free(sc);
        }
        if (g) {
            orc_matmul_bf16(gb, xb, g, hidden, H * vh);
            for (int i = 0; i < H * vh; i++) acc[i] *= 1.0f / (1.0f + expf(-gb[i]));
        }
        orc_matmul_bf16(out + (size_t)b * hidden, acc, o, H * vh, hidden);
    }
    free(ql); free(q); free(c); free(cf); free(acc); free(gb);
}
