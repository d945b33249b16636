/* k3_stack.c -- the synthetic K3 decode stack (config 4), host side in C99.
 *
 * This is the B200 counterpart of the CPU engine's forward() (src/cli/k3_run.c:561-679):
 * embed the token, run every decoder layer, final RMSNorm, LM head, argmax. Each layer is
 * pre-norm residual (the benchmark lists no AttnRes weights): h += attention(norm(h));
 * h += mlp(norm(h)), with KDA or MLA attention by the layer map and a dense SwiGLU MLP on
 * the first_dense layers, the routed MoE elsewhere. All device work goes through the
 * public C ABI of k3_cuda.h; the whole step is captured once into a CUDA graph and
 * replayed, so a decode step is one graph launch.
 *
 * Weights are random-initialised on the device from a seed (the benchmark's synthetic
 * random-init data). Under expert parallelism (k3d_ep_init with more than one rank) each
 * rank allocates only the experts in cfg->moe.[expert_lo, expert_hi) and the step sums
 * the per-rank MoE partials with one NCCL all-reduce per MoE layer.
 */
#include <math.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "k3_cuda.h"

#define K3S_MAX_LAYERS 16
#define K3S_MAX_BATCH 64
#define K3S_MAX_TENSORS 4096

typedef struct {
    char name[64];
    void *ptr;
    size_t bytes;
} K3sTensor;

typedef struct {
    int is_mla, is_dense;
    float *in_norm, *post_norm;
    /* KDA */
    K3dKdaW kda;
    K3dKdaShape kshape;
    float *kda_state;              /* [B][state floats] */
    /* MLA */
    K3dMlaW mla;
    uint16_t *cache;               /* [B][cap][kv_lora + rope] */
    /* dense */
    uint16_t *dg, *du, *dd;
    /* MoE */
    K3dMoeW moe;
    K3ExpertQ *table;              /* device [n_experts] */
    unsigned char *pool;           /* experts [lo, hi), 6 tensors each */
} K3sLayer;

struct K3dModel {
    K3dStackCfg c;
    K3sLayer L[K3S_MAX_LAYERS];
    uint16_t *embed, *lm_head;     /* lm_head: rows [v0, v0 + vshard) of the vocabulary */
    int v0, vshard;                /* the whole vocabulary on one rank; a slice per rank under EP */
    float *final_norm;
    float *h, *xn, *mo;            /* [B][hidden] */
    float *logits;                 /* [B][vocab] */
    int *ids, *next, *pos;         /* device */
    int *ids_host, *next_host;     /* pinned */
    void *key;                     /* argmax keys */
    float *mlp_ws;
    void *ws;
    size_t ws_bytes;
    void *graph;
    const int *g_ids;
    int *g_next;
    float *g_logits;
    int use_graph, warmed;
    int hpos;                      /* positions the caches hold (the host's copy of pos) */
    uint64_t seed, counter;
    double step_bytes;
    K3sTensor t[K3S_MAX_TENSORS];
    int nt;
    unsigned char *stage_expert;   /* creation only: checkpoint-layout expert before tiling */
    int sh_lo, sh_full;            /* this rank's first shared-expert row, and the full count */
    /* tensor parallelism of the trunk under Mode R: a rank holds heads [h0, h0 + nh) of
     * every KDA (and MLA) layer and rows [i0, i0 + ni) of the dense MLP, and its partial
     * output is summed over the ranks by the push combine */
    int tp_kda, tp_mla, tp_dense;
    int kda_h0, mla_h0, dense_i0, dense_ni;
    K3dMlaShape mla_loc;           /* the MLA shape this rank runs (its heads) */
};

static int is_mla_layer(const K3dStackCfg *c, int l)
{
    for (int i = 0; i < 16 && c->mla_layers[i] >= 0; i++)
        if (c->mla_layers[i] == l) return 1;
    return 0;
}

static void *reg(K3dModel *m, const char *name, void *p, size_t bytes)
{
    if (p && m->nt < K3S_MAX_TENSORS) {
        K3sTensor *t = &m->t[m->nt++];
        snprintf(t->name, sizeof t->name, "%s", name);
        t->ptr = p;
        t->bytes = bytes;
    }
    return p;
}

static void *dalloc(K3dModel *m, const char *name, size_t bytes)
{
    void *p = k3d_alloc(bytes);
    return reg(m, name, p, bytes);
}

static size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

/* One expert's six tensors in the checkpoint layout (gate codes, gate scales, up codes, up
 * scales, down codes, down scales, each 256-byte aligned; per = the expert's bytes), and the
 * offsets of the tiled layout ([gate/up codes][gate/up scales][down codes][down scales]),
 * which fits in the same per. */
static void expert_layout(const K3dMoeShape *s, int E, size_t sz[6], size_t off[6], size_t *per,
                          size_t toff[4])
{
    const size_t gu = (size_t)s->inter * E / 2, gus = (size_t)s->inter * E / 32;
    const size_t z[6] = {gu, gus, gu, gus, gu, gus};
    *per = 0;
    for (int i = 0; i < 6; i++) { sz[i] = z[i]; off[i] = *per; *per += align256(z[i]); }
    const size_t tsz[4] = {2 * gu, 2 * gus, gu, gus};
    size_t tper = 0;
    for (int i = 0; i < 4; i++) { toff[i] = tper; tper += align256(tsz[i]); }
}

static uint64_t next_seed(K3dModel *m) { return m->seed * 1000003ull + (++m->counter) * 7919ull; }

static uint16_t *bf16_param(K3dModel *m, const char *name, size_t n, float sd, int *err)
{
    uint16_t *p = (uint16_t *)dalloc(m, name, n * 2);
    if (!p || k3d_fill_bf16_normal(p, n, next_seed(m), sd)) { *err = 1; return NULL; }
    m->step_bytes += 0.0;  /* weights are counted when a step reads them */
    return p;
}

static float *f32_uniform(K3dModel *m, const char *name, size_t n, float lo, float hi, int *err)
{
    float *p = (float *)dalloc(m, name, n * 4);
    if (!p || k3d_fill_f32_uniform(p, n, next_seed(m), lo, hi)) { *err = 1; return NULL; }
    return p;
}



/* Slices of seeded parameters: exactly the bytes a single GPU's tensor holds there. */
static uint16_t *bf16_rows(K3dModel *m, const char *name, size_t cols, size_t r0, size_t nr, float sd, int *err)
{
    uint16_t *p = (uint16_t *)dalloc(m, name, nr * cols * 2);
    if (!p || k3d_fill_bf16_normal_at(p, nr * cols, next_seed(m), sd, r0 * cols)) { *err = 1; return NULL; }
    return p;
}

static uint16_t *bf16_cols(K3dModel *m, const char *name, size_t rows, size_t cols, size_t c0, size_t nc, float sd,
                           int *err)
{
    uint16_t *p = (uint16_t *)dalloc(m, name, rows * nc * 2);
    uint16_t *full = (uint16_t *)k3d_alloc(rows * cols * 2);
    if (!p || !full || k3d_fill_bf16_normal(full, rows * cols, next_seed(m), sd) ||
        k3d_copy2d(p, nc * 2, full + c0, cols * 2, nc * 2, rows) || k3d_sync())
        *err = 1;
    k3d_free(full);
    return p;
}

static float *f32_normal_slice(K3dModel *m, const char *name, size_t i0, size_t n, float sd, int *err)
{
    float *p = (float *)dalloc(m, name, n * 4);
    if (!p || k3d_fill_f32_normal_at(p, n, next_seed(m), sd, i0)) { *err = 1; return NULL; }
    return p;
}

static float *f32_uniform_slice(K3dModel *m, const char *name, size_t i0, size_t n, float lo, float hi, int *err)
{
    float *p = (float *)dalloc(m, name, n * 4);
    if (!p || k3d_fill_f32_uniform_at(p, n, next_seed(m), lo, hi, i0)) { *err = 1; return NULL; }
    return p;
}

K3dModel *k3d_model_create(const K3dStackCfg *cfg, uint64_t seed)
{
    if (!cfg || cfg->n_layers < 1 || cfg->n_layers > K3S_MAX_LAYERS || cfg->batch < 1 ||
        cfg->batch > K3S_MAX_BATCH || cfg->ctx_cap < 1 || cfg->hidden < 1 || cfg->vocab < 1)
        return NULL;
    if (k3d_init(k3d_device() < 0 ? 0 : k3d_device())) return NULL;
    K3dModel *m = (K3dModel *)calloc(1, sizeof(K3dModel));
    if (!m) return NULL;
    m->c = *cfg;
    m->seed = seed;
    m->use_graph = 1;
    /* Under expert parallelism the shared expert is split over the ranks by its
     * intermediate rows: rank r computes rows [r SI / N, (r + 1) SI / N) of gate and up and
     * the same columns of down, and its partial rides the routed experts' combine (SwiGLU
     * acts row by row, so the partials sum to the whole expert). */
    const int sh_full = m->c.moe.shared_inter;
    int sh_lo = 0;
    {
        const int nr = k3d_ep_size(), r = k3d_ep_rank();
        if (m->c.ep_tokens) {
            /* Mode A: every rank's own tokens through the whole shared expert */
            m->c.moe.add_shared = 1;
        } else if (nr > 1 && sh_full > 0 && sh_full % (8 * nr) == 0) {
            m->c.moe.shared_inter = sh_full / nr;
            m->c.moe.add_shared = 1;
            sh_lo = r * (sh_full / nr);
        }
    }
    m->sh_lo = sh_lo;
    m->sh_full = sh_full;
    {
        const int nr = k3d_ep_size(), r = k3d_ep_rank();
        const int tp = nr > 1 && !m->c.ep_tokens;
        const K3dMlaShape *ms = &m->c.mla;
        m->tp_kda = tp && m->c.kda_heads % nr == 0;
        m->tp_mla = tp && ms->n_heads % nr == 0 && (ms->n_heads / nr) % 8 == 0;
        m->tp_dense = tp && m->c.dense_inter % (64 * nr) == 0;
        m->kda_h0 = m->tp_kda ? r * (m->c.kda_heads / nr) : 0;
        m->mla_h0 = m->tp_mla ? r * (ms->n_heads / nr) : 0;
        m->dense_ni = m->tp_dense ? m->c.dense_inter / nr : m->c.dense_inter;
        m->dense_i0 = m->tp_dense ? r * m->dense_ni : 0;
        m->mla_loc = *ms;
        if (m->tp_mla) m->mla_loc.n_heads = ms->n_heads / nr;
    }
    const K3dStackCfg *c = &m->c;
    const int E = c->hidden, B = c->batch;
    const size_t P = (size_t)c->kda_heads * c->kda_head_dim;
    const int D = c->kda_head_dim, H = c->kda_heads;
    int err = 0;
    char nm[64];
    size_t ws = 0;

    m->embed = bf16_param(m, "embed", (size_t)c->vocab * E, 0.02f, &err);
    {
        /* under EP each rank holds one slice of the LM head: the same rows of the same
         * seeded matrix a single GPU holds, so the argmax over the slices is the same */
        const int nr = c->ep_tokens ? 1 : k3d_ep_size(), r = c->ep_tokens ? 0 : k3d_ep_rank();
        m->v0 = (int)((long long)r * c->vocab / nr);
        m->vshard = (int)((long long)(r + 1) * c->vocab / nr) - m->v0;
        const uint64_t sd = next_seed(m);
        m->lm_head = (uint16_t *)dalloc(m, "lm_head", (size_t)m->vshard * E * 2);
        if (!m->lm_head || k3d_fill_bf16_normal_at(m->lm_head, (size_t)m->vshard * E, sd, 0.02f,
                                                   (size_t)m->v0 * E))
            err = 1;
    }
    m->final_norm = f32_uniform(m, "final_norm", E, 0.9f, 1.1f, &err);

    for (int l = 0; l < c->n_layers && !err; l++) {
        K3sLayer *L = &m->L[l];
        L->is_mla = is_mla_layer(c, l);
        L->is_dense = l < c->first_dense;
        snprintf(nm, sizeof nm, "layer%d.in_norm", l);
        L->in_norm = f32_uniform(m, nm, E, 0.9f, 1.1f, &err);
        snprintf(nm, sizeof nm, "layer%d.post_norm", l);
        L->post_norm = f32_uniform(m, nm, E, 0.9f, 1.1f, &err);
        if (L->is_mla) {
            const K3dMlaShape *s = &c->mla;
            const int qh = s->qk_nope + s->qk_rope, kvw = s->kv_lora + s->qk_rope;
            const int kvd = s->qk_nope + s->v_head;
#define MLA_W(field, rows, cols) do { snprintf(nm, sizeof nm, "layer%d.mla." #field, l); \
            L->mla.field = bf16_param(m, nm, (size_t)(rows) * (cols), 0.02f, &err); } while (0)
            /* under tensor parallelism: this rank's heads' rows of q_b, kv_b and g and
             * columns of o; q_a, kv_a and the latent cache are replicated */
            const size_t hl = (size_t)m->mla_loc.n_heads, h0 = (size_t)m->mla_h0;
            MLA_W(q_a, s->q_lora, E);
            snprintf(nm, sizeof nm, "layer%d.mla.q_b", l);
            L->mla.q_b = bf16_rows(m, nm, s->q_lora, h0 * qh, hl * qh, 0.02f, &err);
            MLA_W(kv_a, kvw, E);
            snprintf(nm, sizeof nm, "layer%d.mla.kv_b", l);
            L->mla.kv_b = bf16_rows(m, nm, s->kv_lora, h0 * kvd, hl * kvd, 0.02f, &err);
            snprintf(nm, sizeof nm, "layer%d.mla.o", l);
            L->mla.o = m->tp_mla ? bf16_cols(m, nm, E, (size_t)s->n_heads * s->v_head, h0 * s->v_head,
                                              hl * s->v_head, 0.02f, &err)
                                 : bf16_param(m, nm, (size_t)E * s->n_heads * s->v_head, 0.02f, &err);
            if (s->out_gate) {
                snprintf(nm, sizeof nm, "layer%d.mla.g", l);
                L->mla.g = bf16_rows(m, nm, E, h0 * s->v_head, hl * s->v_head, 0.02f, &err);
            }
#undef MLA_W
            snprintf(nm, sizeof nm, "layer%d.mla.q_a_norm", l);
            L->mla.q_a_norm = f32_uniform(m, nm, s->q_lora, 0.9f, 1.1f, &err);
            snprintf(nm, sizeof nm, "layer%d.mla.kv_a_norm", l);
            L->mla.kv_a_norm = f32_uniform(m, nm, s->kv_lora, 0.9f, 1.1f, &err);
            snprintf(nm, sizeof nm, "layer%d.mla.cache", l);
            L->cache = (uint16_t *)dalloc(m, nm, (size_t)B * c->ctx_cap * kvw * 2);
            if (!L->cache || k3d_memset(L->cache, 0, (size_t)B * c->ctx_cap * kvw * 2)) err = 1;
            const size_t w = k3d_mla_ws_bytes(&m->mla_loc, B, c->ctx_cap);
            if (w > ws) ws = w;
        } else {
            /* under tensor parallelism this rank's heads [h0, h0 + hl): their rows of q, k, v,
             * g, b and f_b, their columns of o, their channels' conv taps, decays and state */
            const size_t hl = m->tp_kda ? (size_t)H / k3d_ep_size() : (size_t)H, h0 = (size_t)m->kda_h0;
            const size_t Pl = hl * D, c0 = h0 * D;
            K3dKdaShape *ks = &L->kshape;
            ks->hidden = E; ks->heads = (int)hl; ks->head_dim = D; ks->conv_k = c->conv_k;
            ks->gate_lb = c->gate_lb; ks->eps = c->eps;
#define KDA_ROWS(field, cols, r0, nrow) do { snprintf(nm, sizeof nm, "layer%d.kda." #field, l); \
            L->kda.field = bf16_rows(m, nm, (cols), (r0), (nrow), 0.02f, &err); } while (0)
            KDA_ROWS(q, E, c0, Pl); KDA_ROWS(k, E, c0, Pl); KDA_ROWS(v, E, c0, Pl); KDA_ROWS(g, E, c0, Pl);
            KDA_ROWS(b, E, h0, hl); KDA_ROWS(f_a, E, 0, (size_t)D); KDA_ROWS(f_b, (size_t)D, c0, Pl);
#undef KDA_ROWS
            snprintf(nm, sizeof nm, "layer%d.kda.o", l);
            L->kda.o = m->tp_kda ? bf16_cols(m, nm, E, P, c0, Pl, 0.02f, &err)
                                 : bf16_param(m, nm, (size_t)E * P, 0.02f, &err);
            const size_t K4 = (size_t)c->conv_k;
            snprintf(nm, sizeof nm, "layer%d.kda.q_conv", l);
            L->kda.q_conv = f32_normal_slice(m, nm, c0 * K4, Pl * K4, 0.5f, &err);
            snprintf(nm, sizeof nm, "layer%d.kda.k_conv", l);
            L->kda.k_conv = f32_normal_slice(m, nm, c0 * K4, Pl * K4, 0.5f, &err);
            snprintf(nm, sizeof nm, "layer%d.kda.v_conv", l);
            L->kda.v_conv = f32_normal_slice(m, nm, c0 * K4, Pl * K4, 0.5f, &err);
            snprintf(nm, sizeof nm, "layer%d.kda.A_log", l);
            L->kda.A_log = f32_uniform_slice(m, nm, h0, hl, 0.0f, 1.5f, &err);
            snprintf(nm, sizeof nm, "layer%d.kda.dt_bias", l);
            L->kda.dt_bias = f32_normal_slice(m, nm, c0, Pl, 0.5f, &err);
            snprintf(nm, sizeof nm, "layer%d.kda.o_norm", l);
            L->kda.o_norm = f32_uniform(m, nm, D, 0.9f, 1.1f, &err);
            const size_t sf = k3d_kda_state_floats(ks);
            snprintf(nm, sizeof nm, "layer%d.kda.state", l);
            L->kda_state = (float *)dalloc(m, nm, (size_t)B * sf * 4);
            if (!L->kda_state || k3d_memset(L->kda_state, 0, (size_t)B * sf * 4)) err = 1;
            const size_t w = k3d_kda_layer_ws_bytes(ks, B);
            if (w > ws) ws = w;
        }
        if (L->is_dense) {
            /* under tensor parallelism rows [i0, i0 + ni) of gate and up, the same columns
             * of down */
            const size_t ni = (size_t)m->dense_ni, i0 = (size_t)m->dense_i0;
            snprintf(nm, sizeof nm, "layer%d.dense.gate", l);
            L->dg = bf16_rows(m, nm, E, i0, ni, 0.02f, &err);
            snprintf(nm, sizeof nm, "layer%d.dense.up", l);
            L->du = bf16_rows(m, nm, E, i0, ni, 0.02f, &err);
            snprintf(nm, sizeof nm, "layer%d.dense.down", l);
            L->dd = m->tp_dense ? bf16_cols(m, nm, E, (size_t)c->dense_inter, i0, ni, 0.02f, &err)
                                : bf16_param(m, nm, (size_t)E * c->dense_inter, 0.02f, &err);
        } else {
            const K3dMoeShape *s = &c->moe;
            size_t sz[6], off[6], per, toff[4];
            expert_layout(s, E, sz, off, &per, toff);
            const int tiled = s->expert_layout == 1;
            const int nloc = s->expert_hi - s->expert_lo;
            snprintf(nm, sizeof nm, "layer%d.moe.pool", l);
            L->pool = (unsigned char *)dalloc(m, nm, (size_t)(nloc > 0 ? nloc : 1) * per);
            K3ExpertQ *tab = (K3ExpertQ *)calloc((size_t)s->n_experts, sizeof(K3ExpertQ));
            if (!L->pool || !tab) { err = 1; free(tab); break; }
            if (tiled && !m->stage_expert) {
                /* one checkpoint-layout expert the fills land in before tiling; freed at
                 * the end of model creation (all on the library stream, so reuse is
                 * ordered) */
                m->stage_expert = (unsigned char *)k3d_alloc(per);
                if (!m->stage_expert) { err = 1; free(tab); break; }
            }
            /* one seed per matrix kind and layer, mixed with the expert index: expert e
             * holds the same bytes whichever rank fills it, and the seed counter advances
             * the same way on every rank (the weights after this layer match too) */
            uint64_t msd[3];
            for (int j = 0; j < 3; j++) msd[j] = next_seed(m);
            for (int e = s->expert_lo; e < s->expert_hi && !err; e++) {
                unsigned char *base = L->pool + (size_t)(e - s->expert_lo) * per;
                unsigned char *src = tiled ? m->stage_expert : base;
                K3ExpertQ q;
                q.p1 = src + off[0]; q.s1 = src + off[1];
                q.p3 = src + off[2]; q.s3 = src + off[3];
                q.p2 = src + off[4]; q.s2 = src + off[5];
                for (int j = 0; j < 3; j++)
                    if (k3d_fill_mxfp4(src + off[2 * j], sz[2 * j], src + off[2 * j + 1],
                                       sz[2 * j + 1], msd[j] ^ ((uint64_t)(e + 1) * 0x9E3779B97F4A7C15ull),
                                       117, 121))
                        err = 1;
                if (tiled) {
                    K3ExpertQ t;
                    t.p1 = base + toff[0]; t.s1 = base + toff[1];
                    t.p3 = NULL; t.s3 = NULL;
                    t.p2 = base + toff[2]; t.s2 = base + toff[3];
                    if (k3d_expert_pretile(&t, &q, E, s->inter)) err = 1;
                    tab[e] = t;
                } else {
                    tab[e] = q;
                }
            }
            snprintf(nm, sizeof nm, "layer%d.moe.table", l);
            L->table = (K3ExpertQ *)dalloc(m, nm, (size_t)s->n_experts * sizeof(K3ExpertQ));
            if (!L->table || k3d_upload(L->table, tab, (size_t)s->n_experts * sizeof(K3ExpertQ)))
                err = 1;
            free(tab);
            L->moe.experts = L->table;
            snprintf(nm, sizeof nm, "layer%d.moe.router_w", l);
            L->moe.router_w = bf16_param(m, nm, (size_t)s->n_experts * E, 0.02f, &err);
            snprintf(nm, sizeof nm, "layer%d.moe.router_bias", l);
            L->moe.router_bias = f32_uniform(m, nm, s->n_experts, -0.1f, 0.1f, &err);
            if (s->shared_inter > 0 && s->shared_inter == sh_full) {
                snprintf(nm, sizeof nm, "layer%d.moe.sh_gate", l);
                L->moe.sh_gate = bf16_param(m, nm, (size_t)s->shared_inter * E, 0.02f, &err);
                snprintf(nm, sizeof nm, "layer%d.moe.sh_up", l);
                L->moe.sh_up = bf16_param(m, nm, (size_t)s->shared_inter * E, 0.02f, &err);
                snprintf(nm, sizeof nm, "layer%d.moe.sh_down", l);
                L->moe.sh_down = bf16_param(m, nm, (size_t)E * s->shared_inter, 0.02f, &err);
            } else if (s->shared_inter > 0) {
                /* this rank's slice of the same seeded matrices a single GPU holds */
                const size_t SIl = (size_t)s->shared_inter;
                uint16_t **dst[2] = {(uint16_t **)&L->moe.sh_gate, (uint16_t **)&L->moe.sh_up};
                const char *nms[2] = {"sh_gate", "sh_up"};
                for (int k = 0; k < 2 && !err; k++) {
                    snprintf(nm, sizeof nm, "layer%d.moe.%s", l, nms[k]);
                    uint16_t *pk = (uint16_t *)dalloc(m, nm, SIl * E * 2);
                    if (!pk || k3d_fill_bf16_normal_at(pk, SIl * E, next_seed(m), 0.02f, (size_t)sh_lo * E))
                        err = 1;
                    *dst[k] = pk;
                }
                snprintf(nm, sizeof nm, "layer%d.moe.sh_down", l);
                uint16_t *pd = (uint16_t *)dalloc(m, nm, (size_t)E * SIl * 2);
                uint16_t *full = (uint16_t *)k3d_alloc((size_t)E * sh_full * 2);
                if (!pd || !full || k3d_fill_bf16_normal(full, (size_t)E * sh_full, next_seed(m), 0.02f) ||
                    k3d_copy2d(pd, SIl * 2, full + sh_lo, (size_t)sh_full * 2, SIl * 2, (size_t)E) ||
                    k3d_sync())
                    err = 1;
                k3d_free(full);
                L->moe.sh_down = pd;
            }
            const size_t w = c->ep_tokens ? k3d_moe_a2a_ws_bytes(&c->moe, B, k3d_ep_size())
                                          : k3d_moe_ws_bytes(&c->moe, B);
            if (w > ws) ws = w;
        }
    }
    if (!err) {
        m->h = (float *)dalloc(m, "h", (size_t)B * E * 4);
        m->xn = (float *)dalloc(m, "xn", (size_t)B * E * 4);
        m->mo = (float *)dalloc(m, "mo", (size_t)B * E * 4);
        m->logits = (float *)dalloc(m, "logits", (size_t)B * c->vocab * 4);
        m->ids = (int *)dalloc(m, "ids", (size_t)B * 4);
        m->next = (int *)dalloc(m, "next", (size_t)B * 4);
        m->pos = (int *)dalloc(m, "pos", 16);
        m->key = dalloc(m, "argmax_key", (size_t)B * 8);
        m->mlp_ws = (float *)dalloc(m, "mlp_ws", (size_t)B * (c->dense_inter > 0 ? c->dense_inter : 1) * 4);
        m->ws_bytes = ws;
        m->ws = dalloc(m, "ws", ws);
        m->ids_host = (int *)k3d_host_alloc((size_t)B * 4);
        m->next_host = (int *)k3d_host_alloc((size_t)B * 4);
        if (!m->h || !m->xn || !m->mo || !m->logits || !m->ids || !m->next || !m->pos ||
            !m->key || !m->mlp_ws || !m->ws || !m->ids_host || !m->next_host)
            err = 1;
        if (!err && k3d_memset(m->pos, 0, 16)) err = 1;
        if (!err && k3d_sync()) err = 1;
        /* the peer buffers of the MoE combine (every rank maps every other rank's) */
        if (!err && k3d_ep_size() > 1 && !c->ep_tokens && k3d_ep_peer_init((size_t)B * E)) err = 1;
    }
    if (m->stage_expert) {
        if (k3d_sync()) err = 1;
        k3d_free(m->stage_expert);
        m->stage_expert = NULL;
    }
    if (err) {
        k3d_model_destroy(m);
        return NULL;
    }
    return m;
}

void k3d_model_destroy(K3dModel *m)
{
    if (!m) return;
    if (m->graph) k3d_graph_destroy(m->graph);
    for (int i = 0; i < m->nt; i++) k3d_free(m->t[i].ptr);
    k3d_host_free(m->ids_host);
    k3d_host_free(m->next_host);
    free(m);
}

int k3d_model_fill_context(K3dModel *m, int len, uint64_t seed)
{
    if (!m || len < 0 || len >= m->c.ctx_cap) return K3D_EINVAL;
    const K3dStackCfg *c = &m->c;
    const int B = c->batch;
    /* the seeds follow the global sequence index: under Mode A rank r's sequences are the
     * batch's [r B, (r + 1) B), filled as one GPU holding the whole batch fills them */
    const int g0 = c->ep_tokens ? k3d_ep_rank() * B : 0;
    for (int l = 0; l < c->n_layers; l++) {
        K3sLayer *L = &m->L[l];
        if (L->is_mla) {
            const int kvw = c->mla.kv_lora + c->mla.qk_rope;
            for (int b = 0; b < B && len > 0; b++) {
                int r = k3d_fill_bf16_normal(L->cache + (size_t)b * c->ctx_cap * kvw,
                                             (size_t)len * kvw, seed * 131 + l * 17 + (g0 + b), 1.0f);
                if (r) return r;
            }
        } else {
            /* this rank's heads' slice of the state a single GPU holds: the state matrices
             * [H][D][D] of heads [h0, h0 + hl) and the q, k, v conv histories of their
             * channels, from the same seeded streams */
            const size_t sf = k3d_kda_state_floats(&L->kshape);
            const size_t D = (size_t)L->kshape.head_dim, hl = (size_t)L->kshape.heads, h0 = (size_t)m->kda_h0;
            const size_t ns = hl * D * D, Pl = hl * D, P = (size_t)c->kda_heads * D, hk = (size_t)c->conv_k - 1;
            for (int b = 0; b < B; b++) {
                float *st = L->kda_state + (size_t)b * sf;
                int r = k3d_fill_f32_normal_at(st, ns, seed * 137 + l * 19 + (g0 + b), 0.01f, h0 * D * D);
                for (int j = 0; j < 3 && !r; j++)
                    r = k3d_fill_f32_normal_at(st + ns + (size_t)j * Pl * hk, Pl * hk, seed * 139 + l * 23 + (g0 + b),
                                               1.0f, (size_t)j * P * hk + h0 * D * hk);
                if (r) return r;
            }
        }
    }
    int p[4] = {len, len, len, len};
    m->hpos = len;
    return k3d_upload(m->pos, p, sizeof p);
}

/* One decode step, launched eagerly on the library stream. */
static int step_eager(K3dModel *m, const int *ids, int *next, float *logits)
{
    const K3dStackCfg *c = &m->c;
    const int B = c->batch, E = c->hidden;
    const int ep = k3d_ep_size() > 1;
    int r;
#define TRY(x) do { if ((r = (x)) != 0) return r; } while (0)
    TRY(k3d_embed_bf16(m->h, ids, m->embed, B, E, c->vocab));
    for (int l = 0; l < c->n_layers; l++) {
        K3sLayer *L = &m->L[l];
        /* the layer applies its input RMSNorm itself (inside its projection GEMV); under
         * tensor parallelism it writes this rank's heads' partial, which the push combine
         * sums into the residual */
        if (L->is_mla && m->tp_mla) {
            TRY(k3d_mla_decode_normed(m->mo, m->h, L->in_norm, c->eps, &L->mla, &m->mla_loc, B, L->cache,
                                      c->ctx_cap, m->pos, 0, m->ws, m->ws_bytes));
            TRY(k3d_ep_combine_add(m->h, m->mo, (size_t)B * E, 1));
        } else if (L->is_mla) {
            TRY(k3d_mla_decode_normed(m->h, m->h, L->in_norm, c->eps, &L->mla, &m->mla_loc, B, L->cache,
                                      c->ctx_cap, m->pos, 1, m->ws, m->ws_bytes));
        } else if (m->tp_kda) {
            TRY(k3d_kda_layer_decode_normed_out(m->mo, m->h, L->in_norm, c->eps, &L->kda, &L->kshape, B,
                                                L->kda_state, m->ws, m->ws_bytes, 0));
            TRY(k3d_ep_combine_add(m->h, m->mo, (size_t)B * E, 1));
        } else {
            TRY(k3d_kda_layer_decode_normed(m->h, L->in_norm, c->eps, &L->kda, &L->kshape, B,
                                            L->kda_state, m->ws, m->ws_bytes));
        }
        TRY(k3d_rmsnorm(m->xn, m->h, L->post_norm, E, B, c->eps));
        if (L->is_dense && m->tp_dense) {
            TRY(k3d_swiglu_mlp_bf16(m->mo, m->xn, L->dg, L->du, L->dd, E, m->dense_ni, B, 0, m->mlp_ws));
            TRY(k3d_ep_combine_add(m->h, m->mo, (size_t)B * E, 1));
        } else if (L->is_dense) {
            TRY(k3d_swiglu_mlp_bf16(m->h, m->xn, L->dg, L->du, L->dd, E, c->dense_inter, B, 1,
                                    m->mlp_ws));
        } else if (c->ep_tokens) {
            /* Mode A: this rank's tokens' rows to their experts' ranks and back, planned on
             * the device (fixed-size exchanges), the top-k sum and the shared expert added
             * into the residual */
            TRY(k3d_moe_swiglu_a2a_dev(m->h, m->xn, &L->moe, &c->moe, B, 1, NULL, NULL, m->ws, m->ws_bytes));
        } else if (ep) {
            /* this rank's experts (and shared-expert slice), then the NVLink push combine
             * that sums every rank's partial into the residual */
            TRY(k3d_moe_swiglu(m->mo, m->xn, &L->moe, &c->moe, B, 0, NULL, NULL, m->ws, m->ws_bytes));
            TRY(k3d_ep_combine_add(m->h, m->mo, (size_t)B * E, 1));
        } else {
            TRY(k3d_moe_swiglu(m->h, m->xn, &L->moe, &c->moe, B, 1, NULL, NULL, m->ws, m->ws_bytes));
        }
    }
    if (m->vshard == c->vocab)
        TRY(k3d_lm_head_argmax_normed(next, logits, m->h, m->final_norm, c->eps, m->lm_head, c->vocab,
                                      E, B, m->key));
    else
        TRY(k3d_lm_head_argmax_shard_normed(next, logits, m->h, m->final_norm, c->eps, m->lm_head, m->v0,
                                            m->vshard, E, B, m->key));
    TRY(k3d_add_i32(m->pos, 1, 1));
#undef TRY
    return K3D_OK;
}

int k3d_model_use_graph(K3dModel *m, int on)
{
    if (!m) return K3D_EINVAL;
    m->use_graph = on;
    return K3D_OK;
}

int k3d_model_step_dev(K3dModel *m, const int *ids, int *next_ids, float *logits)
{
    if (!m || !ids || !next_ids) return K3D_EINVAL;
    /* a step writes cache position hpos: refused once the caches are full (the kernels
     * would only raise a device error and skip the attention) */
    if (m->hpos >= m->c.ctx_cap) return K3D_EBOUND;
    if (!m->use_graph || !m->warmed) {
        /* the first step runs eagerly: it initialises every kernel's attributes and
         * lazily created buffers before anything is captured */
        int r = step_eager(m, ids, next_ids, logits);
        if (!r) m->warmed = 1;
        if (!r) m->hpos++;
        return r;
    }
    if (!m->graph || m->g_ids != ids || m->g_next != next_ids || m->g_logits != logits) {
        if (m->graph) { k3d_graph_destroy(m->graph); m->graph = NULL; }
        /* stream priorities in the graph (the router and routed experts ahead of the
         * side stream's shared expert): batch-1 decode 534 -> 542 tok/s; above four
         * sequences, where the shared expert is a tensor-core GEMM, 2% slower */
        k3d_set_graph_priorities(m->c.batch <= 4);
        int r = k3d_graph_begin();
        if (r) return r;
        r = step_eager(m, ids, next_ids, logits);
        void *g = k3d_graph_end();
        if (r) { k3d_graph_destroy(g); return r; }
        if (!g) return k3d_status() ? k3d_status() : K3D_ECUDA;
        m->graph = g;
        m->g_ids = ids;
        m->g_next = next_ids;
        m->g_logits = logits;
    }
    const int r = k3d_graph_launch(m->graph);
    if (!r) m->hpos++;
    return r;
}

int k3d_model_step_host(K3dModel *m, const int *ids_host, int *next_host)
{
    if (!m || !ids_host || !next_host) return K3D_EINVAL;
    const size_t n = (size_t)m->c.batch * sizeof(int);
    memcpy(m->ids_host, ids_host, n);
    int r = k3d_upload(m->ids, m->ids_host, n);
    if (!r) r = k3d_model_step_dev(m, m->ids, m->next, m->logits);
    if (!r) r = k3d_download(m->next_host, m->next, n);
    if (!r) memcpy(next_host, m->next_host, n);
    return r;
}

void *k3d_model_tensor(K3dModel *m, const char *name, size_t *bytes)
{
    if (!m || !name) return NULL;
    for (int i = 0; i < m->nt; i++)
        if (!strcmp(m->t[i].name, name)) {
            if (bytes) *bytes = m->t[i].bytes;
            return m->t[i].ptr;
        }
    return NULL;
}

/* Algorithmic HBM bytes of one step: every weight a token reads (routed experts counted
 * for the unique experts of the last MoE call, shared expert, router), KDA states read
 * and written, the MLA cache read over pos + 1 positions and one entry written. */
double k3d_model_last_step_bytes(K3dModel *m)
{
    if (!m) return 0.0;
    const K3dStackCfg *c = &m->c;
    const double E = c->hidden, B = c->batch;
    double bytes = 2.0 * m->vshard * E + 2.0 * B * E * 4;   /* lm_head (this rank's rows) + embed rows */
    int pos = 0;
    k3d_download(&pos, m->pos, sizeof pos);
    const int U = k3d_moe_last_unique();
    for (int l = 0; l < c->n_layers; l++) {
        const K3sLayer *L = &m->L[l];
        bytes += 2.0 * E * 4;                                /* norms */
        if (L->is_mla) {
            const K3dMlaShape *s = &m->mla_loc;                 /* this rank's heads */
            const double qh = s->qk_nope + s->qk_rope, kvw = s->kv_lora + s->qk_rope;
            bytes += 2.0 * (s->q_lora * E + s->n_heads * qh * s->q_lora + kvw * E +
                            s->n_heads * (double)(s->qk_nope + s->v_head) * s->kv_lora +
                            E * s->n_heads * s->v_head +
                            (s->out_gate ? s->n_heads * (double)s->v_head * E : 0.0));
            bytes += B * 2.0 * kvw * pos;                    /* cache read (pos positions) */
        } else {
            const double P = (double)L->kshape.heads * c->kda_head_dim, D = c->kda_head_dim;
            bytes += 2.0 * (4 * P * E + L->kshape.heads * E + D * E + P * D + E * P);
            bytes += B * 2.0 * 4.0 * k3d_kda_state_floats(&L->kshape);   /* read + write */
        }
        if (L->is_dense) {
            bytes += 2.0 * 3.0 * m->dense_ni * E;
        } else {
            const K3dMoeShape *s = &c->moe;
            const double per = 3.0 * (s->inter * E / 2.0 + s->inter * E / 32.0);
            bytes += (U > 0 ? U : s->topk) * per;
            bytes += 2.0 * s->n_experts * E + 2.0 * 3.0 * s->shared_inter * E;
        }
    }
    return bytes;
}

/* ------------------------------------------------------ conversation state ----
 * The CPU engine's state file (K3ST version 1, src/cli/k3_run.c:158-300): a header with a
 * configuration fingerprint, the sequence's token ids, one KDA state slot per layer
 * (k3_kda_layer's layout; zeros for MLA and dense layers), then per MLA layer the cached
 * positions of the EXPANDED keys and values (kv_b times the normalised latent, [H][nope +
 * v] per position, the CPU engine's cache) and per MLA layer the rope slots. The device
 * keeps the compressed bf16 latent instead, so saving expands it through kv_b on the
 * tensor-core GEMM, and a trailer after the CPU engine's payload ("K3LT": the cache rows
 * exactly as the device holds them) lets a device load restore them bit for bit. The CPU
 * engine reads exactly its payload and never the trailer. A file without the trailer
 * (written by the CPU engine) is loaded by recovering each position's latent from its
 * expanded keys and values by least squares: (kv_b^T kv_b) c = kv_b^T kv, the Gram matrix
 * and the right-hand sides on the GPU, the Cholesky solve in double on the host. */
#define K3ST_MAGIC "K3ST"
#define K3ST_VERSION 1
#define K3LT_MAGIC "K3LT"
#define K3ST_CHUNK 256                 /* positions per device pass */

typedef struct {
    char    magic[4];
    int32_t version;
    int32_t fp[12];
    int32_t n_bound, n_mla, cached, nseq;
    int64_t kper;
    int64_t kvpp, ropepp;
} K3StHeader;                          /* the field order and types of the CPU engine's */

typedef struct {
    char    magic[4];
    int32_t version, n_mla, cached, kvw;
} K3LtTrailer;

static void state_fingerprint(const K3dStackCfg *c, int32_t fp[12])
{
    fp[0] = c->hidden;         fp[1] = c->n_layers;      fp[2] = c->vocab;
    fp[3] = c->kda_heads;      fp[4] = c->kda_head_dim;  fp[5] = c->conv_k;
    fp[6] = c->mla.n_heads;    fp[7] = c->mla.qk_nope;   fp[8] = c->mla.qk_rope;
    fp[9] = c->mla.v_head;     fp[10] = c->moe.n_experts; fp[11] = c->moe.topk;
}

static int state_n_mla(const K3dModel *m)
{
    int n = 0;
    for (int l = 0; l < m->c.n_layers; l++) n += m->L[l].is_mla;
    return n;
}

static int64_t state_kper(const K3dStackCfg *c)
{
    const int64_t P = (int64_t)c->kda_heads * c->kda_head_dim;
    return P * c->kda_head_dim + 3 * P * (c->conv_k - 1);
}

static int read_header(FILE *f, K3StHeader *hd)
{
    if (fread(hd, 1, sizeof *hd, f) != sizeof *hd || memcmp(hd->magic, K3ST_MAGIC, 4) != 0)
        return K3D_EINVAL;
    return hd->version == K3ST_VERSION ? K3D_OK : K3D_EINVAL;
}

int k3d_state_peek(const char *path, K3dStateInfo *info)
{
    if (!path || !info) return K3D_EINVAL;
    FILE *f = fopen(path, "rb");
    if (!f) return K3D_EINVAL;
    K3StHeader hd;
    int r = read_header(f, &hd);
    memset(info, 0, sizeof *info);
    if (!r) {
        info->version = hd.version;
        info->n_bound = hd.n_bound;
        info->n_mla = hd.n_mla;
        info->cached = hd.cached;
        info->nseq = hd.nseq;
        const long tail = (long)sizeof hd + (long)hd.nseq * 4 + (long)(hd.kper * hd.n_bound * 4) +
                          (long)hd.n_mla * hd.cached * (long)(hd.kvpp + hd.ropepp) * 4;
        K3LtTrailer tr;
        info->has_latent = fseek(f, tail, SEEK_SET) == 0 && fread(&tr, 1, sizeof tr, f) == sizeof tr &&
                           memcmp(tr.magic, K3LT_MAGIC, 4) == 0;
    }
    fclose(f);
    return r;
}

/* Cholesky factor of the n x n symmetric positive definite G (lower, in place). */
static int cholesky(double *G, int n)
{
    for (int j = 0; j < n; j++) {
        double d = G[(size_t)j * n + j];
        for (int k = 0; k < j; k++) d -= G[(size_t)j * n + k] * G[(size_t)j * n + k];
        if (!(d > 0.0)) return -1;
        d = sqrt(d);
        G[(size_t)j * n + j] = d;
        for (int i = j + 1; i < n; i++) {
            double v = G[(size_t)i * n + j];
            for (int k = 0; k < j; k++) v -= G[(size_t)i * n + k] * G[(size_t)j * n + k];
            G[(size_t)i * n + j] = v / d;
        }
    }
    return 0;
}

static void chol_solve(const double *Lf, int n, const float *rhs, float *out, double *tmp)
{
    for (int i = 0; i < n; i++) {
        double v = rhs[i];
        for (int k = 0; k < i; k++) v -= Lf[(size_t)i * n + k] * tmp[k];
        tmp[i] = v / Lf[(size_t)i * n + i];
    }
    for (int i = n - 1; i >= 0; i--) {
        double v = tmp[i];
        for (int k = i + 1; k < n; k++) v -= Lf[(size_t)k * n + i] * tmp[k];
        tmp[i] = v / Lf[(size_t)i * n + i];
    }
    for (int i = 0; i < n; i++) out[i] = (float)tmp[i];
}

int k3d_model_state_save(K3dModel *m, const char *path, const int *seq, int nseq, int b)
{
    if (!m || !path || nseq < 0 || (nseq > 0 && !seq) || b < 0 || b >= m->c.batch) return K3D_EINVAL;
    if (m->tp_kda || m->tp_mla) return K3D_EINVAL;     /* a rank holds only its heads' state */
    const K3dStackCfg *c = &m->c;
    const K3dMlaShape *ms = &c->mla;
    const int kvw = ms->kv_lora + ms->qk_rope, H = ms->n_heads, kvd = ms->qk_nope + ms->v_head;
    const int64_t kper = state_kper(c);
    int pos = 0, r = k3d_sync();
    if (!r) r = k3d_download(&pos, m->pos, sizeof pos);
    if (r) return r;
    if (pos < 0 || pos > c->ctx_cap) return K3D_EBOUND;
    K3StHeader hd;
    memset(&hd, 0, sizeof hd);
    memcpy(hd.magic, K3ST_MAGIC, 4);
    hd.version = K3ST_VERSION;
    state_fingerprint(c, hd.fp);
    hd.n_bound = c->n_layers;
    hd.n_mla = state_n_mla(m);
    hd.cached = pos;
    hd.nseq = nseq;
    hd.kper = kper;
    hd.kvpp = (int64_t)H * kvd;
    hd.ropepp = ms->qk_rope;
    FILE *f = fopen(path, "wb");
    if (!f) return K3D_EINVAL;
    const int CH = K3ST_CHUNK;
    float *hbuf = (float *)malloc((size_t)(kper > (int64_t)CH * H * kvd ? kper : (int64_t)CH * H * kvd) * 4);
    float *lat = hd.n_mla ? (float *)k3d_alloc((size_t)CH * ms->kv_lora * 4) : NULL;
    float *kv = hd.n_mla ? (float *)k3d_alloc((size_t)CH * H * kvd * 4) : NULL;
    uint16_t *rows = (uint16_t *)malloc((size_t)CH * kvw * 2);
    if (!hbuf || !rows || (hd.n_mla && (!lat || !kv))) r = K3D_ENOMEM;
    if (!r && fwrite(&hd, sizeof hd, 1, f) != 1) r = K3D_EINVAL;
    if (!r && nseq && fwrite(seq, sizeof(int), (size_t)nseq, f) != (size_t)nseq) r = K3D_EINVAL;
    for (int l = 0; l < c->n_layers && !r; l++) {
        const K3sLayer *L = &m->L[l];
        if (!L->is_mla && L->kda_state) {
            r = k3d_download(hbuf, L->kda_state + (size_t)b * kper, (size_t)kper * 4);
        } else {
            memset(hbuf, 0, (size_t)kper * 4);
        }
        if (!r && fwrite(hbuf, 4, (size_t)kper, f) != (size_t)kper) r = K3D_EINVAL;
    }
    /* expanded keys and values, position-major per MLA layer */
    for (int l = 0; l < c->n_layers && !r; l++) {
        const K3sLayer *L = &m->L[l];
        if (!L->is_mla) continue;
        const uint16_t *cb = L->cache + (size_t)b * c->ctx_cap * kvw;
        for (int p0 = 0; p0 < pos && !r; p0 += CH) {
            const int n = pos - p0 < CH ? pos - p0 : CH;
            r = k3d_bf16_rows_to_f32(lat, cb + (size_t)p0 * kvw, (size_t)kvw, n, ms->kv_lora);
            if (!r) r = k3d_gemv_bf16(kv, lat, L->mla.kv_b, ms->kv_lora, H * kvd, n, 0);
            if (!r) r = k3d_download(hbuf, kv, (size_t)n * H * kvd * 4);
            if (!r && fwrite(hbuf, 4, (size_t)n * H * kvd, f) != (size_t)n * H * kvd) r = K3D_EINVAL;
        }
    }
    /* rope slots */
    for (int l = 0; l < c->n_layers && !r; l++) {
        const K3sLayer *L = &m->L[l];
        if (!L->is_mla) continue;
        const uint16_t *cb = L->cache + (size_t)b * c->ctx_cap * kvw;
        for (int p0 = 0; p0 < pos && !r; p0 += CH) {
            const int n = pos - p0 < CH ? pos - p0 : CH;
            r = k3d_bf16_rows_to_f32(lat, cb + (size_t)p0 * kvw + ms->kv_lora, (size_t)kvw, n, ms->qk_rope);
            if (!r) r = k3d_download(hbuf, lat, (size_t)n * ms->qk_rope * 4);
            if (!r && fwrite(hbuf, 4, (size_t)n * ms->qk_rope, f) != (size_t)n * ms->qk_rope) r = K3D_EINVAL;
        }
    }
    /* the trailer: the device cache rows themselves */
    if (!r && hd.n_mla) {
        K3LtTrailer tr;
        memcpy(tr.magic, K3LT_MAGIC, 4);
        tr.version = 1;
        tr.n_mla = hd.n_mla;
        tr.cached = pos;
        tr.kvw = kvw;
        if (fwrite(&tr, sizeof tr, 1, f) != 1) r = K3D_EINVAL;
        for (int l = 0; l < c->n_layers && !r; l++) {
            const K3sLayer *L = &m->L[l];
            if (!L->is_mla) continue;
            const uint16_t *cb = L->cache + (size_t)b * c->ctx_cap * kvw;
            for (int p0 = 0; p0 < pos && !r; p0 += CH) {
                const int n = pos - p0 < CH ? pos - p0 : CH;
                r = k3d_download(rows, cb + (size_t)p0 * kvw, (size_t)n * kvw * 2);
                if (!r && fwrite(rows, 2, (size_t)n * kvw, f) != (size_t)n * kvw) r = K3D_EINVAL;
            }
        }
    }
    if (fclose(f) != 0 && !r) r = K3D_EINVAL;
    free(hbuf);
    free(rows);
    k3d_free(lat);
    k3d_free(kv);
    return r;
}

/* The latent of every cached position of one MLA layer from its expanded keys and values
 * at file offset `off` (cached x H*kvd floats), written into the device cache rows. */
static int load_latent_lsq(K3dModel *m, const K3sLayer *L, uint16_t *cb, FILE *f, long off, int cached)
{
    const K3dMlaShape *ms = &m->c.mla;
    const int kvw = ms->kv_lora + ms->qk_rope, R = ms->n_heads * (ms->qk_nope + ms->v_head);
    const int n_l = ms->kv_lora, CH = K3ST_CHUNK;
    int r = 0;
    uint16_t *kvbT = (uint16_t *)k3d_alloc((size_t)n_l * R * 2);
    float *xt = (float *)k3d_alloc((size_t)(n_l > CH ? n_l : CH) * R * 4);   /* kv_b^T widened; later kv rows */
    float *rhs = (float *)k3d_alloc((size_t)(n_l > CH ? n_l : CH) * n_l * 4);
    double *G = (double *)malloc((size_t)n_l * n_l * sizeof(double));
    float *hb = (float *)malloc((size_t)(n_l > CH ? n_l : CH) * (R > n_l ? R : n_l) * 4);
    double *tmp = (double *)malloc((size_t)n_l * sizeof(double));
    if (!kvbT || !xt || !rhs || !G || !hb || !tmp) r = K3D_ENOMEM;
    /* Gram matrix kv_b^T kv_b: kv_b^T as the weight matrix, its own rows as the tokens */
    if (!r) r = k3d_transpose_u16(kvbT, L->mla.kv_b, R, n_l);
    if (!r) r = k3d_bf16_rows_to_f32(xt, kvbT, (size_t)R, n_l, R);
    if (!r) r = k3d_gemv_bf16(rhs, xt, kvbT, R, n_l, n_l, 0);
    if (!r) r = k3d_download(hb, rhs, (size_t)n_l * n_l * 4);
    if (!r) {
        for (size_t i = 0; i < (size_t)n_l * n_l; i++) G[i] = hb[i];
        if (cholesky(G, n_l)) r = K3D_EINVAL;                   /* kv_b without full rank */
    }
    if (!r && fseek(f, off, SEEK_SET) != 0) r = K3D_EINVAL;
    for (int p0 = 0; p0 < cached && !r; p0 += CH) {
        const int n = cached - p0 < CH ? cached - p0 : CH;
        if (fread(hb, 4, (size_t)n * R, f) != (size_t)n * R) { r = K3D_EINVAL; break; }
        r = k3d_upload(xt, hb, (size_t)n * R * 4);
        if (!r) r = k3d_gemv_bf16(rhs, xt, kvbT, R, n_l, n, 0);
        if (!r) r = k3d_download(hb, rhs, (size_t)n * n_l * 4);
        if (r) break;
        for (int p = 0; p < n; p++) chol_solve(G, n_l, hb + (size_t)p * n_l, hb + (size_t)p * n_l, tmp);
        r = k3d_upload(rhs, hb, (size_t)n * n_l * 4);
        if (!r) r = k3d_f32_rows_to_bf16(cb + (size_t)p0 * kvw, (size_t)kvw, rhs, n, n_l);
    }
    if (!r) r = k3d_sync();
    k3d_free(kvbT);
    k3d_free(xt);
    k3d_free(rhs);
    free(G);
    free(hb);
    free(tmp);
    return r;
}

int k3d_model_state_load(K3dModel *m, const char *path, int *seq, int seq_cap, int b)
{
    if (!m || !path || b < 0 || b >= m->c.batch) return K3D_EINVAL;
    if (m->tp_kda || m->tp_mla) return K3D_EINVAL;     /* a rank holds only its heads' state */
    const K3dStackCfg *c = &m->c;
    const K3dMlaShape *ms = &c->mla;
    const int kvw = ms->kv_lora + ms->qk_rope, H = ms->n_heads, kvd = ms->qk_nope + ms->v_head;
    FILE *f = fopen(path, "rb");
    if (!f) return K3D_EINVAL;
    K3StHeader hd;
    int32_t fp[12];
    state_fingerprint(c, fp);
    int r = read_header(f, &hd);
    /* a file from another architecture would decode fluent, wrong text: refused, as the
     * CPU engine refuses it (k3_run.c:226-240) */
    if (!r && (memcmp(fp, hd.fp, sizeof fp) != 0 || hd.n_bound != c->n_layers || hd.n_mla != state_n_mla(m) ||
               hd.kper != state_kper(c) || hd.kvpp != (int64_t)H * kvd || hd.ropepp != ms->qk_rope))
        r = K3D_EINVAL;
    if (!r && (hd.cached < 0 || hd.cached > c->ctx_cap)) r = K3D_EBOUND;
    if (!r && (hd.nseq < 0 || (hd.nseq > 0 && seq && hd.nseq > seq_cap))) r = K3D_EBOUND;
    if (r) { fclose(f); return r; }
    const int cached = hd.cached, CH = K3ST_CHUNK;
    const int64_t kper = hd.kper;
    const long after_seq = (long)sizeof hd + (long)hd.nseq * 4;
    const long kv_off = after_seq + (long)(kper * hd.n_bound * 4);
    const long rope_off = kv_off + (long)hd.n_mla * cached * (long)hd.kvpp * 4;
    const long tail = rope_off + (long)hd.n_mla * cached * (long)hd.ropepp * 4;
    if (seq && hd.nseq && fread(seq, sizeof(int), (size_t)hd.nseq, f) != (size_t)hd.nseq) r = K3D_EINVAL;
    float *hbuf = (float *)malloc((size_t)kper * 4);
    if (!hbuf) r = K3D_ENOMEM;
    if (!r && fseek(f, after_seq, SEEK_SET) != 0) r = K3D_EINVAL;
    for (int l = 0; l < c->n_layers && !r; l++) {
        K3sLayer *L = &m->L[l];
        if (fread(hbuf, 4, (size_t)kper, f) != (size_t)kper) { r = K3D_EINVAL; break; }
        if (!L->is_mla && L->kda_state) r = k3d_upload(L->kda_state + (size_t)b * kper, hbuf, (size_t)kper * 4);
    }
    free(hbuf);
    K3LtTrailer tr;
    const int exact = !r && cached > 0 && hd.n_mla > 0 && fseek(f, tail, SEEK_SET) == 0 &&
                      fread(&tr, 1, sizeof tr, f) == sizeof tr && memcmp(tr.magic, K3LT_MAGIC, 4) == 0 &&
                      tr.version == 1 && tr.n_mla == hd.n_mla && tr.cached == cached && tr.kvw == kvw;
    if (exact) {
        /* the trailer holds the device rows themselves */
        uint16_t *rows = (uint16_t *)malloc((size_t)CH * kvw * 2);
        if (!rows) r = K3D_ENOMEM;
        for (int l = 0; l < c->n_layers && !r; l++) {
            K3sLayer *L = &m->L[l];
            if (!L->is_mla) continue;
            uint16_t *cb = L->cache + (size_t)b * c->ctx_cap * kvw;
            for (int p0 = 0; p0 < cached && !r; p0 += CH) {
                const int n = cached - p0 < CH ? cached - p0 : CH;
                if (fread(rows, 2, (size_t)n * kvw, f) != (size_t)n * kvw) { r = K3D_EINVAL; break; }
                r = k3d_upload(cb + (size_t)p0 * kvw, rows, (size_t)n * kvw * 2);
            }
        }
        free(rows);
    } else if (!r && cached > 0) {
        int mi = 0;
        float *hb = (float *)malloc((size_t)CH * ms->qk_rope * 4);
        float *dv = (float *)k3d_alloc((size_t)CH * ms->qk_rope * 4);
        if (!hb || !dv) r = K3D_ENOMEM;
        for (int l = 0; l < c->n_layers && !r; l++) {
            K3sLayer *L = &m->L[l];
            if (!L->is_mla) continue;
            uint16_t *cb = L->cache + (size_t)b * c->ctx_cap * kvw;
            r = load_latent_lsq(m, L, cb, f, kv_off + (long)mi * cached * (long)hd.kvpp * 4, cached);
            if (!r && fseek(f, rope_off + (long)mi * cached * (long)hd.ropepp * 4, SEEK_SET) != 0) r = K3D_EINVAL;
            for (int p0 = 0; p0 < cached && !r; p0 += CH) {
                const int n = cached - p0 < CH ? cached - p0 : CH;
                if (fread(hb, 4, (size_t)n * ms->qk_rope, f) != (size_t)n * ms->qk_rope) { r = K3D_EINVAL; break; }
                r = k3d_upload(dv, hb, (size_t)n * ms->qk_rope * 4);
                if (!r) r = k3d_f32_rows_to_bf16(cb + (size_t)p0 * kvw + ms->kv_lora, (size_t)kvw, dv, n,
                                                 ms->qk_rope);
                if (!r) r = k3d_sync();
            }
            mi++;
        }
        free(hb);
        k3d_free(dv);
    }
    fclose(f);
    if (!r) {
        int p[4] = {cached, cached, cached, cached};
        r = k3d_upload(m->pos, p, sizeof p);
        if (!r) m->hpos = cached;
    }
    if (!r) r = k3d_sync();
    return r;
}

/* --------------------------------------------------------- checkpoint binding ----
 * The released checkpoint's names (src/model/k3_bind.c:167-241, src/io/k3_load.c:11)
 * bound to this stack's weights. All requests are resolved and checked first; only then is
 * anything read, so a checkpoint that does not fit the configuration leaves the model as
 * it was. */
void k3h_ckpt_fail(const char *fmt, ...);

#define CK_PRE "language_model.model."
enum { CK_MAT = 1, CK_VEC, CK_ROUTER, CK_SH_DOWN };

typedef struct {
    char name[160];
    int kind;
    void *dst;
    int64_t want, take, row0, rows, cols;   /* CK_MAT: rows [row0, row0 + rows) of cols; CK_SH_DOWN: columns */
    K3dCkptTensor t;
} CkReq;

typedef struct {
    CkReq *r;
    int n, cap, bad;
    const K3dCkpt *ck;
} CkPlan;

static CkReq *ck_add(CkPlan *p, int kind, void *dst, int64_t want, const char *fmt, ...)
{
    if (p->n == p->cap) {
        const int nc = p->cap ? 2 * p->cap : 256;
        CkReq *r = (CkReq *)realloc(p->r, (size_t)nc * sizeof(CkReq));
        if (!r) { p->bad++; return NULL; }
        p->r = r;
        p->cap = nc;
    }
    CkReq *q = &p->r[p->n];
    memset(q, 0, sizeof *q);
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(q->name, sizeof q->name, fmt, ap);
    va_end(ap);
    q->kind = kind;
    q->dst = dst;
    q->want = want;
    q->take = want;
    if (k3d_ckpt_find(p->ck, q->name, &q->t)) {
        if (!p->bad) k3h_ckpt_fail("missing tensor %s", q->name);
        p->bad++;
        return NULL;
    }
    int64_t numel = 1;
    for (int i = 0; i < q->t.ndim; i++) numel *= q->t.shape[i];
    const int dt = q->t.dtype;
    const char *why = NULL;
    if (want >= 0 && numel != want) why = "element count";
    else if ((kind == CK_MAT || kind == CK_SH_DOWN) && dt != K3D_DT_BF16) why = "dtype (matrices must be BF16)";
    else if (kind == CK_VEC && dt != K3D_DT_F32 && dt != K3D_DT_BF16 && dt != K3D_DT_F16) why = "dtype";
    else if (kind == CK_ROUTER && dt != K3D_DT_F32 && dt != K3D_DT_BF16) why = "dtype";
    if (why) {
        if (!p->bad)
            k3h_ckpt_fail("%s: %s does not fit the model (%lld elements, dtype %d; expected %lld)", q->name, why,
                          (long long)numel, dt, (long long)want);
        p->bad++;
        return NULL;
    }
    p->n++;
    return q;
}

static float half_to_f32(uint16_t h)
{
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 1023u;
    uint32_t u;
    if (e == 31) u = s | 0x7f800000u | (m << 13);
    else if (e) u = s | ((e + 112u) << 23) | (m << 13);
    else if (!m) u = s;
    else {                                   /* subnormal: normalise */
        int k = 0;
        uint32_t mm = m;
        while (!(mm & 1024u)) { mm <<= 1; k++; }
        u = s | ((uint32_t)(113 - k) << 23) | ((mm & 1023u) << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

#define CK_HOST (64u << 20)

static int ck_copy_bytes(const K3dCkpt *ck, const K3dCkptTensor *t, int64_t off, int64_t bytes, void *dst,
                         unsigned char *hb, const char *name)
{
    for (int64_t d = 0; d < bytes;) {
        const int64_t n = bytes - d < (int64_t)CK_HOST ? bytes - d : (int64_t)CK_HOST;
        if (k3d_ckpt_read(ck, t->shard, t->off + off + d, n, hb) != n) {
            k3h_ckpt_fail("short read of %s", name);
            return K3D_EINVAL;
        }
        const int r = k3d_upload((char *)dst + d, hb, (size_t)n);
        if (r) return r;
        d += n;
    }
    return K3D_OK;
}

static int ck_load_req(const K3dCkpt *ck, const CkReq *q, unsigned char *hb)
{
    const int es = k3d_ckpt_elem_size(q->t.dtype);
    if (q->kind == CK_MAT) {
        if (q->rows) return ck_copy_bytes(ck, &q->t, q->row0 * q->cols * 2, q->rows * q->cols * 2, q->dst, hb, q->name);
        return ck_copy_bytes(ck, &q->t, 0, q->t.nbytes, q->dst, hb, q->name);
    }
    if (q->kind == CK_SH_DOWN) {
        /* columns [row0, row0 + cols) of each of the `rows` rows of a [rows][take] matrix */
        const int64_t rowb = q->cols * 2;
        unsigned char *out = hb;
        if (q->rows * rowb > (int64_t)CK_HOST) { k3h_ckpt_fail("%s too large", q->name); return K3D_EINVAL; }
        for (int64_t r = 0; r < q->rows; r++)
            if (k3d_ckpt_read(ck, q->t.shard, q->t.off + (r * q->take + q->row0) * 2, rowb, out + r * rowb) != rowb) {
                k3h_ckpt_fail("short read of %s", q->name);
                return K3D_EINVAL;
            }
        return k3d_upload(q->dst, out, (size_t)(q->rows * rowb));
    }
    /* vectors widened to fp32 (a prefix of `take` elements), the router as bf16 */
    const int64_t n = q->kind == CK_VEC ? q->take : q->want;
    if (n * 4 > (int64_t)CK_HOST || n * es > (int64_t)CK_HOST / 2) {
        k3h_ckpt_fail("%s too large", q->name);
        return K3D_EINVAL;
    }
    unsigned char *raw = hb + CK_HOST / 2;
    if (k3d_ckpt_read(ck, q->t.shard, q->t.off, n * es, raw) != n * es) {
        k3h_ckpt_fail("short read of %s", q->name);
        return K3D_EINVAL;
    }
    if (q->kind == CK_ROUTER) {
        if (q->t.dtype == K3D_DT_BF16) return k3d_upload(q->dst, raw, (size_t)n * 2);
        uint16_t *o = (uint16_t *)hb;
        for (int64_t i = 0; i < n; i++) {
            uint32_t u;
            memcpy(&u, raw + 4 * i, 4);
            if (u & 0xffffu) {
                k3h_ckpt_fail("%s: fp32 router weights that bf16 does not hold exactly", q->name);
                return K3D_EINVAL;
            }
            o[i] = (uint16_t)(u >> 16);
        }
        return k3d_upload(q->dst, o, (size_t)n * 2);
    }
    float *o = (float *)hb;
    for (int64_t i = 0; i < n; i++) {
        if (q->t.dtype == K3D_DT_F32) memcpy(&o[i], raw + 4 * i, 4);
        else {
            uint16_t h;
            memcpy(&h, raw + 2 * i, 2);
            if (q->t.dtype == K3D_DT_BF16) {
                const uint32_t u = (uint32_t)h << 16;
                memcpy(&o[i], &u, 4);
            } else {
                o[i] = half_to_f32(h);
            }
        }
    }
    return k3d_upload(q->dst, o, (size_t)n * 4);
}

typedef struct {
    int layer, e;
    K3dCkptTensor t[6];                      /* w1 packed, w1 scale, w3 packed, w3 scale, w2 packed, w2 scale */
} CkExpert;

int k3d_model_load_checkpoint(K3dModel *m, const K3dCkpt *ck)
{
    if (!m || !ck) return K3D_EINVAL;
    if (m->tp_kda || m->tp_mla || m->tp_dense) {
        k3h_ckpt_fail("checkpoint loading under tensor parallelism is not built (a rank holds head slices)");
        return K3D_EINVAL;
    }
    const K3dStackCfg *c = &m->c;
    const int64_t E = c->hidden, P = (int64_t)c->kda_heads * c->kda_head_dim, D = c->kda_head_dim;
    CkPlan p = {NULL, 0, 0, 0, ck};
    CkReq *q;
    q = ck_add(&p, CK_MAT, m->embed, (int64_t)c->vocab * E, CK_PRE "embed_tokens.weight");
    q = ck_add(&p, CK_VEC, m->final_norm, E, CK_PRE "norm.weight");
    q = ck_add(&p, CK_MAT, m->lm_head, (int64_t)c->vocab * E, "language_model.lm_head.weight");
    if (q) { q->row0 = m->v0; q->rows = m->vshard; q->cols = E; }
    CkExpert *ex = NULL;
    int nex = 0, capex = 0;
    for (int l = 0; l < c->n_layers; l++) {
        K3sLayer *L = &m->L[l];
        ck_add(&p, CK_VEC, L->in_norm, E, CK_PRE "layers.%d.input_layernorm.weight", l);
        ck_add(&p, CK_VEC, L->post_norm, E, CK_PRE "layers.%d.post_attention_layernorm.weight", l);
        if (L->is_mla) {
            const K3dMlaShape *s = &c->mla;
            const int64_t qh = s->qk_nope + s->qk_rope, kvw = s->kv_lora + s->qk_rope;
            ck_add(&p, CK_MAT, (void *)L->mla.q_a, (int64_t)s->q_lora * E, CK_PRE "layers.%d.self_attn.q_a_proj.weight", l);
            ck_add(&p, CK_VEC, (void *)L->mla.q_a_norm, s->q_lora, CK_PRE "layers.%d.self_attn.q_a_layernorm.weight", l);
            ck_add(&p, CK_MAT, (void *)L->mla.q_b, (int64_t)s->n_heads * qh * s->q_lora, CK_PRE "layers.%d.self_attn.q_b_proj.weight", l);
            ck_add(&p, CK_MAT, (void *)L->mla.kv_a, kvw * E, CK_PRE "layers.%d.self_attn.kv_a_proj_with_mqa.weight", l);
            ck_add(&p, CK_VEC, (void *)L->mla.kv_a_norm, s->kv_lora, CK_PRE "layers.%d.self_attn.kv_a_layernorm.weight", l);
            ck_add(&p, CK_MAT, (void *)L->mla.kv_b, (int64_t)s->n_heads * (s->qk_nope + s->v_head) * s->kv_lora,
                   CK_PRE "layers.%d.self_attn.kv_b_proj.weight", l);
            ck_add(&p, CK_MAT, (void *)L->mla.o, E * s->n_heads * s->v_head, CK_PRE "layers.%d.self_attn.o_proj.weight", l);
            if (s->out_gate)
                ck_add(&p, CK_MAT, (void *)L->mla.g, (int64_t)s->n_heads * s->v_head * E, CK_PRE "layers.%d.self_attn.g_proj.weight", l);
        } else {
            const char *mats[4] = {"q", "k", "v", "g"};
            const uint16_t *dm[4] = {L->kda.q, L->kda.k, L->kda.v, L->kda.g};
            for (int i = 0; i < 4; i++)
                ck_add(&p, CK_MAT, (void *)dm[i], P * E, CK_PRE "layers.%d.self_attn.%s_proj.weight", l, mats[i]);
            ck_add(&p, CK_MAT, (void *)L->kda.o, E * P, CK_PRE "layers.%d.self_attn.o_proj.weight", l);
            const char *cv[3] = {"q", "k", "v"};
            const float *dc[3] = {L->kda.q_conv, L->kda.k_conv, L->kda.v_conv};
            for (int i = 0; i < 3; i++)
                ck_add(&p, CK_VEC, (void *)dc[i], P * c->conv_k, CK_PRE "layers.%d.self_attn.%s_conv1d.weight", l, cv[i]);
            ck_add(&p, CK_MAT, (void *)L->kda.f_a, D * E, CK_PRE "layers.%d.self_attn.f_a_proj.weight", l);
            ck_add(&p, CK_MAT, (void *)L->kda.f_b, P * D, CK_PRE "layers.%d.self_attn.f_b_proj.weight", l);
            ck_add(&p, CK_MAT, (void *)L->kda.b, (int64_t)c->kda_heads * E, CK_PRE "layers.%d.self_attn.b_proj.weight", l);
            /* per head: the checkpoint ships head_dim values, the first kda_heads are the heads'
             * (k3_bind.c:218-222) */
            q = ck_add(&p, CK_VEC, (void *)L->kda.A_log, D, CK_PRE "layers.%d.self_attn.A_log", l);
            if (q) {
                q->take = c->kda_heads;
                if (q->take > q->want) { k3h_ckpt_fail("%s: fewer values than heads", q->name); p.bad++; }
            }
            ck_add(&p, CK_VEC, (void *)L->kda.dt_bias, P, CK_PRE "layers.%d.self_attn.dt_bias", l);
            ck_add(&p, CK_VEC, (void *)L->kda.o_norm, D, CK_PRE "layers.%d.self_attn.o_norm.weight", l);
        }
        if (L->is_dense) {
            ck_add(&p, CK_MAT, L->dg, (int64_t)c->dense_inter * E, CK_PRE "layers.%d.mlp.gate_proj.weight", l);
            ck_add(&p, CK_MAT, L->du, (int64_t)c->dense_inter * E, CK_PRE "layers.%d.mlp.up_proj.weight", l);
            ck_add(&p, CK_MAT, L->dd, E * c->dense_inter, CK_PRE "layers.%d.mlp.down_proj.weight", l);
            continue;
        }
        const K3dMoeShape *s = &c->moe;
        ck_add(&p, CK_ROUTER, (void *)L->moe.router_w, (int64_t)s->n_experts * E, CK_PRE "layers.%d.block_sparse_moe.gate.weight", l);
        ck_add(&p, CK_VEC, (void *)L->moe.router_bias, s->n_experts,
               CK_PRE "layers.%d.block_sparse_moe.gate.e_score_correction_bias", l);
        if (s->shared_inter > 0) {
            const int64_t SI = m->sh_full, SIl = s->shared_inter;
            const char *gu[2] = {"gate", "up"};
            const uint16_t *dg[2] = {L->moe.sh_gate, L->moe.sh_up};
            for (int i = 0; i < 2; i++) {
                q = ck_add(&p, CK_MAT, (void *)dg[i], SI * E, CK_PRE "layers.%d.block_sparse_moe.shared_experts.%s_proj.weight", l, gu[i]);
                if (q) { q->row0 = m->sh_lo; q->rows = SIl; q->cols = E; }
            }
            q = ck_add(&p, CK_SH_DOWN, (void *)L->moe.sh_down, E * SI, CK_PRE "layers.%d.block_sparse_moe.shared_experts.down_proj.weight", l);
            if (q) { q->row0 = m->sh_lo; q->rows = E; q->cols = SIl; q->take = SI; }
        }
        /* routed experts: the six U8 tensors, shapes from the configuration, one E8M0 scale
         * per 32 elements, one shard (k3_load.c:16-66) */
        for (int e = s->expert_lo; e < s->expert_hi && !p.bad; e++) {
            if (nex == capex) {
                capex = capex ? 2 * capex : 512;
                CkExpert *x2 = (CkExpert *)realloc(ex, (size_t)capex * sizeof(CkExpert));
                if (!x2) { p.bad++; break; }
                ex = x2;
            }
            CkExpert *x = &ex[nex];
            x->layer = l;
            x->e = e;
            const char *wn[3] = {"w1", "w3", "w2"};
            const int64_t rows[3] = {s->inter, s->inter, E}, in[3] = {E, E, s->inter};
            for (int i = 0; i < 3 && !p.bad; i++) {
                char nm[192];
                for (int k = 0; k < 2; k++) {
                    snprintf(nm, sizeof nm, CK_PRE "layers.%d.block_sparse_moe.experts.%d.%s.%s", l, e, wn[i],
                             k ? "weight_scale" : "weight_packed");
                    K3dCkptTensor *t = &x->t[2 * i + k];
                    if (k3d_ckpt_find(ck, nm, t)) { k3h_ckpt_fail("missing tensor %s", nm); p.bad++; break; }
                    const int64_t cols = k ? in[i] / 32 : in[i] / 2;
                    if (t->dtype != K3D_DT_U8 || t->ndim != 2 || t->shape[0] != rows[i] || t->shape[1] != cols) {
                        k3h_ckpt_fail("%s: expected U8 [%lld][%lld] (one scale per 32 elements)", nm,
                                      (long long)rows[i], (long long)cols);
                        p.bad++;
                        break;
                    }
                    if (t->shard != x->t[0].shard) {
                        k3h_ckpt_fail("layer %d expert %d spans shards", l, e);
                        p.bad++;
                        break;
                    }
                }
            }
            nex++;
        }
    }
    int r = p.bad ? K3D_EINVAL : K3D_OK;
    unsigned char *hb = r ? NULL : (unsigned char *)malloc(CK_HOST);
    if (!r && !hb) r = K3D_ENOMEM;
    for (int i = 0; i < p.n && !r; i++) r = ck_load_req(ck, &p.r[i], hb);
    /* experts: one read when the six tensors tile one run, else six; staged in the
     * checkpoint layout, then tiled where the model keeps tiled experts */
    size_t sz[6], off[6], per, toff[4];
    expert_layout(&c->moe, (int)E, sz, off, &per, toff);
    unsigned char *stage = (!r && nex) ? (unsigned char *)k3d_alloc(per) : NULL;
    unsigned char *hx = (!r && nex) ? (unsigned char *)malloc(per + 6 * 256) : NULL;
    if (!r && nex && (!stage || !hx)) r = K3D_ENOMEM;
    for (int i = 0; i < nex && !r; i++) {
        const CkExpert *x = &ex[i];
        const K3sLayer *L = &m->L[x->layer];
        const K3dMoeShape *s = &c->moe;
        int64_t lo = x->t[0].off, hi = 0, own = 0;
        for (int k = 0; k < 6; k++) {
            if (x->t[k].off < lo) lo = x->t[k].off;
            if (x->t[k].off + x->t[k].nbytes > hi) hi = x->t[k].off + x->t[k].nbytes;
            own += x->t[k].nbytes;
        }
        if (hi - lo == own && own <= (int64_t)per) {
            if (k3d_ckpt_read(ck, x->t[0].shard, lo, own, hx) != own) r = K3D_EINVAL;
            for (int k = 0; k < 6 && !r; k++)
                r = k3d_upload(stage + off[k], hx + (x->t[k].off - lo), (size_t)x->t[k].nbytes);
        } else {
            for (int k = 0; k < 6 && !r; k++) {
                if (k3d_ckpt_read(ck, x->t[k].shard, x->t[k].off, x->t[k].nbytes, hx) != x->t[k].nbytes) r = K3D_EINVAL;
                if (!r) r = k3d_upload(stage + off[k], hx, (size_t)x->t[k].nbytes);
            }
        }
        if (r) { if (r == K3D_EINVAL) k3h_ckpt_fail("short read of layer %d expert %d", x->layer, x->e); break; }
        unsigned char *base = L->pool + (size_t)(x->e - s->expert_lo) * per;
        if (s->expert_layout == 1) {
            K3ExpertQ src, dst;
            src.p1 = stage + off[0]; src.s1 = stage + off[1];
            src.p3 = stage + off[2]; src.s3 = stage + off[3];
            src.p2 = stage + off[4]; src.s2 = stage + off[5];
            dst.p1 = base + toff[0]; dst.s1 = base + toff[1];
            dst.p3 = NULL; dst.s3 = NULL;
            dst.p2 = base + toff[2]; dst.s2 = base + toff[3];
            r = k3d_expert_pretile(&dst, &src, (int)E, s->inter);
        } else {
            r = k3d_copy(base, stage, per);
        }
        if (!r) r = k3d_sync();
    }
    k3d_free(stage);
    free(hx);
    free(hb);
    free(ex);
    free(p.r);
    return r;
}
