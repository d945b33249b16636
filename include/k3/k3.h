/* SPDX-License-Identifier: Apache-2.0 */
/*
 * k3.h -- the Kimi K3 decode operator API, served by sm_100a kernels.
 *
 * This header declares the same C operator surface as the CPU engine's
 * include/k3/k3.h (libxsmm/kimi-k3-in-c), so code written against that header links
 * against libk3cuda.so unchanged. Every struct below has the same members in the same
 * order, and every prototype has the same name, argument order and argument meaning.
 * The interface has to be alike for the library to be a drop-in; the bodies are new.
 *
 * WHERE THE WORK RUNS
 *   Every function that computes runs on the GPU selected with k3d_init() (k3_cuda.h),
 *   or on device 0 if the caller never chose one. There is no CPU fallback: without a
 *   usable CUDA device each call records K3D_ENODEV in the sticky status, prints one
 *   line to stderr and leaves its outputs untouched.
 *
 * POINTERS
 *   Each pointer argument may be either
 *     - a device pointer (k3d_alloc, cudaMalloc, cudaMallocManaged), used in place. The
 *       call is then asynchronous on the library stream; k3d_sync() waits for it.
 *     - an ordinary host pointer. Host arguments are staged through the library
 *       stream and the call returns only after host outputs are written, which is the
 *       synchronous behaviour of the CPU engine. Host WEIGHT matrices are copied on each
 *       call unless the caller enables k3d_set_weight_cache(1), after which each weight
 *       address is uploaded to HBM once and reused.
 *
 * ERRORS
 *   The CPU engine aborts on an allocation failure or an exceeded bound. These entry
 *   points keep their void signatures and instead record the first error in a sticky
 *   status (k3d_status()). k3d_set_abort_on_error(1) restores the abort policy.
 *
 * Reference interface: include/k3/k3.h:68-570 of libxsmm/kimi-k3-in-c.
 */
#ifndef K3_H
#define K3_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ config ---- */
/* Model shape. Same members, order and meaning as the CPU engine's K3Cfg
 * (include/k3/k3.h:73-120). */
typedef struct {
    int hidden;
    int n_layers;
    int vocab;
    float rms_eps;

    /* Kimi Delta Attention */
    int kda_heads;
    int kda_head_dim;          /* d_k == d_v */
    int conv_k;                /* depthwise causal conv taps, SiLU fused */
    float gate_lb;             /* decay lower bound */

    /* gated MLA */
    int n_heads;
    int q_lora;
    int kv_lora;
    int qk_nope;
    int qk_rope;               /* present in the head width; rotated only by k3d_* RoPE paths */
    int v_head;
    int mla_out_gate;

    /* latent MoE */
    int n_experts;
    int topk;
    int n_shared;
    int latent;
    int moe_inter;
    float routed_scale;
    int moe_renorm;
    int latent_norm;

    /* dense layers */
    int first_dense;
    int dense_inter;

    /* block attention residuals */
    int attn_res_block;

    /* SiTU-GLU caps */
    float situ_b1;
    float situ_b2;

    /* one-based indices of the MLA layers */
    int  n_full_attn;
    int *full_attn;
} K3Cfg;

/* Layer map; `layer` is zero-based, full_attn one-based. (k3.h:122-124) */
int  k3_is_mla(const K3Cfg *c, int layer);
int  k3_is_kda(const K3Cfg *c, int layer);
int  k3_is_dense(const K3Cfg *c, int layer);

/* --------------------------------------------------------------------- ops ---- */

/* y = w * x / sqrt(mean(x^2) + eps), per row of n. (k3.h:130) */
void k3_rmsnorm(float *y, const float *x, const float *w, int n, float eps);

/* SiTU-GLU over [gate | up] of 2n: y = b1*tanh(g/b1)*sigmoid(g) * b2*tanh(u/b2).
 * (k3.h:137) */
void k3_situ_glu(float *y, const float *x, int n, float b1, float b2);

/* Causal depthwise conv with fused SiLU; state holds k-1 past inputs per channel and
 * is updated in place; NULL state means zero history. (k3.h:144) */
void k3_shortconv(float *y, const float *x, const float *w, float *state,
                  int channels, int k, int T);

/* g = lb*sigmoid(exp(A_log[h])*(z + dt_bias)), alpha = exp(g). A_log is per head.
 * (k3.h:154) */
void k3_kda_decay(float *g, float *alpha, const float *z, const float *A_log,
                  const float *dt_bias, int H, int D, float lb);

/* One delta-rule step for one head, S [d_k][d_v]: decay rows by alpha, u = S^T k,
 * S += k (beta (v - u))^T, o = S^T q from the updated state. (k3.h:164) */
void k3_kda_step(float *S, float *o, const float *q, const float *k,
                 const float *v, const float *alpha, float beta, int dk, int dv);

/* y[out] = W[out][in] . x[in], fp32 row-major W. (k3.h:168) */
void k3_matmul(float *y, const float *x, const float *W, int in, int out);

/* Gated MLA weights, tagged by wdt (0 fp32, 1 bf16). (k3.h:202-209) */
typedef struct {
    const void  *q_a, *q_b;
    const void  *kv_a, *kv_b;
    const void  *o, *g;
    const float *q_a_norm, *kv_a_norm;
    int          wdt;
} K3MlaW;

size_t k3_mla_scratch(const K3Cfg *c, int T);                                /* k3.h:211 */
size_t k3_mla_scratch_cached(const K3Cfg *c, int T, int cap, int cached_mode); /* k3.h:213 */

/* Gated MLA over an optional expanded fp32 KV cache kvc [cap][H*(nope+v)] and a shared
 * rope slot cache ropec [cap][rope]; NULL caches recompute from x. (k3.h:218-222) */
void   k3_mla_cached(float *out, const float *x, const K3MlaW *w, const K3Cfg *c,
                     int T, float *scratch,
                     float *kvc, float *ropec, int cached, int cap);
void   k3_mla(float *out, const float *x, const K3MlaW *w, const K3Cfg *c,
              int T, float *scratch);

/* Router for one token: sigmoid scores, bias steers selection only, weights from the
 * unbiased scores, optional renorm, times routed_scale. Indices and weights come out
 * bit-identical to the CPU engine. (k3.h:241) */
void k3_router(int *idx, float *w, const float *x, const float *W,
               const float *bias, int hidden, int n_experts, int topk,
               int renorm, float routed_scale);

/* AttnRes: softmax over RMSNormed sources scored against fold, applied to the raw
 * sources. (k3.h:250) */
void k3_attn_res(float *out, const float *src, const float *fold,
                 int nsrc, int n, float eps);

/* Weight tags. (k3.h:270) */
enum { K3_WF32 = 0, K3_WBF16 = 1, K3_WI8 = 2 };

/* bf16 is the top half of an fp32. (k3.h:274-279) */
static inline float k3_bf16f(uint16_t h)
{
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)h << 16;
    return v.f;
}

/* y[out] = W[out][in] . x[in], W bf16. Same values as k3_matmul on the widened W. */
void k3_matmul_bf16(float *y, const float *x, const uint16_t *W, int in, int out);

/* Per-row int8 draft-model matmul (k3.h:285). The draft model is outside this
 * library's scope: the symbol exists so that code built against the CPU header links,
 * and every call records K3D_EUNSUPPORTED. */
void k3_matmul_q8(float *y, const float *x, const void *W, int in, int out);

/* Tagged-pointer dispatch, inline exactly as in the CPU header (k3.h:289-295). */
static inline void k3_mmw(float *y, const float *x, const void *W, int wdt,
                          int in, int out)
{
    if (wdt == K3_WBF16)     k3_matmul_bf16(y, x, (const uint16_t *)W, in, out);
    else if (wdt == K3_WI8)  k3_matmul_q8(y, x, W, in, out);
    else                     k3_matmul(y, x, (const float *)W, in, out);
}

static inline size_t k3_wsz(int wdt) { return wdt == K3_WBF16 ? 2u : 4u; }
static inline size_t k3_row_bytes(int wdt, int in)
{
    return wdt == K3_WI8 ? (size_t)4 + (size_t)in : (size_t)in * k3_wsz(wdt);
}

/* One routed expert in packed MXFP4: codes and E8M0 scales of gate (1), up (3) and
 * down (2). (k3.h:323-327) */
typedef struct {
    const unsigned char *p1, *s1;
    const unsigned char *p3, *s3;
    const unsigned char *p2, *s2;
} K3ExpertQ;

/* Expert source vtable. (k3.h:332-355) */
typedef struct K3ExpertSrc {
    int (*get)(struct K3ExpertSrc *self, int layer, int expert, K3ExpertQ *out);
    int (*getmany)(struct K3ExpertSrc *self, int layer, const int *experts, int n);
    int (*resident)(struct K3ExpertSrc *self, int layer, int expert, K3ExpertQ *out);
    void *ctx;
} K3ExpertSrc;

/* Latent MoE weights. (k3.h:357-380) */
typedef struct {
    const float *gate, *bias;
    const float *w1, *w3, *w2;
    const float *latent_norm;
    const void  *down, *up;
    const void  *sh1, *sh3, *sh2;
    int          wdt;
    struct K3ExpertSrc *src;
    int          layer;
    int          cache_only;
} K3MoeW;

size_t k3_moe_scratch(const K3Cfg *c);                                        /* k3.h:382 */

/* Count of routed experts that could not be fetched; non-zero means corrupt output.
 * (k3.h:388) */
extern long k3_expert_drops;

#define K3_MAX_PROMPT 32768
#define K3_MAX_GEN     4096
#define K3_KV_BYTES_PER_POS 2370000.0

/* Latent MoE for T tokens, per token. idx/wt receive the last token's routing.
 * (k3.h:418) */
void   k3_moe(float *out, const float *x, const K3MoeW *w, const K3Cfg *c,
              int T, int *idx, float *wt, float *scratch);
/* Batched form: each selected expert is read once for the whole batch, with per-token
 * results identical to k3_moe. (k3.h:425) */
void   k3_moe_prefill(float *out, const float *x, const K3MoeW *w, const K3Cfg *c,
                      int T, int *idx, float *wt, float *scratch);

/* KDA layer weights. (k3.h:447-461) */
typedef struct {
    const void  *q, *k, *v;
    const float *q_conv, *k_conv, *v_conv;
    const void  *f_a, *f_b;
    const float *A_log;
    const float *dt_bias;
    const void  *b;
    const void  *g;
    const float *o_norm;
    const void  *o;
    int          wdt;
} K3KdaW;

size_t k3_kda_scratch(const K3Cfg *c, int T);                                 /* k3.h:463 */
/* state: H*D*D recurrent floats then 3*H*D*(conv_k-1) conv floats, updated in place;
 * NULL means a fresh sequence. (k3.h:467) */
void   k3_kda_layer(float *out, const float *x, const K3KdaW *w, const K3Cfg *c,
                    int T, float *state, float *scratch);

/* Decoder layer weights. attn_res_* may be NULL in k3d_* stacks (plain pre-norm
 * residual); the k3_decoder_layer* entry points require them as the CPU engine does.
 * (k3.h:497-506) */
typedef struct {
    const float *in_norm, *post_norm;
    const float *attn_res_norm, *attn_res_proj;
    const float *mlp_res_norm,  *mlp_res_proj;
    const K3KdaW *kda;
    const K3MlaW *mla;
    const K3MoeW *moe;
    const void  *dense_gate, *dense_up, *dense_down;
    int          wdt;
} K3LayerW;

size_t k3_layer_scratch(const K3Cfg *c, int T);                               /* k3.h:508 */
void   k3_decoder_layer(float *h, float *block_residual, int *n_blocks,
                        const K3LayerW *w, const K3Cfg *c, int layer_idx,
                        int T, float *state, float *scratch);                 /* k3.h:509 */
void   k3_decoder_layer_inc(float *h, float *block_residual, int *n_blocks,
                            const K3LayerW *w, const K3Cfg *c, int layer_idx,
                            int T, float *state, float *scratch,
                            float *kvc, float *ropec, int cached, int cap);   /* k3.h:517 */

/* -------------------------------------------------------------------- MXFP4 ---- */
/* OCP MX FP4: two E2M1 codes per byte (low nibble = even element), one E8M0 exponent
 * byte per group; value = E2M1[code] * 2^(scale-127); scale byte 255 (NaN) reads as 0.
 * (k3.h:548-566) */
#define K3_MXFP4_GROUP 32
#define K3_MAX_TOPK 64

void k3_mxfp4_dequant(float *out, const unsigned char *packed,
                      const unsigned char *scales, int rows, int pcols, int group);

void k3_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                     const unsigned char *scales, int in, int rows, int group);

#ifdef __cplusplus
}
#endif

#endif /* K3_H */
