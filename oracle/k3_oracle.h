/* k3_oracle.h -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A CPU restatement of the CPU engine's decode-path arithmetic (libxsmm/kimi-k3-in-c,
 * src/core/k3_ops.c), used only as the checker by tests/, __graft_entry__.smoke() and
 * the cpu_baseline leg of bench.py. Nothing in libk3cuda links or calls it.
 *
 * Each function names the reference lines it follows. Where the reference fixes a
 * summation order the restatement keeps it (the scalar, non-AVX2 paths), so its results
 * can be compared against the compiled reference (oracle/_ref) to ~1e-15 and against
 * the reference's golden fixtures at their manifest tolerance.
 *
 * The orc_*_swiglu / orc_moe_swiglu / orc_mla_absorbed / orc_stack functions compose
 * the reference routines for the benchmark shapes, which the reference API does not
 * cover: SiLU in place of SiTU, no latent projection, RoPE, a bf16 latent cache.
 */
#ifndef K3_ORACLE_H
#define K3_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "k3.h"

#ifdef __cplusplus
extern "C" {
#endif

float orc_bf16f(uint16_t h);
uint16_t orc_f2bf(float f);

/* reference operators (k3_ops.c line ranges in the .c file) */
int   orc_is_mla(const K3Cfg *c, int layer);
void  orc_rmsnorm(float *y, const float *x, const float *w, int n, float eps);
void  orc_situ_glu(float *y, const float *x, int n, float b1, float b2);
void  orc_shortconv(float *y, const float *x, const float *w, float *state,
                    int channels, int k, int T);
void  orc_kda_decay(float *g, float *alpha, const float *z, const float *A_log,
                    const float *dt_bias, int H, int D, float lb);
void  orc_kda_step(float *S, float *o, const float *q, const float *k, const float *v,
                   const float *alpha, float beta, int dk, int dv);
void  orc_matmul(float *y, const float *x, const float *W, int in, int out);
void  orc_matmul_bf16(float *y, const float *x, const uint16_t *W, int in, int out);
void  orc_mmw(float *y, const float *x, const void *W, int wdt, int in, int out);
void  orc_router(int *idx, float *w, const float *x, const float *W, const float *bias,
                 int hidden, int n_experts, int topk, int renorm, float routed_scale);
/* the same with a bf16 gate matrix, widened exactly */
void  orc_router_bf16(int *idx, float *w, const float *x, const uint16_t *W,
                      const float *bias, int hidden, int n_experts, int topk, int renorm,
                      float routed_scale);
void  orc_attn_res(float *out, const float *src, const float *fold, int nsrc, int n,
                   float eps);
size_t orc_mla_scratch_cached(const K3Cfg *c, int T, int cap, int cached_mode);
void  orc_mla_cached(float *out, const float *x, const K3MlaW *w, const K3Cfg *c, int T,
                     float *scratch, float *kvc, float *ropec, int cached, int cap);
size_t orc_moe_scratch(const K3Cfg *c);
/* experts: NULL for the resident fp32 bank (w->w1/w3/w2), or a host array of
 * n_experts packed MXFP4 experts (what the reference reads through K3ExpertSrc) */
void  orc_moe(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T,
              int *idx, float *wt, float *scratch, const K3ExpertQ *experts);
size_t orc_kda_scratch(const K3Cfg *c, int T);
void  orc_kda_layer(float *out, const float *x, const K3KdaW *w, const K3Cfg *c, int T,
                    float *state, float *scratch);
size_t orc_layer_scratch(const K3Cfg *c, int T);
void  orc_decoder_layer_inc(float *h, float *block_residual, int *n_blocks,
                            const K3LayerW *w, const K3Cfg *c, int layer_idx, int T,
                            float *state, float *scratch, float *kvc, float *ropec,
                            int cached, int cap, const K3ExpertQ *experts);
void  orc_mxfp4_dequant(float *out, const unsigned char *packed,
                        const unsigned char *scales, int rows, int pcols, int group);
void  orc_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                       const unsigned char *scales, int in, int rows, int group);

/* ---- compositions at the benchmark shapes ---- */
float orc_silu(float g);
/* config 0: y = down(silu(gate x) * (up x)), MXFP4 */
void  orc_expert_swiglu(float *y, const float *x, const K3ExpertQ *e, int hidden, int inter);
/* config 1: one token at a time (T tokens), bf16 router W and shared expert */
void  orc_moe_swiglu(float *out, const float *x, int T, int hidden, int inter,
                     int n_experts, int topk, int renorm, float routed_scale,
                     const uint16_t *router_w, const float *router_bias,
                     const K3ExpertQ *experts, int shared_inter, const uint16_t *sh_gate,
                     const uint16_t *sh_up, const uint16_t *sh_down,
                     int expert_lo, int expert_hi, int add_shared, int *idx_out,
                     float *w_out);
/* RoPE on interleaved pairs, frequency theta^(-2i/d) */
void  orc_rope(float *x, int d, int pos, float theta);
/* config 2: MLA decode over a bf16 latent cache, expanded form (see the .c file) */
void  orc_set_mla_new_entry_fp32(int on);
void  orc_mla_decode(float *out, const float *x, int B, int hidden, int H, int q_lora,
                     int kv_lora, int qn, int qr, int vh, float theta, float eps,
                     const uint16_t *q_a, const uint16_t *q_b, const uint16_t *kv_a,
                     const uint16_t *kv_b, const uint16_t *o, const uint16_t *g,
                     const float *q_a_norm, const float *kv_a_norm, uint16_t *cache, int cap,
                     int pos);
void  orc_mla_decode_absorbed(float *out, const float *x, int B, int hidden, int H, int q_lora,
                     int kv_lora, int qn, int qr, int vh, float theta, float eps,
                     const uint16_t *q_a, const uint16_t *q_b, const uint16_t *kv_a,
                     const uint16_t *kv_b, const uint16_t *o, const uint16_t *g,
                     const float *q_a_norm, const float *kv_a_norm, uint16_t *cache, int cap,
                     int pos);
/* config 3: B*H heads of k3_kda_step */
void  orc_kda_decode(float *S, float *o, const float *q, const float *k, const float *v,
                     const float *alpha, const float *beta, int B, int H, int dk, int dv);

#ifdef __cplusplus
}
#endif

#endif
