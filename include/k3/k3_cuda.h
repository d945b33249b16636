/* SPDX-License-Identifier: Apache-2.0 */
/*
 * k3_cuda.h -- device context and B200-native decode entry points of libk3cuda.so.
 *
 * Two groups of symbols live here.
 *
 *  1. The device context (k3d_init ... k3d_graph_*). The CPU engine has no context
 *     object; its entry points in k3.h run on the context this header manages: one
 *     CUDA device, one stream, one sticky error status per process.
 *
 *  2. Decode-path operators at the shapes of the synthetic K3 benchmark, which the CPU
 *     engine's API cannot express: SwiGLU experts without the latent projection, a bf16
 *     shared expert, RoPE'd MLA over a bf16 latent cache with absorbed weights, batched
 *     KDA decode, the 8-layer decode stack and expert parallelism over NCCL. Each cites
 *     the CPU routine whose arithmetic it follows. These take DEVICE pointers only, are
 *     asynchronous on the library stream and can be captured into a CUDA graph.
 *
 * All functions return K3D_OK (0) or a K3D_E* code; the first non-zero code is also kept
 * in the sticky status read by k3d_status().
 */
#ifndef K3_CUDA_H
#define K3_CUDA_H

#include <stddef.h>
#include <stdint.h>
#include "k3.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ----------------------------------------------------------------- status ---- */
enum {
    K3D_OK = 0,
    K3D_ENODEV = 1,        /* no usable CUDA device */
    K3D_EINVAL = 2,        /* bad argument: null pointer, size, alignment, host pointer */
    K3D_ENOMEM = 3,        /* device allocation failed */
    K3D_ECUDA = 4,         /* a CUDA runtime call failed */
    K3D_EDEVICE = 5,       /* a kernel raised the device error flag */
    K3D_EUNSUPPORTED = 6,  /* outside this library's scope (e.g. K3_WI8) */
    K3D_ENCCL = 7,         /* an NCCL call failed */
    K3D_EBOUND = 8,        /* a capacity bound was exceeded (cache position, top-k) */
    K3D_ETIMEOUT = 9       /* a bounded device-side wait gave up */
};

/* Select the CUDA device and create the library stream. Idempotent for the same
 * device; the k3.h entry points call k3d_init(0) on first use if nobody did. One device
 * per process: once the context exists, k3d_init with another device returns K3D_EINVAL
 * (run one process per GPU, as the expert-parallel launch does). */
int         k3d_init(int device);
int         k3d_device(void);
/* The first error since the last k3d_clear_status(); also folds in the device error
 * flag as of the last k3d_sync(). */
int         k3d_status(void);
void        k3d_clear_status(void);
const char *k3d_strerror(int code);
const char *k3d_last_message(void);
/* 1: a recorded error prints and calls abort(), the CPU engine's fatal policy. */
void        k3d_set_abort_on_error(int on);
/* Device-side error detail: the code a kernel stored and the site id that stored it. */
int         k3d_device_error(int *code, int *site);
/* Limit of the pipelined kernels' bounded waits (mbarriers, cross-CTA counters), in SM
 * clock cycles; <= 0 restores the default 4e9 (about 2 s). A wait that runs out records
 * K3D_ETIMEOUT (read by k3d_sync / k3d_status); its kernel waits for the copies it
 * issued, frees its tensor memory and returns, so the context stays usable. */
int         k3d_set_wait_limit(long long cycles);

/* Memory. k3d_alloc returns 256-byte aligned device memory or NULL. */
void  *k3d_alloc(size_t bytes);
void   k3d_free(void *p);
int    k3d_upload(void *dst_dev, const void *src_host, size_t bytes);
int    k3d_download(void *dst_host, const void *src_dev, size_t bytes);
int    k3d_memset(void *dst_dev, int value, size_t bytes);
int    k3d_copy(void *dst_dev, const void *src_dev, size_t bytes);
/* rows x width bytes from src (rows spitch bytes apart) to dst (dpitch apart), device. */
int    k3d_copy2d(void *dst_dev, size_t dpitch, const void *src_dev, size_t spitch, size_t width,
                  size_t rows);
/* Page-locked host memory, for host<->device copies at full PCIe speed. */
void  *k3d_host_alloc(size_t bytes);
void   k3d_host_free(void *p);
/* Host weight residency for the k3.h entry points. Off (the default): a host weight is
 * copied to the device on every call, which is always correct. On: the first call that
 * sees a host weight address uploads it once and later calls reuse the HBM copy; the
 * caller promises not to rewrite those bytes (or to call k3d_forget) -- a ring buffer of
 * streamed layers, as the CPU engine's trunk reader keeps, must leave this off. */
void   k3d_set_weight_cache(int on);
/* Forget the HBM copy made for a host weight pointer passed to a k3.h entry point. */
void   k3d_forget(const void *host_ptr);
void   k3d_forget_all(void);
size_t k3d_weight_cache_bytes(void);

/* Stream, events, graphs. */
int    k3d_sync(void);
void  *k3d_stream(void);
int    k3d_set_stream(void *cuda_stream);
void  *k3d_event_create(void);
int    k3d_event_record(void *ev);
float  k3d_event_elapsed_ms(void *start, void *stop);
void   k3d_event_destroy(void *ev);
int    k3d_graph_begin(void);
void  *k3d_graph_end(void);
/* Whether graphs made by k3d_graph_end keep each captured kernel's stream priority
 * (default 1: the library's stream runs above the side stream's shared expert, which
 * helps batch-1 decode; the decode stack turns it off above four sequences, where it
 * measured 2% slower). No counterpart in the reference. */
int    k3d_set_graph_priorities(int on);
int    k3d_graph_launch(void *graph_exec);
void   k3d_graph_destroy(void *graph_exec);
/* Section timers. When enabled, the library records CUDA events on its stream around its
 * main kernel groups ("moe.experts", "moe.router", "moe.shared", "moe.combine", ...);
 * k3d_prof_ms() synchronises and returns the accumulated device time of one section and
 * the number of times it ran. Recording is skipped while a graph is being captured. */
void   k3d_prof_enable(int on);
void   k3d_prof_reset(void);
double k3d_prof_ms(const char *section, long *count);
/* Number of kernels this library launched since the last reset (host-side count). */
long   k3d_launch_count(void);
void   k3d_launch_count_reset(void);
int    k3d_sm_count(void);

/* -------------------------------------------------------- synthetic fill ---- */
/* Deterministic device-side fills for the synthetic benchmark inputs. The value of
 * element i depends only on (seed, i). Normal values are an Irwin-Hall sum of four
 * 16-bit uniforms scaled to the requested standard deviation. */
int k3d_fill_bf16_normal(uint16_t *dst, size_t n, uint64_t seed, float stddev);
/* Elements [offset, offset + n) of the sequence k3d_fill_bf16_normal writes for `seed`
 * (a slice of a larger seeded matrix, e.g. one rank's rows). */
int k3d_fill_bf16_normal_at(uint16_t *dst, size_t n, uint64_t seed, float sd, size_t offset);
int k3d_fill_f32_normal(float *dst, size_t n, uint64_t seed, float stddev);
int k3d_fill_f32_uniform(float *dst, size_t n, uint64_t seed, float lo, float hi);
/* Slices of the same seeded streams: elements [offset, offset + n) of the fill above. */
int k3d_fill_f32_normal_at(float *dst, size_t n, uint64_t seed, float sd, size_t offset);
int k3d_fill_f32_uniform_at(float *dst, size_t n, uint64_t seed, float lo, float hi, size_t offset);
/* E2M1 codes uniform over all 16 values; E8M0 bytes uniform in [s_lo, s_hi]. */
int k3d_fill_mxfp4(unsigned char *packed, size_t packed_bytes,
                   unsigned char *scales, size_t scale_bytes,
                   uint64_t seed, int s_lo, int s_hi);
int k3d_fill_i32_uniform(int *dst, size_t n, uint64_t seed, int lo, int hi);

/* ------------------------------------------------------------------ MXFP4 ---- */
/* Config 0: y = W_down . (silu(W_gate . x) * (W_up . x)), one MXFP4 expert. x [hidden],
 * y [hidden], fp32. Follows k3_moe's per-expert body (k3_ops.c:628-631) with SiLU in
 * place of SiTU. `e` is a HOST struct holding device pointers. ws: k3d_expert_ws_bytes. */
size_t k3d_expert_ws_bytes(int hidden, int inter);
int    k3d_expert_swiglu(float *y, const float *x, const K3ExpertQ *e,
                         int hidden, int inter, void *ws, size_t ws_bytes);

/* ------------------------------------------------------------------- MoE ---- */
/* One MoE layer without the latent projection: router (k3_router semantics, bf16 W),
 * routed MXFP4 SwiGLU experts combined in top-k order, plus an optional unweighted
 * bf16 SwiGLU shared expert. Follows k3_moe / moe_prefill_chunk
 * (k3_ops.c:556-656, 717-825) with SwiGLU and no latent step. */
typedef struct {
    int   hidden;          /* 7168 */
    int   inter;           /* routed expert intermediate, 2048 */
    int   n_experts;       /* 384 */
    int   topk;            /* 8, at most K3_MAX_TOPK */
    int   renorm;          /* 1 */
    float routed_scale;    /* 2.5 */
    int   shared_inter;    /* 2048; 0 = no shared expert */
    int   expert_lo;       /* experts [expert_lo, expert_hi) are computed here */
    int   expert_hi;
    int   add_shared;      /* 1: this rank adds the shared expert (one rank under EP) */
    int   expert_layout;   /* 0: checkpoint layout (p1,s1,p3,s3,p2,s2 as in the model
                            *    files); 1: tiled (k3d_expert_pretile), tcgen05 kernel only */
} K3dMoeShape;

typedef struct {
    const uint16_t  *router_w;      /* [n_experts][hidden] bf16 */
    const float     *router_bias;   /* [n_experts] */
    const K3ExpertQ *experts;       /* DEVICE array [n_experts] */
    const uint16_t  *sh_gate;       /* [shared_inter][hidden] bf16 */
    const uint16_t  *sh_up;         /* [shared_inter][hidden] bf16 */
    const uint16_t  *sh_down;       /* [hidden][shared_inter] bf16 */
} K3dMoeW;

size_t k3d_moe_ws_bytes(const K3dMoeShape *s, int T);
/* out[T][hidden] (+)= moe(x[T][hidden]). accumulate = 1 adds into out (residual).
 * idx/wts (device, [T][topk]) receive the routing; either may be NULL. */
int    k3d_moe_swiglu(float *out, const float *x, const K3dMoeW *w, const K3dMoeShape *s,
                      int T, int accumulate, int *idx, float *wts,
                      void *ws, size_t ws_bytes);
/* Rewrites one expert into the tiled layout: the stage-ordered image of the tcgen05
 * kernel's shared-memory tiles, so each pipeline stage is a few large bulk copies.
 * dst->p1 / dst->s1 receive gate and up together (2*inter*hidden/2 and 2*inter*hidden/32
 * bytes), dst->p2 / dst->s2 the down matrix (same sizes as src->p2 / src->s2); dst->p3
 * and dst->s3 are unused. E8M0 255 becomes 0 (the CPU engine reads 255 as zero). hidden
 * and inter must be multiples of 512. Device pointers; asynchronous on the library
 * stream. Use with K3dMoeShape.expert_layout = 1. */
int    k3d_expert_pretile(const K3ExpertQ *dst, const K3ExpertQ *src, int hidden, int inter);
/* Which MXFP4 expert kernel k3d_expert_swiglu / k3d_moe_swiglu run: 0 (default) the
 * tcgen05 block-scaled tensor-core kernel whenever the shapes allow it (hidden and inter
 * multiples of 512, T * topk <= 64), 1 the mma.sync kernel, 2 the CUDA-core kernels, 3 the
 * tcgen05 kernel with the activation operand in every pipeline stage (kind 0, for tiled
 * experts, keeps it resident across the stages that share it up to 64 assignments, and
 * lets up to four tokens routed to one expert share its weight stages above 64), 4 as 0
 * but decode-sized MoE work lists (up to 16 assignments at config 1) run as ONE launch that
 * does gate/up, the act split and down (bit-identical; measured slower than the three
 * launches of kind 0 so far, so not the default).
 * Experts in the tiled layout always run on the tcgen05 kernel.
 * All give the same results within the expert tolerance; the switch exists to measure
 * and test each. */
int    k3d_set_expert_kernel(int kind);
/* The router alone on a bf16 W: idx/w [T][topk], device. */
int    k3d_router_bf16(int *idx, float *w, const float *x, const uint16_t *W,
                       const float *bias, int T, int hidden, int n_experts, int topk,
                       int renorm, float routed_scale);
/* k3d_router_bf16 without device allocation. No reference counterpart: the CPU engine
 * never allocates device memory. k3d_router_bf16 takes its score buffer from the
 * library workspace, which grows with cudaMalloc (a device-wide synchronisation) the
 * first time a larger T * n_experts arrives. This variant instead uses one fixed
 * scratch array compiled into the library (3 * K3D_ROUTER_NOALLOC_MAX floats, 384 KB),
 * for callers that must not allocate once running: a serving loop whose device memory
 * is fixed at start-up, or a host whose allocator owns all device memory.
 *   - T * n_experts above K3D_ROUTER_NOALLOC_MAX returns K3D_EBOUND and launches nothing.
 *   - The first call on a device does set-up (it looks up the scratch array's address);
 *     make that first call before any stream capture.
 *   - The scratch array is shared: calls that overlap (other threads, other streams)
 *     race on it. Serialise them.
 * Results are bit-identical to k3d_router_bf16. */
#define K3D_ROUTER_NOALLOC_MAX 32768
int    k3d_router_bf16_noalloc(int *idx, float *w, const float *x, const uint16_t *W,
                               const float *bias, int T, int hidden, int n_experts,
                               int topk, int renorm, float routed_scale);
/* Experts (summed over all router calls in this process) whose fp32 logit could not be
 * settled from the exact dot product and its error bound, and were recomputed with the
 * CPU engine's sequential double loop. Diagnostic; results are bit-exact either way. */
long long k3d_router_fallbacks(void);
/* Number of distinct experts routed to by the last eagerly launched k3d_moe_swiglu call
 * (synchronises the stream; -1 before the first call). Used for the bytes numerator. */
int    k3d_moe_last_unique(void);

/* --------------------------------------------------------------- GEMV ---- */
/* y[T][out] = x[T][in] . W^T for bf16 W; accumulate = 1 adds into y. */
int k3d_gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out, int T,
                  int accumulate);

/* ------------------------------------------------------------------- KDA ---- */
/* Batched KDA decode step: per (sequence b, head h) exactly k3_kda_step
 * (k3_ops.c:186-243) on S[b][h] ([dk][dv] fp32, updated in place). q, k, alpha
 * [B][H][dk], v and o [B][H][dv], beta [B][H]; q arrives pre-scaled as in k3.h. */
int k3d_kda_decode(float *S, float *o, const float *q, const float *k, const float *v,
                   const float *alpha, const float *beta, int B, int H, int dk, int dv);
/* T-step recurrence for one sequence, all heads: the same result as T sequential
 * k3d_kda_decode calls. q,k,alpha [T][H][dk]; v,o [T][H][dv]; beta [T][H].
 * chunk = 0 runs the sequential recurrence, bit-identical to k3_kda_step.
 * chunk = 64 runs the chunked (WY) form: the same recurrence regrouped into 64-step
 * chunks, equal to the sequential result within fp32 rounding (decays in [0, 1]; a decay
 * of 0 acts as 2^-126). It needs dk a multiple of 8 up to 128, dv a multiple of 32 up to
 * 128, and 16-byte aligned S, o, q, k and alpha; its per-chunk records use library scratch
 * (about 148 KB per (chunk, head) at dk = dv = 128, for at most 8 chunks at a time).
 * Other chunk values return K3D_EINVAL. */
int k3d_kda_prefill(float *S, float *o, const float *q, const float *k, const float *v,
                    const float *alpha, const float *beta, int T, int H, int dk, int dv,
                    int chunk);

/* Full KDA decode layer (one token per sequence) at bf16 weights: k3_kda_layer
 * (k3_ops.c:850-937) at T = 1. h (+)= o_proj(...) of the normed input xn; state is the
 * CPU engine's per-sequence layout (H*D*D recurrent floats, then 3*H*D*(conv_k-1) conv
 * history floats), k3d_kda_state_floats() per sequence, updated in place. */
typedef struct {
    int   hidden, heads, head_dim, conv_k;
    float gate_lb, eps;
} K3dKdaShape;

typedef struct {
    const uint16_t *q, *k, *v, *g;     /* [H*D][hidden] */
    const uint16_t *b;                 /* [H][hidden] */
    const uint16_t *f_a;               /* [D][hidden] */
    const uint16_t *f_b;               /* [H*D][D] */
    const uint16_t *o;                 /* [hidden][H*D] */
    const float *q_conv, *k_conv, *v_conv;   /* [H*D][conv_k] */
    const float *A_log;                /* [H] */
    const float *dt_bias;              /* [H*D] */
    const float *o_norm;               /* [D] */
} K3dKdaW;

size_t k3d_kda_layer_ws_bytes(const K3dKdaShape *s, int B);
size_t k3d_kda_state_floats(const K3dKdaShape *s);
int    k3d_kda_layer_decode(float *h, const float *xn, const K3dKdaW *w, const K3dKdaShape *s,
                            int B, float *state, void *ws, size_t ws_bytes);
/* The same layer taking the raw residual h as its input: it applies the layer's input
 * RMSNorm (weights norm_w [hidden], eps; k3_rmsnorm's arithmetic, k3_ops.c:94-102) itself,
 * inside the projection GEMV's load where that kernel runs, saving the separate norm
 * launch and its output buffer. No reference counterpart (the CPU engine norms first). */
int    k3d_kda_layer_decode_normed(float *h, const float *norm_w, float eps, const K3dKdaW *w,
                                   const K3dKdaShape *s, int B, float *state, void *ws,
                                   size_t ws_bytes);
/* The same, with the layer's output written (accumulate = 0) or added (1) to out instead
 * of the residual h it reads: a tensor-parallel rank's partial (its heads' share of the
 * output projection), summed over the ranks afterwards. */
int    k3d_kda_layer_decode_normed_out(float *out, const float *h, const float *norm_w, float eps,
                                       const K3dKdaW *w, const K3dKdaShape *s, int B, float *state,
                                       void *ws, size_t ws_bytes, int accumulate);
/* Which kernel runs the per-head step of the decode layer: 0 (default) chooses 2 for up to
 * four sequences and 1 above; 1 stages the head's state tile in shared memory, one CTA per
 * head; 2 keeps each thread's state column in registers, one CTA per head; 3 splits each
 * head's value columns over a cluster of head_dim / 32 one-warp CTAs (registers, the head
 * norm's sum through distributed shared memory). 2 and 3 apply where head_dim is 32, 64 or
 * 128 and conv_k is 4 (else 1 runs). Bit-identical; the switch exists to measure and test
 * each. No reference counterpart. */
int    k3d_set_kda_head_kernel(int kind);

/* ------------------------------------------------------------------- MLA ---- */
typedef struct {
    int   hidden, n_heads, q_lora, kv_lora, qk_nope, qk_rope, v_head;
    float rope_theta;      /* 50000; 0 disables the rotation (NoPE) */
    float eps;
    int   out_gate;        /* 1: sigmoid(g x) gates the heads before o_proj */
} K3dMlaShape;

typedef struct {
    const uint16_t *q_a;       /* [q_lora][hidden] */
    const uint16_t *q_b;       /* [H*(nope+rope)][q_lora] */
    const uint16_t *kv_a;      /* [kv_lora+rope][hidden] */
    const uint16_t *kv_b;      /* [H*(nope+v)][kv_lora] */
    const uint16_t *o;         /* [hidden][H*v] */
    const uint16_t *g;         /* [H*v][hidden], NULL when out_gate == 0 */
    const float    *q_a_norm;  /* [q_lora] */
    const float    *kv_a_norm; /* [kv_lora] */
} K3dMlaW;

size_t k3d_mla_ws_bytes(const K3dMlaShape *s, int B, int cap);
/* One decode token per sequence. cache [B][cap][kv_lora+rope] bf16 holds the normalised
 * latent and the rotated rope key of every earlier position; *pos (device int) is the
 * number of cached positions, the new token is written at index *pos and attends over
 * *pos + 1 positions. Follows k3_mla_cached (k3_ops.c:321-410) in absorbed form. */
int k3d_mla_decode(float *out, const float *x, const K3dMlaW *w, const K3dMlaShape *s,
                   int B, uint16_t *cache, int cap, const int *pos, int accumulate,
                   void *ws, size_t ws_bytes);
/* k3d_mla_decode with x the raw residual, RMS-normalised by the layer itself (norm_w
 * [hidden], eps), as k3d_kda_layer_decode_normed. No reference counterpart. */
int k3d_mla_decode_normed(float *out, const float *x, const float *norm_w, float eps,
                          const K3dMlaW *w, const K3dMlaShape *s, int B, uint16_t *cache,
                          int cap, const int *pos, int accumulate, void *ws, size_t ws_bytes);

/* ------------------------------------------------------------- small ops ---- */
int k3d_rmsnorm(float *y, const float *x, const float *w, int n, int rows, float eps);
int k3d_silu_mul(float *y, const float *gu, int n, int rows); /* gu = [gate | up] per row */
/* h[b] = bf16 table row ids[b], widened (the CPU's k3_embed_row, k3_bind.h:148-157) */
int k3d_embed_bf16(float *h, const int *ids, const uint16_t *table, int B, int hidden, int vocab);
/* dense SwiGLU MLP: h[b] (+)= down(silu(gate x) * (up x)), bf16 weights; ws holds
 * B*inter floats */
int k3d_swiglu_mlp_bf16(float *h, const float *x, const uint16_t *gate, const uint16_t *up,
                        const uint16_t *down, int hidden, int inter, int B, int accumulate,
                        float *ws);
/* logits = W x (bf16 W [vocab][hidden]) and next[b] = first index of the maximum logit
 * (argmax_ of k3_run.c:134-135); logits may be NULL; key_ws holds B 8-byte keys. */
int k3d_lm_head_argmax(int *next, float *logits, const float *x, const uint16_t *W, int vocab,
                       int hidden, int B, void *key_ws);
/* The LM head on the raw residual, with the final RMSNorm (norm_w, eps) applied on load.
 * No reference counterpart. */
int k3d_lm_head_argmax_normed(int *next, float *logits, const float *x, const float *norm_w,
                              float eps, const uint16_t *W, int vocab, int hidden, int B,
                              void *key_ws);
/* The LM head over one slice of the vocabulary (rows [v0, v0 + vocab_shard) in W_shard),
 * for expert-parallel decode where each rank holds a slice: the ranks' packed (logit,
 * index) maxima are combined with an all-reduce max over NCCL (k3d_ep_init; on one rank
 * none is needed), so next[B] is the argmax over the whole vocabulary, first maximum on
 * ties, as k3d_lm_head_argmax_normed gives it. logits (optional) receives this slice's
 * [B][vocab_shard] logits. No reference counterpart (the CPU engine is single-process). */
int k3d_lm_head_argmax_shard_normed(int *next, float *logits, const float *x, const float *norm_w,
                                    float eps, const uint16_t *W_shard, int v0, int vocab_shard,
                                    int hidden, int B, void *key_ws);
/* y[i] += x[i] for i < n (device floats) */
int k3d_add_f32(float *y, const float *x, size_t n);
/* Row-wise conversions between bf16 (rows with a pitch, in elements) and packed fp32,
 * round to nearest even towards bf16, and a transpose of a rows x cols matrix of 16-bit
 * values (dst is cols x rows). Device pointers. No reference counterpart. */
int k3d_bf16_rows_to_f32(float *dst, const uint16_t *src, size_t spitch, int rows, int cols);
int k3d_f32_rows_to_bf16(uint16_t *dst, size_t dpitch, const float *src, int rows, int cols);
int k3d_transpose_u16(uint16_t *dst, const uint16_t *src, int rows, int cols);
/* p[i] += delta for i < n (device ints; advances cache positions inside a graph) */
int k3d_add_i32(int *p, int n, int delta);

/* --------------------------------------------------------------- EP/NCCL ---- */
/* Expert parallelism over NCCL: one process per GPU. rank 0 calls
 * k3d_ep_unique_id, ships the 128 bytes to the other ranks, and every rank calls
 * k3d_ep_init. */
int k3d_ep_unique_id(unsigned char id[128]);
int k3d_ep_init(int rank, int nranks, const unsigned char id[128]);
int k3d_ep_finalize(void);
int k3d_ep_rank(void);
int k3d_ep_size(void);
/* In-place sum of a float buffer over all ranks (NCCL). */
int k3d_ep_allreduce_f32(float *buf, size_t n);
/* The MoE combine of expert parallelism over NVLink peer memory: every rank exports one
 * receive buffer (CUDA IPC) and maps every other rank's; collective, call on every rank
 * after k3d_ep_init with the largest vector the combine will carry (floats). */
int k3d_ep_peer_init(size_t max_floats);
/* h[i] (+)= sum over ranks of partial[i] (accumulate = 1 adds into h), the same on every
 * rank: one kernel stores this rank's partial into every rank's buffer, publishes it with
 * a release flag per destination, waits (bounded; K3D_ETIMEOUT) for every rank's flag and
 * sums the partials in rank order. Device pointers, 16-byte aligned; asynchronous on the
 * library stream and capturable in a CUDA graph. Without k3d_ep_peer_init (or for vectors
 * longer than it was sized for) it runs ncclAllReduce and an add instead. */
int k3d_ep_combine_add(float *h, const float *partial, size_t n, int accumulate);
/* The push combine's protocol: 0 (default) every element as one 8-byte word carrying its
 * own call tag (no fence, no flag round trip), 1 the data, a system fence and a release
 * flag per slice. Same bits; every rank must choose the same. */
int k3d_set_ep_combine(int kind);

/* Mode A expert parallelism: all-to-all dispatch and combine for data-parallel tokens (a
 * batch split over the ranks, e.g. B = 64). Every rank passes ITS OWN tokens x[T][hidden]
 * (T may differ between ranks; at most t_max on every rank) and holds the experts
 * [expert_lo, expert_hi) = [rank * E / nranks, (rank + 1) * E / nranks) in w->experts
 * (entries indexed by global expert id). Each rank routes its tokens; the fp32 row of each
 * (token, slot) goes to the rank of its expert with grouped NCCL send/recv, is run through
 * that rank's experts and comes back the same way; the tokens' rank sums the rows in top-k
 * order, adds the shared expert (s->add_shared: set it on every rank) and writes
 * out[T][hidden] (+= with accumulate). Routing and the receive counts decide the transfer
 * sizes, so the call synchronises the host twice and cannot be captured into a graph.
 * nranks = k3d_ep_size() (1 without k3d_ep_init: all experts local, same result).
 * No reference counterpart: the CPU engine is single-process. */
size_t k3d_moe_a2a_ws_bytes(const K3dMoeShape *s, int t_max, int nranks);
int    k3d_moe_swiglu_a2a(float *out, const float *x, const K3dMoeW *w, const K3dMoeShape *s,
                          int T, int t_max, int accumulate, int *idx, float *wts,
                          void *ws, size_t ws_bytes);
/* Mode A planned on the device, for graph capture: the same rows, experts and top-k
 * combine (bit-identical results), but every rank passes the same T (its own tokens),
 * the dispatch plan is computed by a kernel, and each exchange moves fixed regions of
 * T * topk rows per pair of ranks (grouped NCCL send/recv of fixed sizes), so nothing is
 * read back to the host. More NVLink traffic than k3d_moe_swiglu_a2a (the full region
 * whatever the routing); the workspace is k3d_moe_a2a_ws_bytes(s, T, nranks). */
int    k3d_moe_swiglu_a2a_dev(float *out, const float *x, const K3dMoeW *w, const K3dMoeShape *s,
                              int T, int accumulate, int *idx, float *wts, void *ws, size_t ws_bytes);
/* The Mode A dispatch plan, on HOST arrays (no device work): for assignments idx[TK]
 * (expert ids), cnt[r] rows go to rank r (expert e on rank e / (n_experts / nranks)),
 * rank r's rows start at row off[r] of the send buffer, each rank's rows in assignment
 * order, and pos[a] is the row of assignment a. n_experts must be a multiple of nranks. */
int    k3d_a2a_plan(const int *idx, int TK, int n_experts, int nranks, int *cnt, int *off,
                    int *pos);

/* ----------------------------------------------------------- decode stack ---- */
typedef struct {
    int   hidden, vocab, n_layers;
    float eps;
    /* KDA */
    int   kda_heads, kda_head_dim, conv_k;
    float gate_lb;
    /* MLA */
    K3dMlaShape mla;
    /* MoE: shape of layers >= first_dense */
    K3dMoeShape moe;
    int   first_dense, dense_inter;
    /* zero-based MLA layers, -1 terminated list */
    int   mla_layers[16];
    /* batch (1..64: up to 4 tokens stream the weights through GEMVs, more run the
     * tensor-core GEMM) and cache */
    int   batch;
    int   ctx_cap;
    /* Under expert parallelism: 0 (Mode R) every rank steps the same batch (attention and
     * router replicated, the MoE partials summed by the NVLink push combine, the shared
     * expert and the LM head split over the ranks); 1 (Mode A) every rank steps its OWN
     * batch of `batch` sequences (rank r holds the global sequences [r batch, (r + 1)
     * batch)) with the whole shared expert and LM head, and each MoE layer exchanges rows
     * with k3d_moe_swiglu_a2a_dev, so the step stays one CUDA graph. Every rank passes the
     * same batch. Ignored on one rank except that Mode A's MoE path is taken. */
    int   ep_tokens;
} K3dStackCfg;

typedef struct K3dModel K3dModel;

/* Random-init weights on the device (synthetic benchmark), MLA cache and KDA state
 * allocated for cfg->batch sequences of up to ctx_cap positions. Under EP each rank
 * allocates only its own experts. */
K3dModel *k3d_model_create(const K3dStackCfg *cfg, uint64_t seed);
void      k3d_model_destroy(K3dModel *m);
/* Fill the MLA latent caches and KDA states as after `len` tokens of context with
 * seeded synthetic values (latent ~N(0,1), state ~N(0,0.01), conv history ~N(0,1)). */
int       k3d_model_fill_context(K3dModel *m, int len, uint64_t seed);
/* One decode step for the batch: ids (device [B]) in, next ids (device [B], argmax of
 * the logits) out, logits (device [B][vocab]) optional. Captures into a graph. Under EP
 * (k3d_ep_init with more than one rank) each rank holds a slice of the LM head and logits
 * receives that slice, [B][rows of the slice]; next is the argmax over all of them.
 * A step writes the next cache position: with the caches full (ctx_cap positions since
 * the last fill or state load) it returns K3D_EBOUND and launches nothing. */
int       k3d_model_step_dev(K3dModel *m, const int *ids, int *next_ids, float *logits);
/* The same through host buffers: copies ids in, runs the step, copies next ids out. */
int       k3d_model_step_host(K3dModel *m, const int *ids_host, int *next_host);
/* Use a CUDA graph for k3d_model_step_* (default 1). */
int       k3d_model_use_graph(K3dModel *m, int on);
/* Device pointers to model internals for tests: name = "embed", "lm_head",
 * "final_norm", "pos", "layer<i>.<tensor>". Returns NULL if unknown. */
void     *k3d_model_tensor(K3dModel *m, const char *name, size_t *bytes);
/* Algorithmic bytes the last step read or wrote in HBM (weights + caches + states). */
double    k3d_model_last_step_bytes(K3dModel *m);

/* Conversation state in the CPU engine's file format (K3ST version 1, k3_run.c:158-300,
 * which has no library interface: k3_state_peek/k3_state_save/k3_state_load are static
 * in the CLI): the configuration fingerprint, the token ids, one KDA state slot per layer,
 * the MLA caches as expanded keys and values (kv_b times the latent, fp32) and rope slots,
 * only the occupied positions. The CPU engine can resume from a file saved here and the
 * reverse. After the CPU engine's payload a save appends the device's own bf16 cache rows
 * ("K3LT"), which the CPU engine does not read; a load with that trailer restores the
 * caches bit for bit, one without it recovers each latent from the expanded keys and
 * values by least squares (within bf16 rounding of the original).
 *   peek: the header only, so the caller can size seq before loading; has_latent says
 *         whether the trailer is there.
 *   save: sequence b of the batch at the model's current position; seq (nseq ids, host)
 *         are the tokens the caller keeps for it.
 *   load: into sequence b; refuses (K3D_EINVAL) a file whose fingerprint, layer counts
 *         or per-layer sizes differ from this model, K3D_EBOUND when it holds more
 *         positions than ctx_cap or more ids than seq_cap. Sets the model's position to
 *         the file's (the position is shared by the batch). seq may be NULL. A load that
 *         fails part-way leaves the caches partly written. */
typedef struct {
    int version, n_bound, n_mla, cached, nseq, has_latent;
} K3dStateInfo;
int       k3d_state_peek(const char *path, K3dStateInfo *info);
int       k3d_model_state_save(K3dModel *m, const char *path, const int *seq, int nseq, int b);
int       k3d_model_state_load(K3dModel *m, const char *path, int *seq, int seq_cap, int b);

/* Released-checkpoint loading (the device counterpart of src/io/k3_st.c, the names and
 * element-count checks of src/model/k3_bind.c:167-241 and the expert checks of
 * src/io/k3_load.c:46-103). k3d_ckpt_open indexes every *.safetensors file of dir (shards
 * in file-name order) and validates every header entry (known dtype, span = elements x
 * element size, inside the file); lookups are O(1). Host only: none of the k3d_ckpt_*
 * calls touches the GPU. k3d_ckpt_error gives the reason of the last failure. */
typedef struct K3dCkpt K3dCkpt;
enum { K3D_DT_U8 = 1, K3D_DT_BF16 = 2, K3D_DT_F16 = 3, K3D_DT_F32 = 4 };
typedef struct {
    int     shard, dtype, ndim;
    int64_t shape[4];
    int64_t off, nbytes;          /* absolute byte offset within the shard file, size */
} K3dCkptTensor;
K3dCkpt    *k3d_ckpt_open(const char *dir);
void        k3d_ckpt_close(K3dCkpt *ck);
int         k3d_ckpt_count(const K3dCkpt *ck);
int         k3d_ckpt_find(const K3dCkpt *ck, const char *name, K3dCkptTensor *out);  /* K3D_EINVAL if absent */
int64_t     k3d_ckpt_read(const K3dCkpt *ck, int shard, int64_t off, int64_t nbytes, void *buf);
int         k3d_ckpt_elem_size(int dtype);
const char *k3d_ckpt_error(void);
/* Binds the checkpoint's tensors (the released names: language_model.model.layers.L.
 * self_attn.*, block_sparse_moe.gate / experts.E.w{1,2,3}.weight_{packed,scale} /
 * shared_experts.*, mlp.* for dense layers, embed_tokens, norm, language_model.lm_head)
 * to the model's weights and uploads them, replacing the random initialisation. Every
 * tensor is checked before a byte is read: present, the expected element count for the
 * model's configuration, bf16 for matrices (fp32 / bf16 / f16 for vectors, widened),
 * U8 MXFP4 experts with one E8M0 scale per 32 elements and all six tensors in one shard.
 * An expert whose six tensors form one contiguous run is read with one read. Under expert
 * parallelism only this rank's experts, LM-head rows and shared-expert slice are read.
 * Returns K3D_EINVAL (reason in k3d_ckpt_error) without uploading anything when a check
 * fails. Caches and states are left as they are. */
int         k3d_model_load_checkpoint(K3dModel *m, const K3dCkpt *ck);

#ifdef __cplusplus
}
#endif

#endif /* K3_CUDA_H */
