// k3_stack_ops.cu -- the pieces of a decode step around the layers: embedding gather,
// dense SwiGLU MLP, LM head with the argmax fused into its epilogue, position advance.
#include "k3_common.cuh"
#include "k3_ops.cuh"

namespace k3 {

__global__ void k_embed(float *h, const int *ids, const uint16_t *table, int hidden, int vocab)
{
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    int id = ids[b];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) k3_raise(K3D_EBOUND, K3_SITE_STACK);
        id = 0;
    }
    const uint16_t *row = table + (size_t)id * hidden;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        h[(size_t)b * hidden + i] = bf16_to_f32(row[i]);
}

__global__ void k_add_f32(float *y, const float *x, size_t n)
{
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], x[i]);
}

__global__ void k_add_i32(int *p, int n, int delta)
{
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] += delta;
}

}  // namespace k3

using namespace k3;

extern "C" {

int k3d_embed_bf16(float *h, const int *ids, const uint16_t *table, int B, int hidden, int vocab)
{
    K3_TRY(ensure_ctx());
    if (!h || !ids || !table || B < 1 || hidden < 1) return fail(K3D_EINVAL, "k3d_embed_bf16");
    launch_pdl(k_embed, dim3((hidden + 1023) / 1024, B), dim3(256), 0, stream(), h, ids, table, hidden, vocab);
    note_launch();
    return check_launch("embed");
}

int k3d_swiglu_mlp_bf16(float *h, const float *x, const uint16_t *gate, const uint16_t *up,
                        const uint16_t *down, int hidden, int inter, int B, int accumulate,
                        float *ws)
{
    K3_TRY(ensure_ctx());
    if (!h || !x || !gate || !up || !down || !ws) return fail(K3D_EINVAL, "k3d_swiglu_mlp_bf16");
    prof_begin("dense.mlp");
    K3_TRY(gemv_bf16_swiglu(ws, x, gate, up, hidden, inter, B, stream()));
    K3_TRY(gemv_bf16(h, ws, down, inter, hidden, B, accumulate, stream()));
    prof_end("dense.mlp");
    return K3D_OK;
}

int k3d_lm_head_argmax(int *next, float *logits, const float *x, const uint16_t *W, int vocab,
                       int hidden, int B, void *key_ws)
{
    K3_TRY(ensure_ctx());
    if (!next || !x || !W || !key_ws) return fail(K3D_EINVAL, "k3d_lm_head_argmax");
    prof_begin("lm_head");
    const int r = gemv_bf16_argmax(logits, (unsigned long long *)key_ws, next, x, W, hidden, vocab, B,
                                   stream());
    prof_end("lm_head");
    return r;
}

int k3d_lm_head_argmax_normed(int *next, float *logits, const float *x, const float *norm_w,
                              float eps, const uint16_t *W, int vocab, int hidden, int B,
                              void *key_ws)
{
    K3_TRY(ensure_ctx());
    if (!next || !x || !norm_w || !W || !key_ws) return fail(K3D_EINVAL, "k3d_lm_head_argmax_normed");
    const NormIn ni{norm_w, eps};
    prof_begin("lm_head");
    const int r = gemv_bf16_argmax(logits, (unsigned long long *)key_ws, next, x, W, hidden, vocab, B,
                                   stream(), &ni);
    prof_end("lm_head");
    return r;
}

int k3d_lm_head_argmax_shard_normed(int *next, float *logits, const float *x, const float *norm_w,
                                    float eps, const uint16_t *W_shard, int v0, int vocab_shard,
                                    int hidden, int B, void *key_ws)
{
    K3_TRY(ensure_ctx());
    if (!next || !x || !norm_w || !W_shard || !key_ws || v0 < 0 || vocab_shard < 1 || B < 1)
        return fail(K3D_EINVAL, "k3d_lm_head_argmax_shard_normed");
    const NormIn ni{norm_w, eps};
    unsigned long long *key = (unsigned long long *)key_ws;
    cudaStream_t st = stream();
    prof_begin("lm_head");
    K3_TRY(lm_head_keys(logits, key, x, W_shard, hidden, vocab_shard, B, st, &ni));
    if (v0) K3_TRY(key_offset(key, B, v0, st));
    K3_TRY(ep_allreduce_max_u64(key, (size_t)B, st));
    const int r = argmax_finish(next, key, B, st);
    prof_end("lm_head");
    return r;
}

int k3d_add_f32(float *y, const float *x, size_t n)
{
    K3_TRY(ensure_ctx());
    if (!y || !x) return fail(K3D_EINVAL, "k3d_add_f32");
    if (!n) return K3D_OK;
    size_t g = (n + 255) / 256;
    if (g > (size_t)sm_count() * 8) g = (size_t)sm_count() * 8;
    launch_pdl(k_add_f32, dim3((int)g), dim3(256), 0, stream(), y, x, n);
    note_launch();
    return check_launch("add_f32");
}

int k3d_add_i32(int *p, int n, int delta)
{
    K3_TRY(ensure_ctx());
    if (!p || n < 1) return fail(K3D_EINVAL, "k3d_add_i32");
    launch_pdl(k_add_i32, dim3((n + 255) / 256), dim3(256), 0, stream(), p, n, delta);
    note_launch();
    return check_launch("add_i32");
}

}  // extern "C"
