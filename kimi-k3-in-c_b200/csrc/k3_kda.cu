// k3_kda.cu -- the KDA delta-rule state update on the device.
//
//   k3_kda_step     one head, reference API (k3_ops.c:186-243)
//   k3d_kda_decode  B sequences x H heads, one step each (config 3 decode)
//   k3d_kda_prefill T steps for all heads of one sequence (config 3 prefill)
//
// One thread owns one COLUMN j of the head's state S [dk][dv]. Every quantity the CPU
// computes per column is then a sequential loop over i inside one thread, in the CPU's
// order and with the CPU's roundings:
//     s_i   = S[i][j] * alpha[i]                      decay
//     u_j   = sum_i k_i * s_i      (skipping k_i == 0) read
//     S'_ij = s_i + (k_i * beta) * (v_j - u_j)        delta write (skip k_i == 0)
//     o_j   = sum_i q_i * S'_ij    (skipping q_i == 0) output from the updated state
// so the result is bit-identical to k3_kda_step. Explicit _rn intrinsics keep the
// compiler from contracting multiply-adds the CPU build (-ffp-contract=off) does not.
// A warp reads 32 consecutive columns of one row, so every state access is a fully
// coalesced 128-byte line; the column lives in registers between the read and the
// write, so the state crosses HBM exactly once in each direction per step.
#include "k3_common.cuh"
#include "k3_ops.cuh"

namespace k3 {

// Column j of one head's state, held in shared memory tile St [dk][dv] (row-major).
// Pass 1 decays and reads u; pass 2 writes the delta, reads o and stores to global.
__device__ __forceinline__ void kda_column(float *St, float *Sg, int dv, float *o,
                                           const float *q, const float *k, float vj,
                                           const float *alpha, float beta, int dk, int j)
{
    float u = 0.0f;
    for (int i = 0; i < dk; i++) {
        const float si = __fmul_rn(St[i * dv + j], alpha[i]);
        St[i * dv + j] = si;
        const float ki = k[i];
        if (ki != 0.0f) u = __fadd_rn(u, __fmul_rn(ki, si));
    }
    const float d = __fsub_rn(vj, u);
    float acc = 0.0f;
    for (int i = 0; i < dk; i++) {
        float si = St[i * dv + j];
        const float ki = k[i];
        if (ki != 0.0f) si = __fadd_rn(si, __fmul_rn(__fmul_rn(ki, beta), d));
        const float qi = q[i];
        if (qi != 0.0f) acc = __fadd_rn(acc, __fmul_rn(qi, si));
        if (Sg) Sg[(size_t)i * dv + j] = si;
        else St[i * dv + j] = si;
    }
    *o = acc;
}

// One CTA per (sequence, head): the whole [dk][dv] state tile is staged in shared memory
// with coalesced 16-byte loads, updated column-per-thread, and written back once.
// blockDim.x == dv (<= 1024). Shared: dk*dv state + 3*dk vectors.
__global__ void k_kda_decode(float *S, float *o, const float *q, const float *k, const float *v,
                             const float *alpha, const float *beta, int dk, int dv)
{
    extern __shared__ float sh[];
    const size_t bh = blockIdx.x;
    float *St = sh;
    float *qs = sh + (size_t)dk * dv, *ks = qs + dk, *as = ks + dk;
    float *Sh = S + bh * (size_t)dk * dv;
    const int n = dk * dv;
    if ((n & 3) == 0 && (((uintptr_t)Sh) & 15u) == 0) {
        const float4 *S4 = reinterpret_cast<const float4 *>(Sh);
        float4 *T4 = reinterpret_cast<float4 *>(St);
        #pragma unroll 8
        for (int f = threadIdx.x; f < n / 4; f += blockDim.x) T4[f] = S4[f];
    } else {
        #pragma unroll 8
        #pragma unroll 8
    for (int f = threadIdx.x; f < n; f += blockDim.x) St[f] = Sh[f];
    }
    for (int i = threadIdx.x; i < dk; i += blockDim.x) {
        qs[i] = q[bh * dk + i];
        ks[i] = k[bh * dk + i];
        as[i] = alpha[bh * dk + i];
    }
    __syncthreads();
    const int j = threadIdx.x;
    if (j < dv) kda_column(St, Sh, dv, o + bh * dv + j, qs, ks, v[bh * dv + j], as, beta[bh], dk, j);
}

// T sequential steps of one head per CTA; the state tile stays in shared memory across
// all steps (read from HBM once, written once).
__global__ void k_kda_seq(float *S, float *o, const float *q, const float *k, const float *v,
                          const float *alpha, const float *beta, int T, int H, int dk, int dv)
{
    extern __shared__ float sh[];
    const int h = blockIdx.x;
    float *St = sh;
    float *qs = sh + (size_t)dk * dv, *ks = qs + dk, *as = ks + dk;
    float *Sh = S + (size_t)h * dk * dv;
    const int n = dk * dv;
    for (int f = threadIdx.x; f < n; f += blockDim.x) St[f] = Sh[f];
    const int j = threadIdx.x;
    for (int t = 0; t < T; t++) {
        const size_t th = (size_t)t * H + h;
        __syncthreads();
        for (int i = threadIdx.x; i < dk; i += blockDim.x) {
            qs[i] = q[th * dk + i];
            ks[i] = k[th * dk + i];
            as[i] = alpha[th * dk + i];
        }
        __syncthreads();
        if (j < dv) kda_column(St, nullptr, dv, o + th * dv + j, qs, ks, v[th * dv + j], as,
                               beta[th], dk, j);
    }
    __syncthreads();
    for (int f = threadIdx.x; f < n; f += blockDim.x) Sh[f] = St[f];
}

static bool kda_fits(int dk, int dv)
{
    return dv >= 1 && dv <= 1024 && ((size_t)dk * dv + 3 * (size_t)dk) * 4 <= 200 * 1024;
}

static void kda_attrs()
{
    static bool init = false;
    if (!init) {
        allow_smem_max(k_kda_decode);
        allow_smem_max(k_kda_seq);
        init = true;
    }
}

int kda_decode(float *S, float *o, const float *q, const float *k, const float *v,
               const float *alpha, const float *beta, int B, int H, int dk, int dv,
               cudaStream_t st)
{
    if (B <= 0 || H <= 0 || dk <= 0 || dv <= 0) return K3D_OK;
    if (!kda_fits(dk, dv))
        return fail(K3D_EINVAL, "kda state %dx%d does not fit one CTA's shared memory", dk, dv);
    kda_attrs();
    const size_t smem = ((size_t)dk * dv + 3 * (size_t)dk) * sizeof(float);
    const int threads = ((dv + 31) / 32) * 32;
    k_kda_decode<<<B * H, threads, smem, st>>>(S, o, q, k, v, alpha, beta, dk, dv);
    note_launch();
    return check_launch("kda decode");
}

int kda_seq(float *S, float *o, const float *q, const float *k, const float *v,
            const float *alpha, const float *beta, int T, int H, int dk, int dv, cudaStream_t st)
{
    if (T <= 0 || H <= 0 || dk <= 0 || dv <= 0) return K3D_OK;
    if (!kda_fits(dk, dv))
        return fail(K3D_EINVAL, "kda state %dx%d does not fit one CTA's shared memory", dk, dv);
    kda_attrs();
    const size_t smem = ((size_t)dk * dv + 3 * (size_t)dk) * sizeof(float);
    const int threads = ((dv + 31) / 32) * 32;
    k_kda_seq<<<H, threads, smem, st>>>(S, o, q, k, v, alpha, beta, T, H, dk, dv);
    note_launch();
    return check_launch("kda seq");
}

}  // namespace k3

using namespace k3;

extern "C" {

void k3_kda_step(float *S, float *o, const float *q, const float *k, const float *v,
                 const float *alpha, float beta, int dk, int dv)
{
    if (ensure_ctx() || dk <= 0 || dv <= 0) return;
    Stage st;
    float *Sd = (float *)st.inout(S, (size_t)dk * dv * sizeof(float));
    const float *Q = (const float *)st.in(q, (size_t)dk * sizeof(float));
    const float *K = (const float *)st.in(k, (size_t)dk * sizeof(float));
    const float *V = (const float *)st.in(v, (size_t)dv * sizeof(float));
    const float *A = (const float *)st.in(alpha, (size_t)dk * sizeof(float));
    float *O = (float *)st.out(o, (size_t)dv * sizeof(float));
    float *Bd = (float *)scratch(sizeof(float), 3);
    if (st.err || !Bd) return;
    cudaMemcpyAsync(Bd, &beta, sizeof(float), cudaMemcpyHostToDevice, stream());
    if (kda_decode(Sd, O, Q, K, V, A, Bd, 1, 1, dk, dv, stream())) return;
    st.finish();
}

int k3d_kda_decode(float *S, float *o, const float *q, const float *k, const float *v,
                   const float *alpha, const float *beta, int B, int H, int dk, int dv)
{
    K3_TRY(ensure_ctx());
    if (!S || !o || !q || !k || !v || !alpha || !beta)
        return fail(K3D_EINVAL, "k3d_kda_decode null pointer");
    return kda_decode(S, o, q, k, v, alpha, beta, B, H, dk, dv, stream());
}

int k3d_kda_prefill(float *S, float *o, const float *q, const float *k, const float *v,
                    const float *alpha, const float *beta, int T, int H, int dk, int dv,
                    int chunk)
{
    K3_TRY(ensure_ctx());
    if (!S || !o || !q || !k || !v || !alpha || !beta)
        return fail(K3D_EINVAL, "k3d_kda_prefill null pointer");
    if (chunk != 0)
        return fail(K3D_EUNSUPPORTED, "k3d_kda_prefill: chunked form not built yet (chunk=%d)", chunk);
    return kda_seq(S, o, q, k, v, alpha, beta, T, H, dk, dv, stream());
}

}  // extern "C"
