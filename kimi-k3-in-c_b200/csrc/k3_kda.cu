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
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) {
        allow_smem_max(k_kda_decode);
        allow_smem_max(k_kda_seq);
        init |= dev_bit();
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

// ------------------------------------------------------------- chunked prefill ----
// The T-step recurrence in chunks of C = 64 steps (the WY / UT form of the delta rule).
// Within a chunk that starts from state S0, with a_t the running product of the decays up
// to and including step t (G_t = log2 a_t, per key channel i):
//     L_ts = sum_i k_t[i] k_s[i] 2^(G_t[i]-G_s[i])   (s < t)
//     M_ts = sum_i q_t[i] k_s[i] 2^(G_t[i]-G_s[i])   (s <= t)
//     (I + diag(beta) L) X = diag(beta) (V - Kt S0),  Kt_t = 2^G_t * k_t
//     X = U - W S0 with U, W the forward substitutions of beta*V and beta*Kt
//     O = Qt S0 + M X,                                  Qt_t = 2^G_t * q_t
//     S_C = diag(2^G_last) S0 + Kb^T X,                 Kb_s = 2^(G_last-G_s) * k_s
// which is the sequential step of k3_kda_step (k3_ops.c:186-243) unrolled over the chunk:
// X_t = beta_t (v_t - u_t) is the delta row step t writes. The result matches the
// sequential recurrence within floating-point rounding, not bit for bit.
//
// k_kda_chunk_prep, one CTA per (chunk, head), all chunks of a segment in parallel:
// computes W, U, Qt, Kb, M and 2^G_last into a per-(chunk, head) record. Every exponent
// 2^(G_t-G_s) has t >= s, so it is <= 1 for decays in [0, 1]. When every |G| of the chunk
// is at most 60 (no overflow of 2^-G), L and M are plain products of 2^G*k and 2^-G*k;
// otherwise (strong decay) each pair takes its own exponential. log2 of a decay is clamped
// at -126, so a decay of exactly 0 acts as 2^-126. Exponentials and logarithms are the
// hardware approximations (ex2.approx, lg2.approx).
// k_kda_chunk_scan, one CTA per (head, 64 value columns; 32 when dv is not a multiple of
// 64): walks the chunks in order with the state block in shared memory; per chunk
// X = U - W S, O = Qt S + M X, S = g S + Kb^T X, each product on the tensor cores
// (mma.sync tf32, fp32 operands split in two, 3 MMAs per step). Operands are copied in
// with cp.async two phases ahead of their use, through three rotating buffers.
namespace kdc {

constexpr int C = 64;            // steps per chunk
constexpr int DKM = 128;         // largest key dim
constexpr int LDT = C + 4;       // row stride of the transposed [dk][C] tiles
constexpr int THREADS = 256;
constexpr int SEG = 8;           // chunks per prep/scan pair (records stay in L2)

struct Rec {
    size_t wt, qt, kb, mt, u, gc, total;
};

__host__ __device__ __forceinline__ Rec rec(int dk, int dv)
{
    Rec r;
    r.wt = 0;                                   // W^T [dk][C]
    r.qt = (size_t)dk * C;                      // Qt^T [dk][C]
    r.kb = r.qt + (size_t)dk * C;               // Kb [C][dk]
    r.mt = r.kb + (size_t)C * dk;               // M^T [C][C] (M^T[s][t], zero for s > t)
    r.u = r.mt + (size_t)C * C;                 // U [C][dv]
    r.gc = r.u + (size_t)C * dv;                // 2^G_last [dk]
    r.total = r.gc + (size_t)((dk + 3) & ~3);
    return r;
}

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float at4(const float4 &v, int a)
{
    return a == 0 ? v.x : a == 1 ? v.y : a == 2 ? v.z : v.w;
}

// The hardware base-2 exponential and logarithm (ex2.approx / lg2.approx, about 2^-22
// relative error; subnormal results flush to zero). The chunked form's decays enter only
// through 2^(difference of cumulative log2 decays), so errors of this size stay far below
// the 1e-3 tolerance of the chunked result.
__device__ __forceinline__ float ex2a(float x)
{
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float lg2a(float x)
{
    float r;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

constexpr size_t prep_smem() { return (3 * (size_t)DKM * LDT + C) * sizeof(float); }

__device__ __forceinline__ float4 ldg4(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }
__device__ __forceinline__ void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }

__global__ void __launch_bounds__(THREADS, 2)
k_kda_chunk_prep(const float *__restrict__ q, const float *__restrict__ k,
                 const float *__restrict__ v, const float *__restrict__ alpha,
                 const float *__restrict__ beta, float *__restrict__ ws, long tok0, int T, int H,
                 int dk, int dv)
{
    extern __shared__ __align__(16) float sh[];
    float *kT = sh;                          // k, then 2^G k                      [dk][LDT]
    float *qT = kT + DKM * LDT;              // q, then 2^G q on the product path
    float *gT = qT + DKM * LDT;              // decay, then G, then 2^-G k, then L [C][C]
    float *bs = gT + DKM * LDT;              // beta [C]
    const int c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const long tc0 = tok0 + (long)c * C;
    const int cn = (int)min((long)C, (long)T - tc0);
    const Rec R = rec(dk, dv);
    float *out = ws + ((size_t)c * H + h) * R.total;

    // k, q and the decay, transposed to [i][t]: a warp pass covers 16 steps x 8 channels
    // (two float4 per step), which lands on 32 distinct banks. All loads of a half are
    // issued before its stores. Padded steps (t >= cn) are identities: k = q = 0, decay 1.
    {
        const int tl = lane & 15, ih = (lane >> 4) * 4;
        const int nb = dk / 2;               // (16-step group, 8-channel group) pairs
#pragma unroll
        for (int half = 0; half < 2; half++) {
            float4 kr[4], qr[4], ar[4];
#pragma unroll
            for (int n = 0; n < 4; n++) {
                const int b = warp + 8 * (4 * half + n);
                const int t = (b & 3) * 16 + tl, i = (b >> 2) * 8 + ih;
                kr[n] = qr[n] = make_float4(0.f, 0.f, 0.f, 0.f);
                ar[n] = make_float4(1.f, 1.f, 1.f, 1.f);
                if (b < nb && t < cn) {
                    const size_t g = ((size_t)(tc0 + t) * H + h) * dk + i;
                    kr[n] = ldg4(k + g);
                    qr[n] = ldg4(q + g);
                    ar[n] = ldg4(alpha + g);
                }
            }
#pragma unroll
            for (int n = 0; n < 4; n++) {
                const int b = warp + 8 * (4 * half + n);
                if (b < nb) {
                    const int t = (b & 3) * 16 + tl, i = (b >> 2) * 8 + ih;
#pragma unroll
                    for (int a = 0; a < 4; a++) {
                        kT[(i + a) * LDT + t] = at4(kr[n], a);
                        qT[(i + a) * LDT + t] = at4(qr[n], a);
                        gT[(i + a) * LDT + t] = at4(ar[n], a);
                    }
                }
            }
        }
    }
    if (tid < C) bs[tid] = tid < cn ? beta[(size_t)(tc0 + tid) * H + h] : 0.0f;
    __syncthreads();

    // Cumulative log2 decay per channel (float4 along t: conflict-free).
    bool big = false;
    if (tid < dk) {
        float g = 0.0f;
        float *row = gT + tid * LDT;
#pragma unroll 4
        for (int t = 0; t < C; t += 4) {
            float4 a = ld4(row + t);
            g += fmaxf(lg2a(a.x), -126.0f); a.x = g;
            g += fmaxf(lg2a(a.y), -126.0f); a.y = g;
            g += fmaxf(lg2a(a.z), -126.0f); a.z = g;
            g += fmaxf(lg2a(a.w), -126.0f); a.w = g;
            st4(row + t, a);
            big |= !(fabsf(a.x) <= 60.0f && fabsf(a.w) <= 60.0f && fabsf(a.y) <= 60.0f &&
                     fabsf(a.z) <= 60.0f);
        }
        out[R.gc + tid] = ex2a(g);
    }
    const bool direct = __syncthreads_or(big);

    // Kb [s][i] = 2^(G_last - G_s) k_s and Qt^T [i][t] = 2^G_t q_t, read as float4 along t.
    for (int e = tid; e < dk * (C / 4); e += THREADS) {
        const int i = e % dk, s = (e / dk) * 4;
        const float gl = gT[i * LDT + C - 1];
        const float4 kk = ld4(kT + i * LDT + s), gg = ld4(gT + i * LDT + s);
        float *o = out + R.kb + (size_t)s * dk + i;
        o[0] = kk.x * ex2a(gl - gg.x);
        o[dk] = kk.y * ex2a(gl - gg.y);
        o[2 * dk] = kk.z * ex2a(gl - gg.z);
        o[3 * dk] = kk.w * ex2a(gl - gg.w);
    }
    for (int e = tid; e < dk * (C / 4); e += THREADS) {
        const int i = e / (C / 4), t = (e % (C / 4)) * 4;
        const float4 qq = ld4(qT + i * LDT + t), gg = ld4(gT + i * LDT + t);
        st4(out + R.qt + (size_t)i * C + t,
            make_float4(qq.x * ex2a(gg.x), qq.y * ex2a(gg.y), qq.z * ex2a(gg.z), qq.w * ex2a(gg.w)));
    }
    if (!direct) {
        __syncthreads();
        for (int e = tid; e < dk * (C / 4); e += THREADS) {
            const int i = e / (C / 4), t = (e % (C / 4)) * 4;
            const float4 k0 = ld4(kT + i * LDT + t), gg = ld4(gT + i * LDT + t);
            float4 qq = ld4(qT + i * LDT + t), kk, n;
            float p;
            p = ex2a(gg.x); kk.x = k0.x * p; qq.x *= p; n.x = k0.x * ex2a(-gg.x);
            p = ex2a(gg.y); kk.y = k0.y * p; qq.y *= p; n.y = k0.y * ex2a(-gg.y);
            p = ex2a(gg.z); kk.z = k0.z * p; qq.z *= p; n.z = k0.z * ex2a(-gg.z);
            p = ex2a(gg.w); kk.w = k0.w * p; qq.w *= p; n.w = k0.w * ex2a(-gg.w);
            st4(kT + i * LDT + t, kk);
            st4(qT + i * LDT + t, qq);
            st4(gT + i * LDT + t, n);
        }
    }
    __syncthreads();

    // L and M over the 136 lower-triangular 4x4 tiles, one per thread of the first 136:
    // thread (bt, bsb) owns t = 4bt.., s = 4bsb.. with bsb <= bt.
    float La[4][4], Ma[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) La[a][b] = Ma[a][b] = 0.0f;
    int bt = 0;
    while ((bt + 1) * (bt + 2) / 2 <= tid) bt++;
    const int bsb = tid - bt * (bt + 1) / 2;
    const bool tile = tid < (C / 4) * (C / 4 + 1) / 2;
    if (tile) {
        if (!direct) {
#pragma unroll 2
            for (int i = 0; i < dk; i++) {
                const float4 kt = ld4(kT + i * LDT + 4 * bt), qt = ld4(qT + i * LDT + 4 * bt);
                const float4 ns = ld4(gT + i * LDT + 4 * bsb);
                const float2 n01 = make_float2(ns.x, ns.y), n23 = make_float2(ns.z, ns.w);
#pragma unroll
                for (int a = 0; a < 4; a++) {
                    const float2 ka = make_float2(at4(kt, a), at4(kt, a));
                    const float2 qa = make_float2(at4(qt, a), at4(qt, a));
                    float2 l01 = ffma2(ka, n01, make_float2(La[a][0], La[a][1]));
                    float2 l23 = ffma2(ka, n23, make_float2(La[a][2], La[a][3]));
                    float2 m01 = ffma2(qa, n01, make_float2(Ma[a][0], Ma[a][1]));
                    float2 m23 = ffma2(qa, n23, make_float2(Ma[a][2], Ma[a][3]));
                    La[a][0] = l01.x; La[a][1] = l01.y; La[a][2] = l23.x; La[a][3] = l23.y;
                    Ma[a][0] = m01.x; Ma[a][1] = m01.y; Ma[a][2] = m23.x; Ma[a][3] = m23.y;
                }
            }
        } else {
            for (int i = 0; i < dk; i++) {
                const float4 gt = ld4(gT + i * LDT + 4 * bt), gs = ld4(gT + i * LDT + 4 * bsb);
                const float4 kt = ld4(kT + i * LDT + 4 * bt), ks = ld4(kT + i * LDT + 4 * bsb);
                const float4 qt = ld4(qT + i * LDT + 4 * bt);
#pragma unroll
                for (int a = 0; a < 4; a++)
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        if (bsb < bt || b <= a) {
                            const float kse = at4(ks, b) * ex2a(at4(gt, a) - at4(gs, b));
                            La[a][b] = fmaf(at4(kt, a), kse, La[a][b]);
                            Ma[a][b] = fmaf(at4(qt, a), kse, Ma[a][b]);
                        }
                    }
            }
        }
        // M^T [s][t], zero above the diagonal inside the diagonal tile.
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int s = 4 * bsb + b;
            float4 r;
            r.x = 4 * bt + 0 >= s ? Ma[0][b] : 0.0f;
            r.y = 4 * bt + 1 >= s ? Ma[1][b] : 0.0f;
            r.z = 4 * bt + 2 >= s ? Ma[2][b] : 0.0f;
            r.w = 4 * bt + 3 >= s ? Ma[3][b] : 0.0f;
            st4(out + R.mt + (size_t)s * C + 4 * bt, r);
        }
    } else {
        // the 120 tiles above the diagonal, one per remaining thread: zeros, since the
        // scan's 16-row MMA tiles read M^T[s][t] for s up to the end of t's 16-row block
        int j = tid - (C / 4) * (C / 4 + 1) / 2, ut = 0;
        while (j >= C / 4 - 1 - ut) { j -= C / 4 - 1 - ut; ut++; }
        const int us = ut + 1 + j;
#pragma unroll
        for (int b = 0; b < 4; b++)
            st4(out + R.mt + (size_t)(4 * us + b) * C + 4 * ut, make_float4(0.f, 0.f, 0.f, 0.f));
    }
    __syncthreads();
    if (direct) {
        for (int e = tid; e < dk * (C / 4); e += THREADS) {
            const int i = e / (C / 4), t = (e % (C / 4)) * 4;
            float4 kk = ld4(kT + i * LDT + t);
            const float4 gg = ld4(gT + i * LDT + t);
            kk.x *= ex2a(gg.x); kk.y *= ex2a(gg.y); kk.z *= ex2a(gg.z); kk.w *= ex2a(gg.w);
            st4(kT + i * LDT + t, kk);
        }
        __syncthreads();
    }
    // -L (strictly lower; the substitution reads nothing else) into the G region.
    float *Ls = gT;
    if (tile) {
#pragma unroll
        for (int a = 0; a < 4; a++) {
            const int t = 4 * bt + a;
            float4 r;
            r.x = t > 4 * bsb + 0 ? -La[a][0] : 0.0f;
            r.y = t > 4 * bsb + 1 ? -La[a][1] : 0.0f;
            r.z = t > 4 * bsb + 2 ? -La[a][2] : 0.0f;
            r.w = t > 4 * bsb + 3 ? -La[a][3] : 0.0f;
            st4(Ls + t * C + 4 * bsb, r);
        }
    }
    __syncthreads();

    // Forward substitution, one thread per right-hand-side column: columns < dv are
    // beta*V (giving U, V read straight from global), the next dk columns beta*Kt (W).
    const int col = tid;
    if (col < dv + dk) {
        const bool isv = col < dv;
        const int i = col - dv;
        float x[C];
        if (isv) {
#pragma unroll
            for (int t = 0; t < C; t++)
                x[t] = t < cn ? __ldg(v + ((size_t)(tc0 + t) * H + h) * dv + col) : 0.0f;
        } else {
#pragma unroll
            for (int t = 0; t < C; t += 4) {
                const float4 kk = ld4(kT + i * LDT + t);
                x[t] = kk.x; x[t + 1] = kk.y; x[t + 2] = kk.z; x[t + 3] = kk.w;
            }
        }
#pragma unroll
        for (int t = 0; t < C; t++) {
            float2 p0 = make_float2(x[t], 0.0f), p1 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int s = 0; s + 3 < t; s += 4) {
                const float4 l = ld4(Ls + t * C + s);
                p0 = ffma2(make_float2(l.x, l.y), make_float2(x[s], x[s + 1]), p0);
                p1 = ffma2(make_float2(l.z, l.w), make_float2(x[s + 2], x[s + 3]), p1);
            }
#pragma unroll
            for (int s = t & ~3; s < t; s++) p0.x = fmaf(Ls[t * C + s], x[s], p0.x);
            x[t] = bs[t] * ((p0.x + p0.y) + (p1.x + p1.y));
        }
        if (isv) {
#pragma unroll
            for (int t = 0; t < C; t++) out[R.u + (size_t)t * dv + col] = x[t];
        } else {
#pragma unroll
            for (int t = 0; t < C; t += 4)
                st4(out + R.wt + (size_t)i * C + t, make_float4(x[t], x[t + 1], x[t + 2], x[t + 3]));
        }
    }
}

__device__ __forceinline__ void cp16(void *dst, const void *src)
{
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait2() { asm volatile("cp.async.wait_group 2;" ::: "memory"); }
__device__ __forceinline__ void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void stage(float *dst, const float *src, int nfloats)
{
    for (int f = threadIdx.x; f < nfloats / 4; f += THREADS) cp16(dst + 4 * f, src + 4 * f);
}

// tf32 helpers for the scan's products on the tensor cores (mma.sync m16n8k8, fp32
// accumulate). Every fp32 operand x is split into big = tf32(x) and small = tf32(x - big),
// and a product is accumulated as small*big + big*small + big*big ("3xTF32"): the dropped
// small*small term is below 2^-21 of |a||b|, so the result carries fp32-class accuracy.
__device__ __forceinline__ uint32_t to_tf32(float x)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void split_tf32(float x, uint32_t &big, uint32_t &small)
{
    big = to_tf32(x);
    small = to_tf32(x - __uint_as_float(big));
}

__device__ __forceinline__ void mma_tf32(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// c += A B for one 16x8x8 step: A given as fp32 fragment values (split here), B as two.
__device__ __forceinline__ void mma3(float c[4], const uint32_t ab[4], const uint32_t as[4], float b0f, float b1f)
{
    uint32_t bb0, bs0, bb1, bs1;
    split_tf32(b0f, bb0, bs0);
    split_tf32(b1f, bb1, bs1);
    mma_tf32(c, as, bb0, bb1);
    mma_tf32(c, ab, bs0, bs1);
    mma_tf32(c, ab, bb0, bb1);
}

// Shared-memory row swizzle: element n of row k sits at n ^ 8 (k mod 4) when the row width
// is a multiple of 32, so the four K rows a fragment load touches land on distinct banks.
__device__ __forceinline__ int swz(int k, int n, int width)
{
    return (width & 31) ? n : (n ^ ((k & 3) << 3));
}

// cp.async copy of a [rows][width] record block into the swizzled layout.
__device__ __forceinline__ void stage_sw(float *dst, const float *src, int rows, int width)
{
    const int cpr = width / 4;
    for (int f = threadIdx.x; f < rows * cpr; f += THREADS) {
        const int r = f / cpr, c = f - r * cpr;
        cp16(dst + r * width + swz(r, 4 * c, width), src + 4 * f);
    }
}

// A fragment (16 rows m0.., 8 K rows k0..) of a matrix stored K-major as P[k][m] (row width
// `width`, swizzled): a0 = A[g][q], a1 = A[g+8][q], a2 = A[g][q+4], a3 = A[g+8][q+4].
__device__ __forceinline__ void frag_a(const float *P, int width, int k0, int m0, int g, int q,
                                       uint32_t ab[4], uint32_t as[4])
{
    const int ka = k0 + q, kb = ka + 4;
    split_tf32(P[ka * width + swz(ka, m0 + g, width)], ab[0], as[0]);
    split_tf32(P[ka * width + swz(ka, m0 + g + 8, width)], ab[1], as[1]);
    split_tf32(P[kb * width + swz(kb, m0 + g, width)], ab[2], as[2]);
    split_tf32(P[kb * width + swz(kb, m0 + g + 8, width)], ab[3], as[3]);
}

// Shared memory of the scan for NB value columns per CTA: state block, X, three operand
// buffers (W^T, Qt^T and Kb rotate through them), M^T and 2^G_last.
constexpr size_t scan_smem(int nb)
{
    return ((size_t)DKM * nb + (size_t)C * nb + 3 * (size_t)DKM * C + (size_t)C * C + DKM) *
           sizeof(float);
}

// DKC = 128 compiles the key dimension in (the config-3 head); DKC = 0 reads it from dk.
// NB value columns per CTA (64 when dv allows, else 32). A chunk is three phases (X, O, the
// state update), each reading one operand; the operand of phase p + 2 is copied in while
// phase p computes, so every copy has two phases to land.
// Warps: in X and O, warp w owns rows 16 (w mod 4).. and columns (w / 4) NB/2.. (NB/16
// MMA tiles of 8 columns); in the state update, key rows 16 w.. and all NB columns.
template <int DKC, int NB>
__global__ void __launch_bounds__(THREADS, 1)
k_kda_chunk_scan(float *__restrict__ S, float *__restrict__ o, const float *__restrict__ ws,
                 long tok0, int nch, int T, int H, int dk_, int dv)
{
    constexpr int NT1 = NB / 16, NT3 = NB / 8;
    const int dk = DKC ? DKC : dk_;
    extern __shared__ __align__(16) float sh[];
    float *Sb = sh;                          // state block [dk][NB], swizzled
    float *Xs = Sb + DKM * NB;               // X [C][NB], swizzled
    float *const bufs = Xs + C * NB;         // 3 x [DKM * C]: W^T / Qt^T / Kb, swizzled
    float *Ms = bufs + 3 * DKM * C;          // M^T [C][C], swizzled
    float *gs = Ms + C * C;                  // 2^G_last [dk]
    const int h = blockIdx.x, j0 = blockIdx.y * NB, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
    const int t0 = 16 * (warp & 3), n0 = (warp >> 2) * (NB / 2);
    const Rec R = rec(dk, dv);
    float *Sh = S + (size_t)h * dk * dv;
    auto recp = [&](int c) { return ws + ((size_t)c * H + h) * R.total; };
    auto buf = [&](int phase) { return bufs + (phase % 3) * (DKM * C); };
    // the copies for phase p of the chunk sequence (3 phases per chunk), one commit group
    auto issue = [&](int p) {
        const int c = p / 3, k = p - 3 * c;
        if (c < nch) {
            const float *rc = recp(c);
            if (k == 0) {
                stage_sw(buf(p), rc + R.wt, dk, C);
            } else if (k == 1) {
                stage_sw(buf(p), rc + R.qt, dk, C);
                stage_sw(Ms, rc + R.mt, C, C);
            } else {
                stage_sw(buf(p), rc + R.kb, C, dk);
                stage(gs, rc + R.gc, (dk + 3) & ~3);
            }
        }
        cp_commit();
    };
    // U at this thread's X fragment: rows t0+g, t0+g+8; columns n0 + 8 nt + 2q, +1
    float u[NT1][4];
    auto load_u = [&](const float *U) {
#pragma unroll
        for (int nt = 0; nt < NT1; nt++) {
            const int col = j0 + n0 + 8 * nt + 2 * q;
            const float2 r0 = *reinterpret_cast<const float2 *>(U + (size_t)(t0 + g) * dv + col);
            const float2 r1 = *reinterpret_cast<const float2 *>(U + (size_t)(t0 + g + 8) * dv + col);
            u[nt][0] = r0.x; u[nt][1] = r0.y; u[nt][2] = r1.x; u[nt][3] = r1.y;
        }
    };

    issue(0);
    issue(1);
    for (int e = tid; e < dk * (NB / 4); e += THREADS) {
        const int i = e / (NB / 4), j = (e - i * (NB / 4)) * 4;
        *reinterpret_cast<float4 *>(Sb + i * NB + swz(i, j, NB)) = ld4(Sh + (size_t)i * dv + j0 + j);
    }
    load_u(recp(0) + R.u);

    for (int c = 0; c < nch; c++) {
        const int p1 = 3 * c;
        // P1: X = U - W S
        issue(p1 + 2);
        cp_wait2();
        __syncthreads();
        {
            const float *W = buf(p1);
            float acc[NT1][4] = {};
#pragma unroll 4
            for (int k0 = 0; k0 < dk; k0 += 8) {
                uint32_t ab[4], as[4];
                frag_a(W, C, k0, t0, g, q, ab, as);
#pragma unroll
                for (int nt = 0; nt < NT1; nt++) {
                    const int n = n0 + 8 * nt + g, ka = k0 + q, kb = ka + 4;
                    mma3(acc[nt], ab, as, Sb[ka * NB + swz(ka, n, NB)], Sb[kb * NB + swz(kb, n, NB)]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < NT1; nt++) {
                const int col = n0 + 8 * nt + 2 * q, r0 = t0 + g, r1 = t0 + g + 8;
                *reinterpret_cast<float2 *>(Xs + r0 * NB + swz(r0, col, NB)) =
                    make_float2(u[nt][0] - acc[nt][0], u[nt][1] - acc[nt][1]);
                *reinterpret_cast<float2 *>(Xs + r1 * NB + swz(r1, col, NB)) =
                    make_float2(u[nt][2] - acc[nt][2], u[nt][3] - acc[nt][3]);
            }
        }
        __syncthreads();
        // P2: O = Qt S + M X (M^T[s][t] is zero for s > t inside the diagonal 16x16 block)
        issue(p1 + 3);
        if (c + 1 < nch) load_u(recp(c + 1) + R.u);
        cp_wait2();
        __syncthreads();
        {
            const float *Q = buf(p1 + 1);
            float acc[NT1][4] = {};
#pragma unroll 4
            for (int k0 = 0; k0 < dk; k0 += 8) {
                uint32_t ab[4], as[4];
                frag_a(Q, C, k0, t0, g, q, ab, as);
#pragma unroll
                for (int nt = 0; nt < NT1; nt++) {
                    const int n = n0 + 8 * nt + g, ka = k0 + q, kb = ka + 4;
                    mma3(acc[nt], ab, as, Sb[ka * NB + swz(ka, n, NB)], Sb[kb * NB + swz(kb, n, NB)]);
                }
            }
            for (int k0 = 0; k0 < t0 + 16; k0 += 8) {
                uint32_t ab[4], as[4];
                frag_a(Ms, C, k0, t0, g, q, ab, as);
#pragma unroll
                for (int nt = 0; nt < NT1; nt++) {
                    const int n = n0 + 8 * nt + g, ka = k0 + q, kb = ka + 4;
                    mma3(acc[nt], ab, as, Xs[ka * NB + swz(ka, n, NB)], Xs[kb * NB + swz(kb, n, NB)]);
                }
            }
            const long tc0 = tok0 + (long)c * C;
#pragma unroll
            for (int nt = 0; nt < NT1; nt++) {
                const int col = j0 + n0 + 8 * nt + 2 * q;
                const long ta = tc0 + t0 + g, tb = ta + 8;
                if (ta < T)
                    *reinterpret_cast<float2 *>(o + ((size_t)ta * H + h) * dv + col) = make_float2(acc[nt][0], acc[nt][1]);
                if (tb < T)
                    *reinterpret_cast<float2 *>(o + ((size_t)tb * H + h) * dv + col) = make_float2(acc[nt][2], acc[nt][3]);
            }
        }
        __syncthreads();
        // P3: S = diag(2^G_last) S + Kb^T X
        issue(p1 + 4);
        cp_wait2();
        __syncthreads();
        {
            const float *Kb = buf(p1 + 2);
            const int i0 = 16 * warp;
            if (i0 < dk) {
                float acc[NT3][4] = {};
#pragma unroll
                for (int k0 = 0; k0 < C; k0 += 8) {
                    uint32_t ab[4], as[4];
                    frag_a(Kb, dk, k0, i0, g, q, ab, as);
#pragma unroll
                    for (int nt = 0; nt < NT3; nt++) {
                        const int n = 8 * nt + g, ka = k0 + q, kb = ka + 4;
                        mma3(acc[nt], ab, as, Xs[ka * NB + swz(ka, n, NB)], Xs[kb * NB + swz(kb, n, NB)]);
                    }
                }
#pragma unroll
                for (int nt = 0; nt < NT3; nt++) {
                    const int col = 8 * nt + 2 * q, r0 = i0 + g, r1 = i0 + g + 8;
                    float2 *p0 = reinterpret_cast<float2 *>(Sb + r0 * NB + swz(r0, col, NB));
                    float2 *pp1 = reinterpret_cast<float2 *>(Sb + r1 * NB + swz(r1, col, NB));
                    const float2 s0 = *p0, s1 = *pp1;
                    *p0 = make_float2(gs[r0] * s0.x + acc[nt][0], gs[r0] * s0.y + acc[nt][1]);
                    *pp1 = make_float2(gs[r1] * s1.x + acc[nt][2], gs[r1] * s1.y + acc[nt][3]);
                }
            }
        }
        __syncthreads();
    }
    cp_wait0();
    for (int e = tid; e < dk * (NB / 4); e += THREADS) {
        const int i = e / (NB / 4), j = (e - i * (NB / 4)) * 4;
        *reinterpret_cast<float4 *>(Sh + (size_t)i * dv + j0 + j) = ld4(Sb + i * NB + swz(i, j, NB));
    }
}

}  // namespace kdc

// Chunked prefill: dk a multiple of 8 up to 128, dv a multiple of 32 up to 128, 16-byte
// aligned S, o, q, k and alpha. Segments of SEG chunks: prep then scan, the records in scratch slot 2.
int kda_chunked(float *S, float *o, const float *q, const float *k, const float *v,
                const float *alpha, const float *beta, int T, int H, int dk, int dv,
                cudaStream_t st)
{
    using namespace kdc;
    if (T <= 0 || H <= 0) return K3D_OK;
    if (dk < 8 || dk > DKM || dk % 8 || dv < 32 || dv > 128 || dv % 32)
        return fail(K3D_EINVAL, "k3d_kda_prefill chunk=64: dk %d (8..128, multiple of 8), "
                                "dv %d (32..128, multiple of 32)", dk, dv);
    if (((uintptr_t)S | (uintptr_t)o | (uintptr_t)q | (uintptr_t)k | (uintptr_t)alpha) & 15u)
        return fail(K3D_EINVAL, "k3d_kda_prefill chunk=64: S, o, q, k and alpha must be 16-byte aligned");
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) {
        allow_smem_max(k_kda_chunk_prep);
        allow_smem_max(k_kda_chunk_scan<128, 64>);
        allow_smem_max(k_kda_chunk_scan<0, 64>);
        allow_smem_max(k_kda_chunk_scan<128, 32>);
        allow_smem_max(k_kda_chunk_scan<0, 32>);
        init |= dev_bit();
    }
    const Rec R = rec(dk, dv);
    const int nch = (T + C - 1) / C;
    const int seg = nch < SEG ? nch : SEG;
    float *ws = (float *)scratch((size_t)seg * H * R.total * sizeof(float), 2);
    if (!ws) return fail(K3D_ENOMEM, "k3d_kda_prefill: chunk records");
    for (int c0 = 0; c0 < nch; c0 += seg) {
        const int n = nch - c0 < seg ? nch - c0 : seg;
        const long tok0 = (long)c0 * C;
        k_kda_chunk_prep<<<dim3(n, H), THREADS, prep_smem(), st>>>(q, k, v, alpha, beta, ws, tok0,
                                                                    T, H, dk, dv);
        note_launch();
        K3_TRY(check_launch("kda chunk prep"));
        if (dv % 64 == 0) {
            const dim3 grid(H, dv / 64);
            if (dk == 128)
                k_kda_chunk_scan<128, 64><<<grid, THREADS, scan_smem(64), st>>>(S, o, ws, tok0, n, T, H, dk, dv);
            else
                k_kda_chunk_scan<0, 64><<<grid, THREADS, scan_smem(64), st>>>(S, o, ws, tok0, n, T, H, dk, dv);
        } else {
            const dim3 grid(H, dv / 32);
            if (dk == 128)
                k_kda_chunk_scan<128, 32><<<grid, THREADS, scan_smem(32), st>>>(S, o, ws, tok0, n, T, H, dk, dv);
            else
                k_kda_chunk_scan<0, 32><<<grid, THREADS, scan_smem(32), st>>>(S, o, ws, tok0, n, T, H, dk, dv);
        }
        note_launch();
        K3_TRY(check_launch("kda chunk scan"));
    }
    return K3D_OK;
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
    if (chunk == 64) return kda_chunked(S, o, q, k, v, alpha, beta, T, H, dk, dv, stream());
    if (chunk != 0)
        return fail(K3D_EINVAL, "k3d_kda_prefill: chunk %d (0 sequential, 64 chunked)", chunk);
    return kda_seq(S, o, q, k, v, alpha, beta, T, H, dk, dv, stream());
}

}  // extern "C"
