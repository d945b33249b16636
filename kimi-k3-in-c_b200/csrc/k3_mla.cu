// k3_mla.cu -- MLA decode over a bf16 latent cache with absorbed weights (config 2),
// following k3_mla_cached (k3_ops.c:321-410).
//
// The CPU engine caches per-head EXPANDED keys and values (fp32, 256 per head) because
// re-expanding latents through kv_b costs an O(L) sweep of GEMVs on a CPU. On the GPU the
// cache stays compressed (576 bf16 per position: the normalised latent + the rotated rope
// key, 74x smaller) and kv_b is folded into the query and the output instead:
//     score(h, s) = q_nope_h . (W_uk_h c_s) + q_rope_h . kr_s = (W_uk_h^T q_nope_h) . c_s + ...
//     out_h       = W_uv_h (sum_s p_s c_s)
// so every cached position is read once per step for all heads together (the latent is
// shared by the 64 heads, as the CPU's rope slot is), and no per-position GEMV is needed.
//
// Kernels per decode step (B sequences, one token each):
//   1. grouped bf16 GEMV of x:  q_a -> ql,  kv_a -> c,  g -> gate          (k3_gemv.cu)
//   2. k_mla_prep:   RMSNorm ql; RMSNorm the latent part of c; RoPE the rope part at
//                    position pos; write the bf16 cache entry at pos
//   3. q_b GEMV:     ql -> q [H][nope + rope]
//   4. k_mla_absorb: q_lat_h = W_uk_h^T q_nope_h (512) and RoPE(q_rope_h)
//   5. k_mla_attn:   split-L flash decoding, 8 heads per CTA over tiles of 32 positions;
//                    online softmax in fp32; partial (m, l, ctx) per split
//   6. k_mla_merge:  merge splits, o_h = W_uv_h ctx_h, times sigmoid(gate)
//   7. o_proj GEMV (accumulating into the residual when asked)
#include "k3_common.cuh"
#include "k3_ops.cuh"

namespace k3 {

static const int kHG = 8;     // heads per attention CTA
static const int kTP = 32;    // positions per tile

struct MlaDims {
    int hidden, H, q_lora, kv_lora, qn, qr, vh, kvw, qh, nsplit;
    float theta, eps, scale;
};

__device__ __forceinline__ void rope_pairs(float *v, int d, int pos, float theta, int tid, int nt)
{
    for (int i = tid; i < d / 2; i += nt) {
        const double f = pow((double)theta, -2.0 * (double)i / (double)d);
        const double a = (double)pos * f;
        const float c = (float)cos(a), s = (float)sin(a);
        const float x0 = v[2 * i], x1 = v[2 * i + 1];
        v[2 * i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        v[2 * i + 1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
}

__device__ __forceinline__ double block_sum_d2(double v, double *red)
{
    v = warp_sum_d(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) s += red[i];
    return s;
}

// one CTA per sequence
__global__ void k_mla_prep(float *ql, float *c, uint16_t *cache, const float *q_a_norm,
                           const float *kv_a_norm, const int *pos_p, MlaDims d, int cap)
{
    __shared__ double red[32];
    const int b = blockIdx.x;
    const int pos = *pos_p;
    if (pos < 0 || pos >= cap) {
        if (threadIdx.x == 0) k3_raise(K3D_EBOUND, K3_SITE_MLA);
        return;
    }
    float *qb = ql + (size_t)b * d.q_lora;
    float *cb = c + (size_t)b * d.kvw;
    double ss = 0.0;
    for (int i = threadIdx.x; i < d.q_lora; i += blockDim.x) ss = fma((double)qb[i], (double)qb[i], ss);
    ss = block_sum_d2(ss, red);
    const float inv_q = (float)(1.0 / sqrt(ss / (double)d.q_lora + (double)d.eps));
    __syncthreads();
    double sl = 0.0;
    for (int i = threadIdx.x; i < d.kv_lora; i += blockDim.x) sl = fma((double)cb[i], (double)cb[i], sl);
    sl = block_sum_d2(sl, red);
    const float inv_c = (float)(1.0 / sqrt(sl / (double)d.kv_lora + (double)d.eps));
    for (int i = threadIdx.x; i < d.q_lora; i += blockDim.x)
        qb[i] = __fmul_rn(__fmul_rn(q_a_norm[i], qb[i]), inv_q);
    for (int i = threadIdx.x; i < d.kv_lora; i += blockDim.x)
        cb[i] = __fmul_rn(__fmul_rn(kv_a_norm[i], cb[i]), inv_c);
    __syncthreads();
    if (d.theta > 0.f) rope_pairs(cb + d.kv_lora, d.qr, pos, d.theta, threadIdx.x, blockDim.x);
    __syncthreads();
    uint16_t *dst = cache + ((size_t)b * cap + pos) * d.kvw;
    for (int i = threadIdx.x; i < d.kvw; i += blockDim.x) dst[i] = f32_to_bf16_bits(cb[i]);
}

// grid (H, kv_lora / 128, B), block (16, 8): q_lat[j] = sum_i W_uk[h][i][j] q_nope[i] for a
// 128-wide block of j, 8 j per thread (16-byte loads), the 8 thread rows splitting i;
// then RoPE(q_rope_h). Output qa [B][H][kvw].
__global__ void k_mla_absorb(float *qa, const float *q, const uint16_t *kv_b, const int *pos_p,
                             MlaDims d)
{
    __shared__ float qs[256];
    __shared__ float part[8][128 + 4];
    const int h = blockIdx.x, jb = blockIdx.y, b = blockIdx.z;
    const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * 16 + tx;
    const float *qh = q + ((size_t)b * d.H + h) * d.qh;
    for (int i = tid; i < d.qh; i += 128) qs[i] = qh[i];
    __syncthreads();
    const size_t kvd = (size_t)(d.qn + d.vh);
    const uint16_t *wuk = kv_b + (size_t)h * kvd * d.kv_lora + jb * 128 + tx * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int per = (d.qn + 7) / 8;
#pragma unroll 4
    for (int ii = 0; ii < per; ii++) {
        const int i = ty * per + ii;
        if (i < d.qn) {
            const uint4 w = __ldg(reinterpret_cast<const uint4 *>(wuk + (size_t)i * d.kv_lora));
            const float qi = qs[i];
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                acc[2 * k] = fmaf(__uint_as_float(u[k] << 16), qi, acc[2 * k]);
                acc[2 * k + 1] = fmaf(__uint_as_float(u[k] & 0xffff0000u), qi, acc[2 * k + 1]);
            }
        }
    }
#pragma unroll
    for (int k = 0; k < 8; k++) part[ty][tx * 8 + k] = acc[k];
    __syncthreads();
    float *out = qa + ((size_t)b * d.H + h) * d.kvw;
    {
        const int j = tid;   // 0..127
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < 8; r++) v += part[r][j];
        out[jb * 128 + j] = v;
    }
    if (jb == 0) {
        if (d.theta > 0.f) {
            __syncthreads();
            rope_pairs(qs + d.qn, d.qr, *pos_p, d.theta, tid, 128);
            __syncthreads();
        }
        for (int i = tid; i < d.qr; i += 128) out[d.kv_lora + i] = qs[d.qn + i];
    }
}

// grid (nsplit, H / kHG, B), 256 threads. Partials: part [B][H][nsplit][kv_lora + 2]
// (ctx, m, l).
__global__ void __launch_bounds__(256) k_mla_attn(float *part, const float *qa,
                                                  const uint16_t *cache, const int *pos_p,
                                                  MlaDims d, int cap)
{
    extern __shared__ float sm[];
    const int split = blockIdx.x, hg = blockIdx.y, b = blockIdx.z;
    const int kvw = d.kvw;                 // 576
    const int pitch = kvw + 2;             // bf16 elements per smem row (odd word count)
    float *Q = sm;                                               // [kHG][kvw]
    float *P = Q + kHG * kvw;                                    // [kHG][kTP]
    uint32_t *Ct = reinterpret_cast<uint32_t *>(P + kHG * kTP);  // [kTP][pitch/2] bf16x2
    const int n = *pos_p + 1;              // positions attended (including the new one)
    const int per = (n + d.nsplit - 1) / d.nsplit;
    const int s0 = split * per, s1 = min(n, s0 + per);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < kHG * kvw; i += blockDim.x) {
        const int hh = i / kvw, k = i % kvw;
        Q[i] = qa[((size_t)b * d.H + hg * kHG + hh) * kvw + k];
    }
    float m = -INFINITY, l = 0.f;            // per head, owned by warp `warp` (lane 0 copy)
    float ctx[16];                           // head = warp, j = lane + 32 i
#pragma unroll
    for (int i = 0; i < 16; i++) ctx[i] = 0.f;
    const uint16_t *cb = cache + (size_t)b * cap * kvw;
    for (int t0 = s0; t0 < s1; t0 += kTP) {
        const int nt = min(kTP, s1 - t0);
        __syncthreads();
        // stage the tile: rows of kvw bf16 (16-byte aligned in global) into odd-pitch smem
        const int words = kvw / 2;
        for (int i = tid; i < nt * words; i += blockDim.x) {
            const int p = i / words, w = i % words;
            Ct[p * (pitch / 2) + w] =
                reinterpret_cast<const uint32_t *>(cb + (size_t)(t0 + p) * kvw)[w];
        }
        __syncthreads();
        // scores: warp = head, lane = position
        {
            const int hh = warp, p = lane;
            float s = -INFINITY;
            if (p < nt) {
                const float *q = Q + hh * kvw;
                const uint32_t *cr = Ct + p * (pitch / 2);
                float acc = 0.f;
                for (int w = 0; w < words; w++) {
                    const uint32_t v = cr[w];
                    acc = fmaf(q[2 * w], __uint_as_float(v << 16), acc);
                    acc = fmaf(q[2 * w + 1], __uint_as_float(v & 0xffff0000u), acc);
                }
                s = acc * d.scale;
            }
            const float tmax = warp_max(s);
            const float mnew = fmaxf(m, tmax);
            const float corr = (m == -INFINITY) ? 0.f : expf(m - mnew);
            const float e = (p < nt) ? expf(s - mnew) : 0.f;
            P[hh * kTP + p] = e;
            l = l * corr + warp_sum(e);
            m = mnew;
#pragma unroll
            for (int i = 0; i < 16; i++) ctx[i] *= corr;
        }
        __syncwarp();
        // ctx[h][j] += sum_p P[h][p] * C[p][j]
        for (int p = 0; p < nt; p++) {
            const float pr = P[warp * kTP + p];
            const uint32_t *cr = Ct + p * (pitch / 2);
#pragma unroll
            for (int i = 0; i < 16; i++) {
                const int j = lane + 32 * i;
                if (j < d.kv_lora) {
                    const uint32_t v = cr[j >> 1];
                    const float c = (j & 1) ? __uint_as_float(v & 0xffff0000u) : __uint_as_float(v << 16);
                    ctx[i] = fmaf(pr, c, ctx[i]);
                }
            }
        }
    }
    const int hh = hg * kHG + warp;
    float *dst = part + (((size_t)b * d.H + hh) * d.nsplit + split) * (d.kv_lora + 2);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const int j = lane + 32 * i;
        if (j < d.kv_lora) dst[j] = ctx[i];
    }
    if (lane == 0) { dst[d.kv_lora] = m; dst[d.kv_lora + 1] = l; }
}

// grid (H, B), 256 threads: merge splits, o = W_uv ctx, gate. heads [B][H*vh].
__global__ void k_mla_merge(float *heads, const float *part, const uint16_t *kv_b,
                            const float *gate, MlaDims d)
{
    extern __shared__ float cx[];   // [kv_lora]
    __shared__ float wsc[256];
    __shared__ float Lsum;
    const int h = blockIdx.x, b = blockIdx.y;
    const float *pp = part + ((size_t)b * d.H + h) * d.nsplit * (d.kv_lora + 2);
    const int stride = d.kv_lora + 2;
    if (threadIdx.x == 0) {
        float M = -INFINITY;
        for (int s = 0; s < d.nsplit; s++) M = fmaxf(M, pp[s * stride + d.kv_lora]);
        float L = 0.f;
        for (int s = 0; s < d.nsplit; s++) {
            const float ms = pp[s * stride + d.kv_lora];
            const float w = (ms == -INFINITY) ? 0.f : expf(ms - M);
            wsc[s] = w;
            L += w * pp[s * stride + d.kv_lora + 1];
        }
        Lsum = L;
    }
    __syncthreads();
    const float invL = 1.0f / Lsum;
    for (int j = threadIdx.x; j < d.kv_lora; j += blockDim.x) {
        float a = 0.f;
        for (int s = 0; s < d.nsplit; s++) a = fmaf(wsc[s], pp[s * stride + j], a);
        cx[j] = a * invL;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const size_t kvd = (size_t)(d.qn + d.vh);
    for (int r = warp; r < d.vh; r += nw) {
        const uint16_t *row = kv_b + ((size_t)h * kvd + d.qn + r) * d.kv_lora;
        float acc = 0.f;
        for (int j = lane; j < d.kv_lora; j += 32) acc = fmaf(bf16_to_f32(row[j]), cx[j], acc);
        acc = warp_sum(acc);
        if (lane == 0) {
            const size_t o = (size_t)b * d.H * d.vh + (size_t)h * d.vh + r;
            if (gate) acc = acc * (1.0f / (1.0f + expf(-gate[o])));
            heads[o] = acc;
        }
    }
}

static size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

struct MlaWs {
    float *ql, *c, *gate, *q, *qa, *part, *heads;
    size_t total;
};

static int mla_nsplit(int B, int H, int cap)
{
    int per_b = (H + kHG - 1) / kHG;
    int want = (sm_count() > 0 ? sm_count() : 148) * 2;
    int ns = (want + B * per_b - 1) / (B * per_b);
    const int max_ns = (cap + kTP - 1) / kTP;
    if (ns > max_ns) ns = max_ns;
    if (ns > 256) ns = 256;
    return ns < 1 ? 1 : ns;
}

static MlaWs mla_layout(const K3dMlaShape *s, int B, int cap, void *base)
{
    MlaWs L;
    const int kvw = s->kv_lora + s->qk_rope, qh = s->qk_nope + s->qk_rope;
    const int ns = mla_nsplit(B, s->n_heads, cap);
    size_t off = 0;
    char *bp = (char *)base;
    auto take = [&](size_t bytes) { char *p = bp + off; off += al256(bytes); return (float *)p; };
    L.ql = take((size_t)B * s->q_lora * 4);
    L.c = take((size_t)B * kvw * 4);
    L.gate = take((size_t)B * s->n_heads * s->v_head * 4);
    L.q = take((size_t)B * s->n_heads * qh * 4);
    L.qa = take((size_t)B * s->n_heads * kvw * 4);
    L.part = take((size_t)B * s->n_heads * ns * (s->kv_lora + 2) * 4);
    L.heads = take((size_t)B * s->n_heads * s->v_head * 4);
    L.total = off;
    return L;
}

int mla_decode(float *out, const float *x, const K3dMlaW *w, const K3dMlaShape *s, int B,
               uint16_t *cache, int cap, const int *pos, int accumulate, void *ws,
               cudaStream_t st)
{
    MlaWs L = mla_layout(s, B, cap, ws);
    MlaDims d;
    d.hidden = s->hidden; d.H = s->n_heads; d.q_lora = s->q_lora; d.kv_lora = s->kv_lora;
    d.qn = s->qk_nope; d.qr = s->qk_rope; d.vh = s->v_head;
    d.kvw = s->kv_lora + s->qk_rope; d.qh = s->qk_nope + s->qk_rope;
    d.nsplit = mla_nsplit(B, s->n_heads, cap);
    d.theta = s->rope_theta; d.eps = s->eps; d.scale = 1.0f / sqrtf((float)d.qh);
    prof_begin("mla.proj_in");
    {
        const uint16_t *Ws[3] = {w->q_a, w->kv_a, w->g};
        float *Ys[3] = {L.ql, L.c, L.gate};
        const int rows[3] = {s->q_lora, d.kvw, d.H * d.vh};
        if (B <= 4) {
            K3_TRY(gemv_bf16_multi(s->out_gate ? 3 : 2, Ws, Ys, rows, x, s->hidden, B, st));
        } else {
            K3_TRY(gemv_bf16(L.ql, x, w->q_a, s->hidden, s->q_lora, B, 0, st));
            K3_TRY(gemv_bf16(L.c, x, w->kv_a, s->hidden, d.kvw, B, 0, st));
            if (s->out_gate) K3_TRY(gemv_bf16(L.gate, x, w->g, s->hidden, d.H * d.vh, B, 0, st));
        }
    }
    prof_end("mla.proj_in");
    prof_begin("mla.core");
    k_mla_prep<<<B, 256, 0, st>>>(L.ql, L.c, cache, w->q_a_norm, w->kv_a_norm, pos, d, cap);
    note_launch();
    K3_TRY(check_launch("mla prep"));
    K3_TRY(gemv_bf16(L.q, L.ql, w->q_b, s->q_lora, d.H * d.qh, B, 0, st));
    k_mla_absorb<<<dim3(d.H, d.kv_lora / 128, B), dim3(16, 8), 0, st>>>(L.qa, L.q, w->kv_b, pos, d);
    note_launch();
    K3_TRY(check_launch("mla absorb"));
    const size_t smem = ((size_t)kHG * d.kvw + kHG * kTP) * 4 + (size_t)kTP * (d.kvw + 2) * 2;
    static bool init = false;
    if (!init) {
        allow_smem_max(k_mla_attn);
        init = true;
    }
    k_mla_attn<<<dim3(d.nsplit, d.H / kHG, B), 256, smem, st>>>(L.part, L.qa, cache, pos, d, cap);
    note_launch();
    K3_TRY(check_launch("mla attn"));
    k_mla_merge<<<dim3(d.H, B), 256, (size_t)d.kv_lora * 4, st>>>(L.heads, L.part, w->kv_b,
                                                                  s->out_gate ? L.gate : nullptr, d);
    note_launch();
    K3_TRY(check_launch("mla merge"));
    prof_end("mla.core");
    prof_begin("mla.proj_out");
    K3_TRY(gemv_bf16(out, L.heads, w->o, d.H * d.vh, s->hidden, B, accumulate, st));
    prof_end("mla.proj_out");
    return K3D_OK;
}

}  // namespace k3

using namespace k3;

extern "C" {

size_t k3d_mla_ws_bytes(const K3dMlaShape *s, int B, int cap)
{
    if (!s || B < 1 || cap < 1) return 0;
    return mla_layout(s, B, cap, nullptr).total + 256;
}

int k3d_mla_decode(float *out, const float *x, const K3dMlaW *w, const K3dMlaShape *s, int B,
                   uint16_t *cache, int cap, const int *pos, int accumulate, void *ws,
                   size_t ws_bytes)
{
    K3_TRY(ensure_ctx());
    if (!out || !x || !w || !s || !cache || !pos || !ws)
        return fail(K3D_EINVAL, "k3d_mla_decode null pointer");
    if (!w->q_a || !w->q_b || !w->kv_a || !w->kv_b || !w->o || !w->q_a_norm || !w->kv_a_norm ||
        (s->out_gate && !w->g))
        return fail(K3D_EINVAL, "k3d_mla_decode weight missing");
    if (s->n_heads % kHG || s->kv_lora > 512 || s->kv_lora % 128 || s->qk_rope % 2 ||
        ((s->kv_lora + s->qk_rope) % 8) || s->qk_nope + s->qk_rope > 256 || s->hidden % 8)
        return fail(K3D_EINVAL, "k3d_mla_decode: n_heads %% 8, kv_lora a multiple of 128 up to "
                                "512, even rope, (kv_lora + rope) %% 8, nope + rope <= 256");
    if (ws_bytes < k3d_mla_ws_bytes(s, B, cap)) return fail(K3D_EINVAL, "k3d_mla_decode workspace");
    return mla_decode(out, x, w, s, B, cache, cap, pos, accumulate, ws, stream());
}

}  // extern "C"
