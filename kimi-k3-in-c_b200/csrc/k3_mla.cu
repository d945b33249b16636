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
//   5. k_mla_attn_tc: split-L flash decoding on tensor cores (mma.sync m16n8k16, bf16
//                    in, fp32 accumulate), 16 heads per CTA over tiles of 64 positions:
//                    scores = C_tile Q^T and ctx += P C_tile, with the fp32 operands Q and
//                    P each split into bf16 hi + lo so no precision is lost to bf16;
//                    online softmax in fp32; partial (m, l, ctx) per split
//   6. k_mla_merge:  merge splits, o_h = W_uv_h ctx_h, times sigmoid(gate); one CTA per
//                    (head, 32 output rows)
//   7. o_proj GEMV (accumulating into the residual when asked)
#include <vector>

#include "k3_common.cuh"
#include "k3_ops.cuh"

namespace k3 {


struct MlaDims {
    int hidden, H, q_lora, kv_lora, qn, qr, vh, kvw, qh, nsplit;
    float theta, eps, scale;
};

// cos and sin of the RoPE angle pos * theta^(-2i/d) in double. The angle (up to ~1e6 rad)
// is first reduced modulo 2*pi against a two-part constant (the high part has 33
// significant bits, so k * hi is exact for k < 2^20) so the double cos/sin see a small
// argument and stay on their fast path.
__device__ __forceinline__ void rope_angle(int i, int d, int pos, float theta, float &c, float &s)
{
    const double f = pow((double)theta, -2.0 * (double)i / (double)d);
    const double a = (double)pos * f;
    const double two_pi_hi = 6.28318530717958623200;          // 2*pi rounded to double
    const double two_pi_lo = 2.44929359829470635445e-16;      // 2*pi - two_pi_hi
    const double k = rint(a * 0.15915494309189533577);
    const double hi33 = __longlong_as_double(__double_as_longlong(two_pi_hi) & ~0xFFFFFll);
    const double r = ((a - k * hi33) - k * (two_pi_hi - hi33)) - k * two_pi_lo;
    c = (float)cos(r);
    s = (float)sin(r);
}

__device__ __forceinline__ void rope_apply(float *v, int i, float c, float s)
{
    const float x0 = v[2 * i], x1 = v[2 * i + 1];
    v[2 * i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    v[2 * i + 1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
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

// cos/sin of every position's RoPE angles, computed once per (theta, rope dim, capacity):
// tab[pos][i] = (cos, sin) of pos * theta^(-2i/qr). grid over cap * qr/2 threads.
__global__ void k_rope_table(float2 *tab, int qr, int cap, float theta)
{
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    const int np = qr / 2;
    if (k >= cap * np) return;
    float cs, sn;
    rope_angle(k % np, qr, k / np, theta, cs, sn);
    tab[k] = make_float2(cs, sn);
}

// one CTA per sequence, 256 threads: every global load (q_lora and kv activations, both
// norm weights, the position's RoPE row) is issued up front, so the kernel pays the memory
// latency once. Thread t owns q elements t + 256 i (i < 8) and latent elements t + 256 i
// (i < 3).
__global__ void __launch_bounds__(256) k_mla_prep(float *ql, float *c, uint16_t *cache,
                                                  const float2 *rope_tab, const float *q_a_norm,
                                                  const float *kv_a_norm, const int *pos_p,
                                                  MlaDims d, int cap)
{
    pdl_wait();
    pdl_trigger();
    __shared__ double red[32];
    __shared__ float crope[256];
    const int b = blockIdx.x, tid = threadIdx.x;
    const int pos = *pos_p;
    float *qb = ql + (size_t)b * d.q_lora;
    float *cb = c + (size_t)b * d.kvw;
    float qv[8], qw[8], cv[3], cw[3];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int k = tid + 256 * i;
        qv[i] = k < d.q_lora ? qb[k] : 0.f;
        qw[i] = k < d.q_lora ? q_a_norm[k] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const int k = tid + 256 * i;
        cv[i] = k < d.kvw ? cb[k] : 0.f;
        cw[i] = k < d.kv_lora ? kv_a_norm[k] : 0.f;
    }
    float2 rp = make_float2(1.f, 0.f);
    const bool pos_ok = pos >= 0 && pos < cap;
    if (d.theta > 0.f && pos_ok && tid < d.qr / 2) rp = rope_tab[(size_t)pos * (d.qr / 2) + tid];
    if (!pos_ok) {
        if (tid == 0) k3_raise(K3D_EBOUND, K3_SITE_MLA);
        return;
    }
    double ss = 0.0, sl = 0.0;
#pragma unroll
    for (int i = 0; i < 8; i++) ss = fma((double)qv[i], (double)qv[i], ss);
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const int k = tid + 256 * i;
        if (k < d.kv_lora) sl = fma((double)cv[i], (double)cv[i], sl);
    }
    ss = block_sum_d2(ss, red);
    __syncthreads();
    sl = block_sum_d2(sl, red);
    const float inv_q = (float)(1.0 / sqrt(ss / (double)d.q_lora + (double)d.eps));
    const float inv_c = (float)(1.0 / sqrt(sl / (double)d.kv_lora + (double)d.eps));
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int k = tid + 256 * i;
        if (k < d.q_lora) qb[k] = __fmul_rn(__fmul_rn(qw[i], qv[i]), inv_q);
    }
    uint16_t *dst = cache + ((size_t)b * cap + pos) * d.kvw;
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const int k = tid + 256 * i;
        if (k < d.kv_lora) {
            const float v = __fmul_rn(__fmul_rn(cw[i], cv[i]), inv_c);
            cb[k] = v;
            dst[k] = f32_to_bf16_bits(v);
        } else if (k < d.kvw) {
            crope[k - d.kv_lora] = cv[i];           // the rope part, rotated below
        }
    }
    __syncthreads();
    if (tid < d.qr / 2) {
        if (d.theta > 0.f) rope_apply(crope, tid, rp.x, rp.y);
        const int k = d.kv_lora + 2 * tid;
        cb[k] = crope[2 * tid];
        cb[k + 1] = crope[2 * tid + 1];
        dst[k] = f32_to_bf16_bits(crope[2 * tid]);
        dst[k + 1] = f32_to_bf16_bits(crope[2 * tid + 1]);
    }
}

// The latent half of k_mla_prep for one sequence, by 128 threads: RMSNorm of the latent
// part of c (sum of squares in double), RoPE of the rope part at pos, the bf16 cache entry
// at pos. Thread t owns latent elements t + 128 i.
__device__ __forceinline__ void mla_latent_prep(float *c, uint16_t *cache, const float2 *rope_tab,
                                                const float *kv_a_norm, const int *pos_p,
                                                const MlaDims &d, int cap, int b, int tid)
{
    __shared__ double red[4];
    __shared__ float crope[256];
    const int pos = *pos_p;
    const bool pos_ok = pos >= 0 && pos < cap;
    if (!pos_ok) {
        if (tid == 0) k3_raise(K3D_EBOUND, K3_SITE_MLA);
        return;
    }
    float *cb = c + (size_t)b * d.kvw;
    float cv[6], cw[6];
#pragma unroll
    for (int i = 0; i < 6; i++) {
        const int k = tid + 128 * i;
        cv[i] = k < d.kvw ? cb[k] : 0.f;
        cw[i] = k < d.kv_lora ? kv_a_norm[k] : 0.f;
    }
    float2 rp = make_float2(1.f, 0.f);
    if (d.theta > 0.f && tid < d.qr / 2) rp = rope_tab[(size_t)pos * (d.qr / 2) + tid];
    double sl = 0.0;
#pragma unroll
    for (int i = 0; i < 6; i++)
        if (tid + 128 * i < d.kv_lora) sl = fma((double)cv[i], (double)cv[i], sl);
    sl = warp_sum_d(sl);
    if ((tid & 31) == 0) red[tid >> 5] = sl;
    __syncthreads();
    sl = (red[0] + red[1]) + (red[2] + red[3]);
    const float inv_c = (float)(1.0 / sqrt(sl / (double)d.kv_lora + (double)d.eps));
    uint16_t *dst = cache + ((size_t)b * cap + pos) * d.kvw;
#pragma unroll
    for (int i = 0; i < 6; i++) {
        const int k = tid + 128 * i;
        if (k < d.kv_lora) dst[k] = f32_to_bf16_bits(__fmul_rn(__fmul_rn(cw[i], cv[i]), inv_c));
        else if (k < d.kvw) crope[k - d.kv_lora] = cv[i];
    }
    __syncthreads();
    if (tid < d.qr / 2) {
        if (d.theta > 0.f) rope_apply(crope, tid, rp.x, rp.y);
        const int k = d.kv_lora + 2 * tid;
        dst[k] = f32_to_bf16_bits(crope[2 * tid]);
        dst[k + 1] = f32_to_bf16_bits(crope[2 * tid + 1]);
    }
}

// grid (H, kv_lora / 128 [+ 1], B), block (16, 8): q_lat[j] = sum_i W_uk[h][i][j] q_nope[i]
// for a 128-wide block of j, 8 j per thread (16-byte loads), the 8 thread rows splitting i;
// then RoPE(q_rope_h). Output qa [B][H][kvw]. With latent (decode of up to four tokens,
// where q_b normalises its input itself and k_mla_prep is not launched) the extra row of
// CTAs y = kv_lora / 128 does the latent half of k_mla_prep (CTA x = 0 of each sequence).
__global__ void k_mla_absorb(float *qa, const float *q, const uint16_t *kv_b, const float2 *rope_tab,
                             const int *pos_p, MlaDims d, int cap, float *c, uint16_t *cache,
                             const float *kv_a_norm, int latent)
{
    if (latent && (int)blockIdx.y == d.kv_lora / 128) {
        pdl_wait();
        pdl_trigger();
        if (blockIdx.x == 0)
            mla_latent_prep(c, cache, rope_tab, kv_a_norm, pos_p, d, cap, blockIdx.z,
                            threadIdx.y * 16 + threadIdx.x);
        return;
    }
    __shared__ float qs[256];
    __shared__ float part[8][128 + 4];
    const int h = blockIdx.x, jb = blockIdx.y, b = blockIdx.z;
    const int tx = threadIdx.x, ty = threadIdx.y, tid = ty * 16 + tx;
    const size_t kvd = (size_t)(d.qn + d.vh);
    const uint16_t *wuk = kv_b + (size_t)h * kvd * d.kv_lora + jb * 128 + tx * 8;
    const int per = (d.qn + 7) / 8;          // rows of W_uk per thread row (<= 32)
    // all of a group's 16-byte loads are issued before any arithmetic; the first group's
    // before the programmatic wait (weights)
    uint4 wv[16];
    auto load_group = [&](int g0) {
#pragma unroll
        for (int ii = 0; ii < 16; ii++) {
            // clamped row (always a valid address); out-of-range rows get weight 0 below
            const int i = min(ty * per + min(g0 + ii, per - 1), d.qn - 1);
            wv[ii] = __ldg(reinterpret_cast<const uint4 *>(wuk + (size_t)i * d.kv_lora));
        }
    };
    load_group(0);
    pdl_wait();
    pdl_trigger();
    const float *qh = q + ((size_t)b * d.H + h) * d.qh;
    for (int i = tid; i < d.qh; i += 128) qs[i] = qh[i];
    __syncthreads();
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int g0 = 0; g0 < per; g0 += 16) {
        if (g0 > 0) load_group(g0);
#pragma unroll
        for (int ii = 0; ii < 16; ii++) {
            const int i = min(ty * per + g0 + ii, d.qn - 1);
            const float qi = (g0 + ii < per && ty * per + g0 + ii < d.qn) ? qs[i] : 0.f;
            const uint32_t u[4] = {wv[ii].x, wv[ii].y, wv[ii].z, wv[ii].w};
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
    // q_lat as the attention's bf16 operand pair: hi = bf16(v), lo = bf16(v - hi)
    uint16_t *qhi = reinterpret_cast<uint16_t *>(qa);
    uint16_t *ohi = qhi + ((size_t)b * d.H + h) * d.kvw;
    uint16_t *olo = ohi + (size_t)gridDim.z * d.H * d.kvw;
    auto put = [&](int k, float v) {
        const uint16_t hb = f32_to_bf16_bits(v);
        ohi[k] = hb;
        olo[k] = f32_to_bf16_bits(v - bf16_to_f32(hb));
    };
    {
        const int j = tid;   // 0..127
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < 8; r++) v += part[r][j];
        put(jb * 128 + j, v);
    }
    if (jb == 0) {
        const int pos = *pos_p;
        if (d.theta > 0.f && pos >= 0 && pos < cap) {   // else k_mla_prep raised K3D_EBOUND
            const float2 *rt = rope_tab + (size_t)pos * (d.qr / 2);
            __syncthreads();
            for (int i = tid; i < d.qr / 2; i += 128) rope_apply(qs + d.qn, i, rt[i].x, rt[i].y);
            __syncthreads();
        }
        for (int i = tid; i < d.qr; i += 128) put(d.kv_lora + i, qs[d.qn + i]);
    }
}

// ------------------------------------------------------------ attention core
// Tensor-core split-L flash decoding. grid (nsplit, ceil(H / 16), B), 128 threads
// (4 warps). A CTA owns up to 16 heads (hgn = min(16, H - 16*hg); rows beyond are zero)
// and the positions [s0, s1) of its split, in tiles of 64:
//   scores  S[p][h] = C[p] . q_h      M = 64 positions (16 per warp), N = 16 heads,
//                                     K = kvw; A = C tile (ldmatrix), B = Q rows
//   softmax per head over the tile (max and sum across the 4 warps through shared
//           memory), running (m, l) and the ctx rescale as in flash decoding
//   ctx     O[h][j] += P[h][p] C[p][j]  M = 16 heads, N = kv_lora (kv_lora/4 per warp),
//                                     K = 64 positions; B = C tile (ldmatrix.trans)
// Q (fp32) and P (fp32) are each written as bf16 hi + bf16 lo (hi = bf16(v), lo =
// bf16(v - hi)), two MMAs per step, so the products carry 16 significant bits of each
// fp32 operand; C is bf16 already. Accumulation is fp32 throughout.
// Partials: part [B][H][nsplit][kv_lora + 2] (unnormalised ctx, m, l).
static const int kAHG = 16;     // heads per CTA
static const int kATP = 64;     // positions per tile

__device__ __forceinline__ uint32_t pack_bf16(float lo_elem, float hi_elem)
{
    return (uint32_t)f32_to_bf16_bits(lo_elem) | ((uint32_t)f32_to_bf16_bits(hi_elem) << 16);
}

__device__ __forceinline__ void ldsm4(uint32_t r[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}

__device__ __forceinline__ void ldsm4t(uint32_t r[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}

__device__ __forceinline__ void mma_bf16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp16(uint32_t dst, const void *src, uint32_t src_bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                 :: "r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

// Stages tile rows [t0, t0 + 64) of the cache (rows >= s1 are zero-filled; their source
// address is clamped to a valid row and no bytes are read from it).
__device__ __forceinline__ void mla_stage_tile(uint32_t dst, const uint16_t *cb, int t0, int s1,
                                               int kvw, int pitch)
{
    const int chunks = kvw / 8;                 // 16-byte chunks per row
    // (r, c) of chunk i = threadIdx.x + 128 k, advanced incrementally (no division per chunk)
    int r = threadIdx.x / chunks, c = threadIdx.x % chunks;
    const int dr = 128 / chunks, dc = 128 % chunks;
    for (int i = threadIdx.x; i < kATP * chunks; i += 128) {
        const int row = t0 + r;
        const bool ok = row < s1;
        const uint16_t *src = cb + (size_t)(ok ? row : t0) * kvw + c * 8;
        cp16(dst + (uint32_t)(r * pitch + c * 8) * 2u, src, ok ? 16u : 0u);
        r += dr;
        c += dc;
        if (c >= chunks) { c -= chunks; r++; }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int NT>   // n8 tiles of ctx per warp: kv_lora / 32
__global__ void __launch_bounds__(128) k_mla_attn_tc(float *part, const float *qa,
                                                     const uint16_t *cache, const int *pos_p,
                                                     MlaDims d, int cap)
{
    extern __shared__ __align__(16) unsigned char smraw[];
    const int split = blockIdx.x, hg = blockIdx.y, b = blockIdx.z;
    // The position and the cache rows below it are read before the programmatic wait:
    // nothing in the kernels just before writes them (the position changes between steps,
    // row pos is written by the latent prep of this call, and every kernel before the one
    // still running has completed).
    const int pos = *pos_p;
    if (pos < 0 || pos >= cap) {                // the latent prep has raised K3D_EBOUND
        pdl_wait();
        pdl_trigger();
        return;
    }
    const int kvw = d.kvw;
    const int pitch = kvw + 8;                  // bf16 per smem row: 16 B pad, no conflicts
    const int hgn = min(kAHG, d.H - hg * kAHG);
    uint16_t *Qhi = reinterpret_cast<uint16_t *>(smraw);           // [16][pitch]
    uint16_t *Qlo = Qhi + kAHG * pitch;                             // [16][pitch]
    uint16_t *Ct = Qlo + kAHG * pitch;                              // [2][64][pitch]
    uint16_t *Phi = Ct + 2 * kATP * pitch;                          // [16][72]
    uint16_t *Plo = Phi + kAHG * 72;                                // [16][72]
    float *redm = reinterpret_cast<float *>(Plo + kAHG * 72);       // [4][16]
    float *reds = redm + 4 * kAHG;                                  // [4][16]
    float *mrow = reds + 4 * kAHG;                                  // [16]
    float *lrow = mrow + kAHG;                                      // [16]
    float *crow = lrow + kAHG;                                      // [16]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;

    const int n = pos + 1;
    const int per = (n + d.nsplit - 1) / d.nsplit;
    const int s0 = split * per, s1 = min(n, s0 + per);
    const uint16_t *cb = cache + (size_t)b * cap * kvw;
    const uint32_t ct_s = (uint32_t)__cvta_generic_to_shared(Ct);
    const bool early = s0 < s1 && min(s0 + kATP, s1) <= pos;     // tile 0 lies below row pos
    if (early) mla_stage_tile(ct_s, cb, s0, s1, kvw, pitch);
    pdl_wait();
    pdl_trigger();
    if (s0 < s1 && !early) mla_stage_tile(ct_s, cb, s0, s1, kvw, pitch);

    // Q as the bf16 hi/lo pair the absorb kernel wrote, rows of this CTA's heads (rows >=
    // hgn zero-filled): 16-byte cp.async chunks, all in flight at once (one group)
    {
        const uint16_t *qh0 = reinterpret_cast<const uint16_t *>(qa);
        const uint16_t *ql0 = qh0 + (size_t)gridDim.z * d.H * kvw;
        const int cpr = kvw / 8;                           // 16-byte chunks per row
        const uint32_t qhi_d = (uint32_t)__cvta_generic_to_shared(Qhi);
        const uint32_t qlo_d = (uint32_t)__cvta_generic_to_shared(Qlo);
        for (int i = tid; i < kAHG * cpr; i += 128) {
            const int hh = i / cpr, c = i % cpr;
            const bool ok = hh < hgn;
            const size_t row = ((size_t)b * d.H + hg * kAHG + (ok ? hh : 0)) * kvw + (size_t)c * 8;
            const uint32_t off = (uint32_t)(hh * pitch + c * 8) * 2u;
            cp16(qhi_d + off, qh0 + row, ok ? 16u : 0u);
            cp16(qlo_d + off, ql0 + row, ok ? 16u : 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    if (tid < kAHG) { mrow[tid] = -INFINITY; lrow[tid] = 0.f; }

    float acc[NT][4];
#pragma unroll
    for (int i = 0; i < NT; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    const uint32_t qhi_s = (uint32_t)__cvta_generic_to_shared(Qhi);
    const uint32_t qlo_s = (uint32_t)__cvta_generic_to_shared(Qlo);
    const uint32_t phi_s = (uint32_t)__cvta_generic_to_shared(Phi);
    const uint32_t plo_s = (uint32_t)__cvta_generic_to_shared(Plo);
    const int ksteps = kvw / 16;
    int buf = 0;
    for (int t0 = s0; t0 < s1; t0 += kATP, buf ^= 1) {
        // prefetch the next tile into the other buffer, then wait for this one
        if (t0 + kATP < s1) {
            mla_stage_tile(ct_s + (uint32_t)((buf ^ 1) * kATP * pitch) * 2u, cb, t0 + kATP, s1, kvw, pitch);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const uint32_t cbase = ct_s + (uint32_t)(buf * kATP * pitch) * 2u;

        // ---- scores: rows = positions 16*warp.., cols = 16 heads (two n8 tiles)
        // eight independent accumulator chains (n tile x hi/lo x even/odd k step) keep the
        // tensor pipe busy across the MMA latency; summed after the K loop
        float acc8[8][4];
#pragma unroll
        for (int j = 0; j < 8; j++) acc8[j][0] = acc8[j][1] = acc8[j][2] = acc8[j][3] = 0.f;
        const uint32_t a_row = cbase + (uint32_t)((warp * 16 + (lane & 15)) * pitch + (lane >> 4) * 8) * 2u;
        const uint32_t b_row = (uint32_t)((((lane >> 4) << 3) + (lane & 7)) * pitch + ((lane >> 3) & 1) * 8) * 2u;
        // even k steps into acc8[0..3], odd into acc8[4..7]; the pair is unrolled so that
        // every accumulator index is a constant (a run-time index puts acc8 in local memory)
        for (int ks = 0; ks < ksteps; ks += 2) {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                if (u == 1 && ks + 1 >= ksteps) break;
                uint32_t a[4], bh[4], bl[4];
                ldsm4(a, a_row + (ks + u) * 32u);
                ldsm4(bh, qhi_s + b_row + (ks + u) * 32u);
                ldsm4(bl, qlo_s + b_row + (ks + u) * 32u);
                mma_bf16(acc8[4 * u + 0], a, bh[0], bh[1]);
                mma_bf16(acc8[4 * u + 1], a, bh[2], bh[3]);
                mma_bf16(acc8[4 * u + 2], a, bl[0], bl[1]);
                mma_bf16(acc8[4 * u + 3], a, bl[2], bl[3]);
            }
        }
        float sc[2][4];
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int e = 0; e < 4; e++)
                sc[j][e] = (acc8[j][e] + acc8[2 + j][e]) + (acc8[4 + j][e] + acc8[6 + j][e]);
        // ---- softmax over the tile's positions, per head
        // sc[j][0..1]: position g, heads 8j + 2t4 + {0,1}; sc[j][2..3]: position g + 8
        const int pa = t0 + warp * 16 + g, pb = pa + 8;
        float v[2][4];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            v[j][0] = pa < s1 ? sc[j][0] * d.scale : -INFINITY;
            v[j][1] = pa < s1 ? sc[j][1] * d.scale : -INFINITY;
            v[j][2] = pb < s1 ? sc[j][2] * d.scale : -INFINITY;
            v[j][3] = pb < s1 ? sc[j][3] * d.scale : -INFINITY;
        }
        float mx[2][2];
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                float m = fmaxf(v[j][e], v[j][e + 2]);
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
                mx[j][e] = m;
            }
        if (g == 0) {
#pragma unroll
            for (int j = 0; j < 2; j++) {
                redm[warp * kAHG + 8 * j + 2 * t4] = mx[j][0];
                redm[warp * kAHG + 8 * j + 2 * t4 + 1] = mx[j][1];
            }
        }
        __syncthreads();
        if (tid < kAHG) {
            float m = mrow[tid];
            float tm = fmaxf(fmaxf(redm[tid], redm[kAHG + tid]), fmaxf(redm[2 * kAHG + tid], redm[3 * kAHG + tid]));
            const float mnew = fmaxf(m, tm);
            crow[tid] = (m == -INFINITY) ? 0.f : expf(m - mnew);
            mrow[tid] = mnew;
        }
        __syncthreads();
        float ps[2][2];
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int h = 8 * j + 2 * t4 + e;
                const float mnew = mrow[h];
                const float p0 = (v[j][e] == -INFINITY) ? 0.f : expf(v[j][e] - mnew);
                const float p1 = (v[j][e + 2] == -INFINITY) ? 0.f : expf(v[j][e + 2] - mnew);
                // P[h][position] as bf16 hi + lo (A operand of the ctx MMA, K = position)
                const int ra = warp * 16 + g, rb = ra + 8;
                const uint16_t h0 = f32_to_bf16_bits(p0), h1 = f32_to_bf16_bits(p1);
                Phi[h * 72 + ra] = h0;
                Phi[h * 72 + rb] = h1;
                Plo[h * 72 + ra] = f32_to_bf16_bits(p0 - bf16_to_f32(h0));
                Plo[h * 72 + rb] = f32_to_bf16_bits(p1 - bf16_to_f32(h1));
                float sum = p0 + p1;
                sum += __shfl_xor_sync(0xffffffffu, sum, 4);
                sum += __shfl_xor_sync(0xffffffffu, sum, 8);
                sum += __shfl_xor_sync(0xffffffffu, sum, 16);
                ps[j][e] = sum;
            }
        if (g == 0) {
#pragma unroll
            for (int j = 0; j < 2; j++) {
                reds[warp * kAHG + 8 * j + 2 * t4] = ps[j][0];
                reds[warp * kAHG + 8 * j + 2 * t4 + 1] = ps[j][1];
            }
        }
        __syncthreads();
        if (tid < kAHG)
            lrow[tid] = lrow[tid] * crow[tid] + ((reds[tid] + reds[kAHG + tid]) + (reds[2 * kAHG + tid] + reds[3 * kAHG + tid]));
        // ---- ctx: rows = heads (g, g + 8), cols = this warp's kv_lora / 4 slice
        {
            const float c0 = crow[g], c1 = crow[g + 8];
#pragma unroll
            for (int i = 0; i < NT; i++) {
                acc[i][0] *= c0; acc[i][1] *= c0; acc[i][2] *= c1; acc[i][3] *= c1;
            }
            const uint32_t pa_row = (uint32_t)((lane & 15) * 72 + (lane >> 4) * 8) * 2u;
            // B from C[p][j] (row-major K x N): ldmatrix.trans, lanes 0-15 rows k0.., 16-31
            // the next n8 tile
            const int jb = warp * (NT * 8);
            const uint32_t b_row_t = cbase + (uint32_t)(((lane & 15)) * pitch + jb + (lane >> 4) * 8) * 2u;
#pragma unroll
            for (int kk = 0; kk < kATP / 16; kk++) {
                uint32_t ah[4], al[4];
                ldsm4(ah, phi_s + pa_row + kk * 32u);
                ldsm4(al, plo_s + pa_row + kk * 32u);
#pragma unroll
                for (int i = 0; i < NT; i += 2) {
                    uint32_t bb[4];
                    ldsm4t(bb, b_row_t + (uint32_t)(kk * 16 * pitch + i * 8) * 2u);
                    mma_bf16(acc[i], ah, bb[0], bb[1]);
                    mma_bf16(acc[i + 1], ah, bb[2], bb[3]);
                    mma_bf16(acc[i], al, bb[0], bb[1]);
                    mma_bf16(acc[i + 1], al, bb[2], bb[3]);
                }
            }
        }
        __syncthreads();     // the buffer and P are reused by the next tile
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");   // a split without positions staged Q only
    // ---- partial outputs of this split
    const int jb = warp * (NT * 8);
    const size_t stride = (size_t)d.kv_lora + 2;
#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        const int h = g + 8 * rr;
        if (h < hgn) {
            float *dst = part + (((size_t)b * d.H + hg * kAHG + h) * d.nsplit + split) * stride;
#pragma unroll
            for (int i = 0; i < NT; i++) {
                const int j = jb + 8 * i + 2 * t4;     // even; rows start 8-byte aligned
                *reinterpret_cast<float2 *>(dst + j) = make_float2(acc[i][2 * rr], acc[i][2 * rr + 1]);
            }
        }
    }
    if (tid < hgn) {
        float *dst = part + (((size_t)b * d.H + hg * kAHG + tid) * d.nsplit + split) * stride;
        dst[d.kv_lora] = mrow[tid];
        dst[d.kv_lora + 1] = lrow[tid];
    }
}

static size_t mla_attn_smem(int kvw)
{
    const size_t pitch = (size_t)kvw + 8;
    return (2 * kAHG * pitch + 2 * kATP * pitch + 2 * kAHG * 72) * 2 + (8 * kAHG + 3 * kAHG) * 4;
}

// grid (H, vh / 32, B), 256 threads: merge the splits of head h into ctx (each CTA of the
// head repeats this small step), then 32 rows of o = W_uv ctx, times sigmoid(gate).
// heads [B][H*vh]. The W_uv rows are loaded before the programmatic wait (weights), and
// after it every partial load the merge needs first (m and l of one split per thread, the
// first kMP ctx partials of the thread's column pair) is issued before any reduction.
static const int kMP = 40;
__global__ void __launch_bounds__(256, 2) k_mla_merge(float *heads, const float *part,
                                                   const uint16_t *kv_b, const float *gate,
                                                   const int *pos_p, MlaDims d, int cap)
{
    extern __shared__ __align__(16) float cx[];   // [kv_lora], then W_uv rows [32][kv_lora] bf16
    __shared__ float wsc[256 + 2 * 256];   // split weights, then partial column sums
    __shared__ float red[8];
    const int h = blockIdx.x, rb = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // this CTA's 32 rows of W_uv into shared memory (16-byte cp.async chunks, issued before
    // the programmatic wait: weights), 4 rows per warp later
    const size_t kvd = (size_t)(d.qn + d.vh);
    const uint16_t *rows0 = kv_b + ((size_t)h * kvd + d.qn + rb * 32) * d.kv_lora;
    uint16_t *wsm = reinterpret_cast<uint16_t *>(cx + d.kv_lora);
    {
        const uint32_t w_d = (uint32_t)__cvta_generic_to_shared(wsm);
        const int nchunk = 32 * d.kv_lora / 8;
        for (int i = tid; i < nchunk; i += blockDim.x) cp16(w_d + 16u * i, rows0 + (size_t)i * 8, 16u);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // the output gate of this warp's rows (written by the projection GEMV, long before)
    float gv[4] = {0.f, 0.f, 0.f, 0.f};
    if (gate && lane == 0) {
#pragma unroll
        for (int r = 0; r < 4; r++)
            gv[r] = gate[(size_t)b * d.H * d.vh + (size_t)h * d.vh + rb * 32 + warp * 4 + r];
    }
    pdl_wait();
    pdl_trigger();
    const int pos = *pos_p;
    if (pos < 0 || pos >= cap) {
        for (int r = tid; r < 32; r += blockDim.x)
            heads[(size_t)b * d.H * d.vh + (size_t)h * d.vh + rb * 32 + r] = 0.f;
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        return;
    }
    const float *pp = part + ((size_t)b * d.H + h) * d.nsplit * (d.kv_lora + 2);
    const int stride = d.kv_lora + 2;
    // the splits that own positions (a split past the end wrote nothing); ns <= 256
    const int n = pos + 1, per = (n + d.nsplit - 1) / d.nsplit;
    const int ns = min(d.nsplit, (n + per - 1) / per);
    const int np2 = d.kv_lora / 2;            // 256 for kv_lora 512
    const int nsub = blockDim.x / np2;        // 1 (kv_lora 512) .. 4 (kv_lora 128)
    const int cp = tid % np2, sub = tid / np2;
    const float ms = tid < ns ? pp[tid * stride + d.kv_lora] : -INFINITY;
    const float ls = tid < ns ? pp[tid * stride + d.kv_lora + 1] : 0.f;
    float2 pv[kMP];
#pragma unroll
    for (int k = 0; k < kMP; k++) {
        const int sp = sub + k * nsub;
        pv[k] = (sub < nsub && sp < ns) ? *reinterpret_cast<const float2 *>(pp + (size_t)sp * stride + 2 * cp)
                                        : make_float2(0.f, 0.f);
    }
    float M = warp_max(ms);
    if (lane == 0) red[warp] = M;
    __syncthreads();
    M = red[0];
    for (int i = 1; i < 8; i++) M = fmaxf(M, red[i]);
    __syncthreads();
    float L = 0.f;
    if (tid < ns) {
        const float w = (ms == -INFINITY) ? 0.f : expf(ms - M);
        wsc[tid] = w;
        L = w * ls;
    }
    L = warp_sum(L);
    if (lane == 0) red[warp] = L;
    __syncthreads();
    float Ls = 0.f;
    for (int i = 0; i < 8; i++) Ls += red[i];
    const float invL = 1.0f / Ls;
    // ctx = sum_s w_s part_s / L: thread t takes float2 column pair t % np2 over the
    // splits congruent to t / np2 (mod nsub), then the nsub partial sums are added in a
    // fixed order through shared memory
    {
        float2 a = make_float2(0.f, 0.f);
        if (sub < nsub) {
#pragma unroll
            for (int k = 0; k < kMP; k++) {
                const int sp = sub + k * nsub;
                if (sp < ns) {
                    a.x = fmaf(wsc[sp], pv[k].x, a.x);
                    a.y = fmaf(wsc[sp], pv[k].y, a.y);
                }
            }
#pragma unroll 8
            for (int sp = sub + kMP * nsub; sp < ns; sp += nsub) {
                const float2 v = *reinterpret_cast<const float2 *>(pp + (size_t)sp * stride + 2 * cp);
                a.x = fmaf(wsc[sp], v.x, a.x);
                a.y = fmaf(wsc[sp], v.y, a.y);
            }
        }
        if (nsub == 1) {
            cx[2 * cp] = a.x * invL;
            cx[2 * cp + 1] = a.y * invL;
        } else {
            float2 *pa = reinterpret_cast<float2 *>(wsc + 256);   // [nsub][np2], after the weights
            if (sub < nsub) pa[sub * np2 + cp] = a;
            __syncthreads();
            if (tid < np2) {
                float2 t2 = pa[tid];
                for (int k = 1; k < nsub; k++) { t2.x += pa[k * np2 + tid].x; t2.y += pa[k * np2 + tid].y; }
                cx[2 * tid] = t2.x * invL;
                cx[2 * tid + 1] = t2.y * invL;
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // 4 rows per warp, lane l takes 8-element chunks l, l + 32, ... of each row
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint16_t *wr = wsm + (size_t)warp * 4 * d.kv_lora;
    for (int j0 = lane * 8; j0 < d.kv_lora; j0 += 256) {
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const uint4 wv = *reinterpret_cast<const uint4 *>(wr + (size_t)r * d.kv_lora + j0);
            const uint32_t u[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int m = 0; m < 4; m++) {
                acc[r] = fmaf(__uint_as_float(u[m] << 16), cx[j0 + 2 * m], acc[r]);
                acc[r] = fmaf(__uint_as_float(u[m] & 0xffff0000u), cx[j0 + 2 * m + 1], acc[r]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const float v = warp_sum(acc[r]);
        if (lane == 0) {
            const size_t o = (size_t)b * d.H * d.vh + (size_t)h * d.vh + rb * 32 + warp * 4 + r;
            heads[o] = gate ? v * (1.0f / (1.0f + expf(-gv[r]))) : v;
        }
    }
}

static size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

struct MlaWs {
    float *ql, *c, *gate, *q, *qa, *part, *heads;
    size_t total;
};

// Splits of the positions: one wave of attention CTAs over the SMs (one CTA per SM fits).
static int mla_nsplit(int B, int H, int cap)
{
    const int per_b = (H + kAHG - 1) / kAHG;
    const int want = sm_count() > 0 ? sm_count() : 148;
    int ns = (want + B * per_b - 1) / (B * per_b);
    const int max_ns = (cap + kATP - 1) / kATP;
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

// The RoPE table of (theta, qr, cap), built on first use and kept for the process: a
// decode step then reads one row instead of evaluating pow/cos/sin in double. The first
// call for a shape allocates, so it must not be inside a stream capture.
static const float2 *rope_table(float theta, int qr, int cap, cudaStream_t st)
{
    struct Tab { float theta; int qr, cap; float2 *p; };
    static std::vector<Tab> tabs;
    for (const Tab &t : tabs)
        if (t.theta == theta && t.qr == qr && t.cap >= cap) return t.p;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs != cudaStreamCaptureStatusNone) {
        fail(K3D_EINVAL, "mla: first decode of a RoPE shape (theta %g, rope %d, cap %d) inside a "
                         "stream capture; run one step eagerly first", theta, qr, cap);
        return nullptr;
    }
    float2 *p = nullptr;
    const size_t n = (size_t)cap * (qr / 2);
    if (cudaMalloc(&p, n * sizeof(float2)) != cudaSuccess) {
        cudaGetLastError();
        fail(K3D_ENOMEM, "mla: RoPE table of %zu entries", n);
        return nullptr;
    }
    k_rope_table<<<(int)((n + 255) / 256), 256, 0, st>>>(p, qr, cap, theta);
    note_launch();
    if (check_launch("rope table")) { cudaFree(p); return nullptr; }
    tabs.push_back({theta, qr, cap, p});
    return p;
}

int mla_decode(float *out, const float *x, const K3dMlaW *w, const K3dMlaShape *s, int B,
               uint16_t *cache, int cap, const int *pos, int accumulate, void *ws,
               cudaStream_t st, const NormIn *ni = nullptr)
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
            K3_TRY(gemv_bf16_multi(s->out_gate ? 3 : 2, Ws, Ys, rows, x, s->hidden, B, st, ni));
        } else {
            if (ni) {
                x = norm_to_scratch(x, *ni, s->hidden, B, st);
                if (!x) return k3d_status();
            }
            K3_TRY(gemv_bf16(L.ql, x, w->q_a, s->hidden, s->q_lora, B, 0, st));
            K3_TRY(gemv_bf16(L.c, x, w->kv_a, s->hidden, d.kvw, B, 0, st));
            if (s->out_gate) K3_TRY(gemv_bf16(L.gate, x, w->g, s->hidden, d.H * d.vh, B, 0, st));
        }
    }
    prof_end("mla.proj_in");
    prof_begin("mla.core");
    const float2 *rope_tab = nullptr;
    if (d.theta > 0.f) {
        rope_tab = rope_table(d.theta, d.qr, cap, st);
        if (!rope_tab) return k3d_status();
    }
    // Up to four tokens: q_b takes the raw q_lora activation and applies q_a_norm as it loads
    // it, and the latent half of k_mla_prep rides in the absorb launch; larger batches run
    // k_mla_prep first (their q_b is the tensor-core GEMM).
    const bool fused_prep = B <= 4;
    if (fused_prep) {
        const NormIn qn{w->q_a_norm, d.eps};
        const uint16_t *Wq[1] = {w->q_b};
        float *Yq[1] = {L.q};
        const int rq[1] = {d.H * d.qh};
        K3_TRY(gemv_bf16_multi(1, Wq, Yq, rq, L.ql, s->q_lora, B, st, &qn));
    } else {
        launch_pdl(k_mla_prep, dim3(B), dim3(256), 0, st, L.ql, L.c, cache, rope_tab, w->q_a_norm, w->kv_a_norm, pos, d, cap);
        note_launch();
        K3_TRY(check_launch("mla prep"));
        K3_TRY(gemv_bf16(L.q, L.ql, w->q_b, s->q_lora, d.H * d.qh, B, 0, st));
    }
    launch_pdl(k_mla_absorb, dim3(d.H, d.kv_lora / 128 + (fused_prep ? 1 : 0), B), dim3(16, 8), 0, st, L.qa, L.q,
               w->kv_b, rope_tab, pos, d, cap, L.c, cache, w->kv_a_norm, fused_prep ? 1 : 0);
    note_launch();
    K3_TRY(check_launch("mla absorb"));
    {
        static unsigned long long init = 0;   // one bit per device
        if (!(init & dev_bit())) {
            allow_smem_max(k_mla_attn_tc<4>);
            allow_smem_max(k_mla_attn_tc<8>);
            allow_smem_max(k_mla_attn_tc<12>);
            allow_smem_max(k_mla_attn_tc<16>);
            init |= dev_bit();
        }
        const size_t smem = mla_attn_smem(d.kvw);
        const dim3 grid(d.nsplit, (d.H + kAHG - 1) / kAHG, B);
        switch (d.kv_lora / 32) {
        case 4: launch_pdl(k_mla_attn_tc<4>, dim3(grid), dim3(128), smem, st, L.part, L.qa, cache, pos, d, cap); break;
        case 8: launch_pdl(k_mla_attn_tc<8>, dim3(grid), dim3(128), smem, st, L.part, L.qa, cache, pos, d, cap); break;
        case 12: launch_pdl(k_mla_attn_tc<12>, dim3(grid), dim3(128), smem, st, L.part, L.qa, cache, pos, d, cap); break;
        default: launch_pdl(k_mla_attn_tc<16>, dim3(grid), dim3(128), smem, st, L.part, L.qa, cache, pos, d, cap); break;
        }
        note_launch();
        K3_TRY(check_launch("mla attn"));
    }
    launch_pdl(k_mla_merge, dim3(d.H, d.vh / 32, B), dim3(256), (size_t)d.kv_lora * 4 + 32 * (size_t)d.kv_lora * 2, st, 
        L.heads, L.part, w->kv_b, s->out_gate ? L.gate : nullptr, pos, d, cap);
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

static int mla_decode_checked(float *out, const float *x, const NormIn *ni, const K3dMlaW *w,
                              const K3dMlaShape *s, int B, uint16_t *cache, int cap,
                              const int *pos, int accumulate, void *ws, size_t ws_bytes)
{
    K3_TRY(ensure_ctx());
    if (!out || !x || !w || !s || !cache || !pos || !ws)
        return fail(K3D_EINVAL, "k3d_mla_decode null pointer");
    if (!w->q_a || !w->q_b || !w->kv_a || !w->kv_b || !w->o || !w->q_a_norm || !w->kv_a_norm ||
        (s->out_gate && !w->g))
        return fail(K3D_EINVAL, "k3d_mla_decode weight missing");
    if (s->n_heads % 8 || s->kv_lora > 512 || s->kv_lora % 128 || s->qk_rope % 2 ||
        s->q_lora > 2048 || s->q_lora < 1 ||
        ((s->kv_lora + s->qk_rope) % 16) || s->qk_nope + s->qk_rope > 256 || s->hidden % 8 ||
        s->v_head % 32 || s->qk_rope > 256)
        return fail(K3D_EINVAL, "k3d_mla_decode: n_heads %% 8, kv_lora a multiple of 128 up to "
                                "512, even rope, (kv_lora + rope) %% 16, nope + rope <= 256, "
                                "v_head %% 32, q_lora <= 2048");
    if (ws_bytes < k3d_mla_ws_bytes(s, B, cap)) return fail(K3D_EINVAL, "k3d_mla_decode workspace");
    return mla_decode(out, x, w, s, B, cache, cap, pos, accumulate, ws, stream(), ni);
}

int k3d_mla_decode(float *out, const float *x, const K3dMlaW *w, const K3dMlaShape *s, int B,
                   uint16_t *cache, int cap, const int *pos, int accumulate, void *ws,
                   size_t ws_bytes)
{
    return mla_decode_checked(out, x, nullptr, w, s, B, cache, cap, pos, accumulate, ws, ws_bytes);
}

int k3d_mla_decode_normed(float *out, const float *x, const float *norm_w, float eps,
                          const K3dMlaW *w, const K3dMlaShape *s, int B, uint16_t *cache,
                          int cap, const int *pos, int accumulate, void *ws, size_t ws_bytes)
{
    if (!norm_w) return fail(K3D_EINVAL, "k3d_mla_decode_normed: null norm weights");
    const NormIn ni{norm_w, eps};
    return mla_decode_checked(out, x, &ni, w, s, B, cache, cap, pos, accumulate, ws, ws_bytes);
}

}  // extern "C"
