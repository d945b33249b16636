// k3_gemv_stream.cu -- the bf16 decode GEMVs (plain / accumulate, several matrices sharing
// x, fused SwiGLU pairs, LM head with argmax), streamed through shared memory by bulk copies.
//
// Same arithmetic as the register-staged kernels in k3_gemv.cu (each lane sums its 8-element
// chunks of a row with packed f32x2 FMAs, the warp adds the lanes; fp32 accumulation within
// the 1e-3 relative contract of k3_matmul_bf16, k3_ops.c:1108-1213), organised for HBM:
//   * one CTA per SM with a contiguous, evenly split range of "units" (a row, or a gate/up
//     row pair for SwiGLU), so no SM is left with a partial last wave;
//   * one producer thread streams the range as stages of R consecutive whole rows (about
//     32 KB, never crossing a matrix boundary), each stage ONE bulk copy of contiguous
//     memory (two for a SwiGLU pair: gate rows and up rows) completing on an mbarrier, into
//     a ring of up to 8 stages; large copies keep 100-200 KB per SM in flight (many small
//     copies do not: the copy engine then holds too few bytes in flight); the weights do
//     not depend on earlier kernels, so the first stages are requested before the
//     programmatic-dependent-launch wait;
//   * ring slot s belongs to consumer warp s, which takes every stage of its slot in order
//     (so each warp waits only for the next phase of its own barriers) and finishes each
//     row of the stage (warp sum, epilogue): no cross-warp reduction; x is staged once per
//     CTA in shared memory.
// Every wait is bounded (K3D_ETIMEOUT in the device error flag, then all roles stop); the
// producer waits for its own copies before the CTA exits.
#include <algorithm>

#include "k3_bulk.cuh"
#include "k3_gemv.cuh"
#include "k3_ops.cuh"

namespace k3 {
namespace gstream {

constexpr int kWarps = 8;                       // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;     // + one producer warp
constexpr int kStageTarget = 32768;             // bytes of weights per stage (at least a unit)
constexpr int kMaxStages = 8;
constexpr int kHeader = 1024;                   // barriers and flags ahead of the stages

enum { PLAIN = 0, SWIGLU = 1, ARGMAX = 2 };

struct Args {
    const uint16_t *W[8];     // PLAIN/ARGMAX: segment matrices; SWIGLU: W[0] gate, W[1] up
    float *y[8];              // PLAIN: per segment [T][rows]; SWIGLU: y[0] act [T][inter];
                              // ARGMAX: y[0] logits [T][rows] or null
    int start[9];             // unit prefix over segments (SWIGLU: start[1] = inter)
    int nseg;
    const float *x;           // [T][in]
    int in, T;
    int accumulate;           // PLAIN: y += W x
    unsigned long long *key;  // ARGMAX: [T]
    const float *norm_w;      // non-null: x is a raw residual, normalised on load (RMSNorm
    float norm_eps;           //   with these weights, k3_rmsnorm's arithmetic; in <= 8192)
    int stages;               // ring depth
    int R;                    // units per stage
    int stage_bytes;          // R * rows-per-unit * in * 2
};

// x for the consumer threads only (the producer warp is already streaming): up to 8 loads
// in flight per thread, stored in the swizzled layout bf16_chunk_dot reads.
__device__ __forceinline__ void stage_x_part(float4 *xs, const float *x, int in, int tid, int nt)
{
    const int nf4 = in >> 2;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    for (int f0 = tid; f0 < nf4; f0 += 8 * nt) {
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (f0 + i * nt < nf4) v[i] = __ldg(x4 + f0 + i * nt);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int f = f0 + i * nt;
            if (f < nf4) xs[xb_idx(f >> 1, f & 1)] = v[i];
        }
    }
}

// Stage i of a CTA's range: the next min(R, rest of the range, rest of the segment)
// units. Producer and consumers walk the same sequence.
struct StageWalk {
    int u, seg;
    __device__ __forceinline__ int next(const Args &A, int u1, int &ustart, int &sg)
    {
        while (seg + 1 < A.nseg && u >= A.start[seg + 1]) seg++;
        ustart = u;
        sg = seg;
        const int n = min(A.R, min(u1 - u, A.start[seg + 1] - u));
        u += n;
        return n;
    }
};

template <int MODE, int NT>
__global__ void __launch_bounds__(kThreads, 1) k_gemv_stream(Args A)
{
    extern __shared__ unsigned char smraw[];
    const uint32_t raw = bulk::saddr(smraw);
    const uint32_t base = (raw + 127u) & ~127u;
    unsigned char *gb = smraw + (base - raw);
    const int S = A.stages;
    const uint32_t b_full = base;                   // [S] x 8
    const uint32_t b_empty = base + 8 * kMaxStages;
    volatile int *abort = reinterpret_cast<volatile int *>(gb + 16 * kMaxStages);
    const uint32_t stage0 = base + kHeader;
    const unsigned char *gstage0 = gb + kHeader;
    float4 *xs = reinterpret_cast<float4 *>(gb + kHeader + (size_t)S * A.stage_bytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    constexpr int RPU = MODE == SWIGLU ? 2 : 1;     // rows per unit
    const int in = A.in;
    const size_t rowb = (size_t)in * 2;
    const int U = A.start[A.nseg];
    const int u0 = (int)((long long)blockIdx.x * U / gridDim.x);
    const int u1 = (int)((long long)(blockIdx.x + 1) * U / gridDim.x);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            bulk::mbar_init(b_full + 8 * s, 1);
            bulk::mbar_init(b_empty + 8 * s, 1);      // the slot's warp, once per stage
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kWarps) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            StageWalk wk{u0, 0};
            int i = 0;
            while (wk.u < u1) {
                int us, sg;
                const int n = wk.next(A, u1, us, sg);
                const int st = i % S;
                if (i == S) pdl_wait();    // bounded waits start once the kernel before has completed
                if (i >= S && !bulk::mbar_wait(b_empty + 8 * st, ((i / S) - 1) & 1, abort, K3_SITE_GEMV,
                                               1000 + MODE, i))
                    break;
                const uint32_t fb = b_full + 8 * st;
                const uint32_t dst = stage0 + (uint32_t)st * (uint32_t)A.stage_bytes;
                const uint32_t bytes = (uint32_t)((size_t)n * rowb);
                // self-check: the stage lies in this CTA's ring and the rows in their matrix;
                // a stage that fails is completed without copies (its results are wrong, and
                // the device error flag says so) rather than copied out of bounds
                const bool ok = n >= 1 && n <= A.R && st < S && sg >= 0 && sg < A.nseg &&
                                us >= A.start[sg] && us + n <= A.start[sg + 1] &&
                                (size_t)n * rowb * RPU <= (size_t)A.stage_bytes;
                if (!ok) {
                    k3_raise(K3D_EBOUND, K3_SITE_GEMV);
                    bulk::mbar_arrive(fb);
                    i++;
                    continue;
                }
                bulk::mbar_expect_tx(fb, bytes * RPU);
                if (MODE == SWIGLU) {
                    bulk::g2s(dst, A.W[0] + (size_t)us * in, bytes, fb);
                    bulk::g2s(dst + (uint32_t)((size_t)A.R * rowb), A.W[1] + (size_t)us * in, bytes, fb);
                } else {
                    bulk::g2s(dst, A.W[sg] + (size_t)(us - A.start[sg]) * in, bytes, fb);
                }
                i++;
            }
            // no copy may still be landing when the CTA exits: wait (bounded) for the last
            // use of every stage (already complete unless the consumers stopped early)
            for (int h = max(0, i - S); h < i; h++) {
                const uint32_t fb = b_full + 8 * (h % S);
                const long long t0 = clock64();
                while (!bulk::mbar_try(fb, (h / S) & 1)) {
                    if (clock64() - t0 > bulk::kSpinLimit) { k3_raise(K3D_ETIMEOUT, K3_SITE_GEMV); break; }
                }
            }
        }
        return;
    }

    // -------------------------------------------------------------------- consumers
    const int nf4 = in >> 2;
    constexpr int nt = kWarps * 32;
    // RMSNorm on load: this thread's norm weights (float4 f = tid + k * nt) are constants,
    // loaded before the programmatic wait
    float4 wn[8];
    if (A.norm_w) {
#pragma unroll
        for (int k = 0; k < 8; k++)
            if ((int)threadIdx.x + k * nt < nf4)
                wn[k] = __ldg(reinterpret_cast<const float4 *>(A.norm_w) + threadIdx.x + k * nt);
    }
    pdl_wait();
    pdl_trigger();
    for (int t = 0; t < NT; t++)
        if (t < A.T) stage_x_part(xs + (size_t)t * nf4, A.x + (size_t)t * in, in, threadIdx.x, nt);
    if (A.norm_w) {
        // x = (w * x) * inv_rms(x) per token, with the sum of squares in double as k3_rmsnorm
        // does; each thread rescales the float4s it staged
        __shared__ double red[kWarps][4];
#pragma unroll
        for (int t = 0; t < NT; t++) {
            if (t >= A.T) break;
            double ss = 0.0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int f = threadIdx.x + k * nt;
                if (f < nf4) {
                    const float4 v = xs[(size_t)t * nf4 + xb_idx(f >> 1, f & 1)];
                    ss = fma((double)v.x, (double)v.x, ss);
                    ss = fma((double)v.y, (double)v.y, ss);
                    ss = fma((double)v.z, (double)v.z, ss);
                    ss = fma((double)v.w, (double)v.w, ss);
                }
            }
            ss = warp_sum_d(ss);
            if (lane == 0) red[warp][t] = ss;
        }
        asm volatile("bar.sync 1, %0;" :: "n"(nt) : "memory");
#pragma unroll
        for (int t = 0; t < NT; t++) {
            if (t >= A.T) break;
            double tot = 0.0;
            for (int w = 0; w < kWarps; w++) tot += red[w][t];
            const float inv = (float)(1.0 / sqrt(tot / (double)in + (double)A.norm_eps));
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const int f = threadIdx.x + k * nt;
                if (f < nf4) {
                    float4 &v = xs[(size_t)t * nf4 + xb_idx(f >> 1, f & 1)];
                    v.x = __fmul_rn(__fmul_rn(wn[k].x, v.x), inv);
                    v.y = __fmul_rn(__fmul_rn(wn[k].y, v.y), inv);
                    v.z = __fmul_rn(__fmul_rn(wn[k].z, v.z), inv);
                    v.w = __fmul_rn(__fmul_rn(wn[k].w, v.w), inv);
                }
            }
        }
    }
    asm volatile("bar.sync 1, %0;" :: "n"(kWarps * 32) : "memory");

    const int nch = in >> 3;                        // 8-element chunks of a row
    unsigned long long best[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) best[t] = 0ull;
    // ring slot s belongs to warp s (S <= 8): the warp takes every stage of its slot, in
    // order, so it only ever waits for the next phase of its own barriers (a parity wait
    // cannot tell a phase from the one two further on)
    StageWalk wk{u0, 0};
    int i = 0;
    while (wk.u < u1) {
        int us, sg;
        const int n = wk.next(A, u1, us, sg);
        const int st = i % S;
        if (st == warp) {
            if (!bulk::mbar_wait(b_full + 8 * st, (i / S) & 1, abort, K3_SITE_GEMV, 2000 + MODE * 10 + warp, i))
                break;
            for (int q = 0; q < n; q++) {
                const unsigned char *ur = gstage0 + (size_t)st * A.stage_bytes + (size_t)q * rowb;
                float2 acc[NT][RPU];
#pragma unroll
                for (int t = 0; t < NT; t++)
#pragma unroll
                    for (int r = 0; r < RPU; r++) acc[t][r] = make_float2(0.f, 0.f);
#pragma unroll 4
                for (int c = lane; c < nch; c += 32) {
#pragma unroll
                    for (int r = 0; r < RPU; r++) {
                        const uint4 w = *reinterpret_cast<const uint4 *>(ur + (size_t)r * A.R * rowb + 16 * (size_t)c);
#pragma unroll
                        for (int t = 0; t < NT; t++)
                            if (t < A.T) acc[t][r] = bf16_chunk_dot(w, xs + (size_t)t * nf4, c, acc[t][r]);
                    }
                }
                const int u = us + q;
                const int lr = u - A.start[sg];
                if (u < u0 || u >= u1 || lr < 0 || lr >= A.start[sg + 1] - A.start[sg]) {
                    if (lane == 0) k3_raise(K3D_EBOUND, K3_SITE_GEMV);
                    continue;
                }
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    if (t >= A.T) break;
                    const float v0 = warp_sum(acc[t][0].x + acc[t][0].y);
                    if (MODE == SWIGLU) {
                        const float v1 = warp_sum(acc[t][RPU - 1].x + acc[t][RPU - 1].y);
                        if (lane == 0) A.y[0][(size_t)t * U + u] = silu_f(v0) * v1;
                    } else if (MODE == PLAIN) {
                        if (lane == 0) {
                            float *dst = A.y[sg] + (size_t)t * (A.start[sg + 1] - A.start[sg]) + lr;
                            *dst = A.accumulate ? *dst + v0 : v0;
                        }
                    } else if (lane == 0) {
                        if (A.y[0]) A.y[0][(size_t)t * U + u] = v0;
                        uint32_t ob = __float_as_uint(v0);
                        ob = (ob & 0x80000000u) ? ~ob : (ob | 0x80000000u);
                        const unsigned long long k =
                            ((unsigned long long)ob << 32) | (unsigned long long)(0xffffffffu - (uint32_t)u);
                        if (v0 == v0 && k > best[t]) best[t] = k;
                    }
                }
            }
            // every row of the stage has been read: the slot may be refilled
            __syncwarp();
            if (lane == 0) bulk::mbar_arrive(b_empty + 8 * st);
        }
        i++;
    }
    if (MODE == ARGMAX && lane == 0) {
#pragma unroll
        for (int t = 0; t < NT; t++)
            if (t < A.T && best[t]) atomicMax(A.key + t, best[t]);
    }
}

}  // namespace gstream

using namespace gstream;

// Streams when the shapes allow (in % 8 == 0 and >= 512, 16-byte aligned matrices and x,
// x of all T tokens plus at least 4 stages within the shared-memory limit); returns 1 when
// launched, 0 when the caller should use the register-staged kernels.
template <int MODE>
static int stream_launch(Args &A, cudaStream_t st)
{
    if (A.T < 1 || A.T > 4 || (A.in % 8) != 0 || A.in < 512) return 0;
    if (A.norm_w && (A.in > 8 * 4 * kWarps * 32 || ((uintptr_t)A.norm_w & 15u) != 0)) return 0;
    if (((uintptr_t)A.x & 15u) != 0) return 0;
    const int nw = MODE == SWIGLU ? 2 : A.nseg;
    for (int i = 0; i < nw; i++)
        if (((uintptr_t)A.W[i] & 15u) != 0) return 0;
    const size_t xbytes = (size_t)A.T * A.in * sizeof(float);
    const size_t limit = 226 * 1024;    // the opt-in maximum less room for static shared memory
    const size_t unitb = (size_t)(MODE == SWIGLU ? 2 : 1) * A.in * 2;
    A.R = (int)std::max<size_t>(1, kStageTarget / unitb);
    A.stage_bytes = (int)((size_t)A.R * unitb);
    if (xbytes + kHeader + 128 + 2 * (size_t)A.stage_bytes > limit) return 0;
    const int stages = (int)std::min<size_t>(kMaxStages, (limit - xbytes - kHeader - 128) / A.stage_bytes);
    A.stages = stages;
    const size_t smem = kHeader + 128 + (size_t)stages * A.stage_bytes + xbytes;
    const int U = A.start[A.nseg];
    const int grid = std::max(1, std::min(sm_count(), U));
#define K3_STREAM_LAUNCH(NT)                                                              \
    do {                                                                                  \
        static unsigned long long init = 0;   /* one bit per device */                        \
        if (!(init & dev_bit())) { allow_smem_max(k_gemv_stream<MODE, NT>); init |= dev_bit(); } \
        launch_pdl(k_gemv_stream<MODE, NT>, dim3(grid), dim3(kThreads), smem, st, A);     \
    } while (0)
    switch (A.T) {
        case 1: K3_STREAM_LAUNCH(1); break;
        case 2: K3_STREAM_LAUNCH(2); break;
        default: K3_STREAM_LAUNCH(4); break;
    }
#undef K3_STREAM_LAUNCH
    note_launch();
    return 1;
}

int gemv_stream_multi(int nseg, const uint16_t *const *W, float *const *y, const int *rows,
                      const float *x, int in, int T, int accumulate, cudaStream_t st,
                      const NormIn *ni)
{
    if (nseg < 1 || nseg > 8) return 0;
    Args A{};
    A.nseg = nseg;
    A.start[0] = 0;
    for (int i = 0; i < nseg; i++) {
        A.W[i] = W[i];
        A.y[i] = y[i];
        A.start[i + 1] = A.start[i] + rows[i];
    }
    A.x = x;
    A.in = in;
    A.T = T;
    A.accumulate = accumulate;
    A.norm_w = ni ? ni->w : nullptr;
    A.norm_eps = ni ? ni->eps : 0.0f;
    return stream_launch<PLAIN>(A, st);
}

int gemv_stream_swiglu(float *act, const float *x, const uint16_t *Wg, const uint16_t *Wu,
                       int in, int inter, int T, cudaStream_t st)
{
    Args A{};
    A.nseg = 1;
    A.W[0] = Wg;
    A.W[1] = Wu;
    A.y[0] = act;
    A.start[0] = 0;
    A.start[1] = inter;
    A.x = x;
    A.in = in;
    A.T = T;
    return stream_launch<SWIGLU>(A, st);
}

int gemv_stream_argmax(float *y, unsigned long long *key, const float *x, const uint16_t *W,
                       int in, int out, int T, cudaStream_t st, const NormIn *ni)
{
    Args A{};
    A.nseg = 1;
    A.W[0] = W;
    A.y[0] = y;
    A.start[0] = 0;
    A.start[1] = out;
    A.x = x;
    A.in = in;
    A.T = T;
    A.key = key;
    A.norm_w = ni ? ni->w : nullptr;
    A.norm_eps = ni ? ni->eps : 0.0f;
    return stream_launch<ARGMAX>(A, st);
}

}  // namespace k3
