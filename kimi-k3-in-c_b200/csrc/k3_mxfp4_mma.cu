// k3_mxfp4_mma.cu -- the MXFP4 expert GEMV on tensor cores, fed by bulk TMA copies.
//
// WHAT IT COMPUTES: y[r] = sum_k W[r][k] x[k] for W in packed MXFP4 (the CPU engine's
// k3_matmul_mxfp4, k3_ops.c:1380-1785), for several rows and up to four activation
// vectors at once, with two fused epilogues:
//   MODE_GATEUP  rows 0-7 of a tile are gate rows i..i+7, rows 8-15 the up rows of the
//                same i; the epilogue writes act[i] = silu(gate) * up   (k3_ops.c:628-630)
//   MODE_DOWN    16 rows of the down matrix; the epilogue writes the contribution rows.
//
// WHY TENSOR CORES FOR A MEMORY-BOUND GEMV: decoding E2M1 to fp32 and multiplying on the
// FMA pipe costs ~3 issue slots per weight, which keeps a B200 SM issue-bound below HBM
// speed. Here one cvt.rn.f16x2.e2m1x2 turns two codes into an exact f16 pair and
// mma.sync does the multiply-accumulate in fp32, about one issue slot per weight.
//
// EXACTNESS OF THE OPERANDS:
//   A (weights): E2M1 values are exact in f16; the E8M0 group scale (a power of two) is
//     applied in fp32 to the accumulator of each 32-element group, so a group maps to
//     exactly two chained k16 MMAs and a scale of 255 (NaN) contributes zero.
//   B (activations): each fp32 vector is scaled by a power of two 2^-e so max|x| < 1,
//     then split into hi = f16(x) and lo = f16(x - hi); hi + lo carries 22 significant
//     bits with an absolute floor of 2^-25 * max|x|. Columns of the 16x8 B tile are
//     (vector 0 hi, vector 0 lo, vector 1 hi, ..., vector 3 lo). The epilogue multiplies
//     by 2^e. Result error is at the level of fp32 accumulation, far inside 1e-3.
//
// DATA MOVEMENT: one CTA per SM (persistent), one producer warp and eight consumer
// warps. The producer streams each 16-row tile (codes, one bulk copy per row into a
// padded pitch so ldmatrix rows hit distinct banks; scales, one bulk copy per 8 rows)
// into a ring of S shared-memory stages with cp.async.bulk, completing on an mbarrier.
// The consumer warps split the tile's K range eight ways, load A fragments with
// ldmatrix (a 16-byte row of packed codes is exactly one group of 32 elements), reduce
// their partial sums through shared memory and run the epilogue. Every mbarrier wait is
// bounded: after ~2 s it stores K3D_ETIMEOUT in the device error flag and the CTA exits.
#include "k3_moe.cuh"
#include "k3_ops.cuh"

namespace k3 {

enum { MODE_GATEUP = 0, MODE_DOWN = 1 };

struct MmaJob {
    MoeWork w;
    int mode;
    int in;            // K: elements per row
    int rows;          // gate/up: intermediate size (pairs); down: output rows
    int nblk;          // items (stages) per expert
    int n_items;       // (max active experts) * nblk
    int rt;            // 16-row tiles per stage
    const __half *xb;  // split activations [nvec][2][in]
    const float *xsc;  // per-vector scale 2^e [nvec]
    int x_by_assign;   // 0: vector = token (a / K); 1: vector = assignment a
    float *out;        // gate/up: act [assign][rows]; down: contrib [assign][rows]
    int stages;
    int stage_bytes;
    int pitch;         // bytes per code row in shared memory
};

static const int kCW = 16;          // consumer warps
static const int kThreads = (kCW + 1) * 32;

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(b)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(b)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(b)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
    return ok != 0;
}

// Bounded wait: false after ~2 s (4e9 cycles); the caller then abandons the kernel.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity)
{
    if (mbar_try(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(b, parity)) {
        if (clock64() - t0 > 4000000000LL) return false;
    }
    return true;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *b)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(b)) : "memory");
}

// volatile + memory clobber: must not move above the mbarrier wait that publishes the
// stage it reads
__device__ __forceinline__ void ldsm_x4(uint32_t r[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}

// register-only: free for the compiler to schedule across loop iterations
__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                          const float c[4])
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
          "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

__device__ __forceinline__ void cvt8(uint32_t w, uint32_t out[4])
{
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3]) : "r"(w));
}

__device__ __forceinline__ void named_sync(int id, int n)
{
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(n) : "memory");
}

// Two E8M0 bytes (low byte = first group) -> two fp32 scales. Bytes 1..254 are the
// normal power of two s << 23; 0 (2^-127) and 255 (NaN -> 0) take the exact slow path.
__device__ __forceinline__ void e8m0x2(uint32_t v, float &s0, float &s1)
{
    const uint32_t b0 = v & 0xffu, b1 = (v >> 8) & 0xffu;
    s0 = __uint_as_float(b0 << 23);
    s1 = __uint_as_float(b1 << 23);
    if (((b0 - 1u) > 253u) | ((b1 - 1u) > 253u)) {
        s0 = e8m0_to_f32(b0);
        s1 = e8m0_to_f32(b1);
    }
}

// Resolves a work item; identical in producer and consumers so both walk the same
// sequence of stages.
__device__ __forceinline__ bool job_item(const MmaJob &J, int item, K3ExpertQ &q, int &beg,
                                         int &end, int &blk)
{
    const int u = item / J.nblk;
    blk = item % J.nblk;
    bool ok;
    work_item(J.w, u, q, beg, end, ok);
    return ok;
}

// Items are dealt in contiguous runs, so one CTA mostly stays on one expert (its
// activation fragments stay in registers and its reads stay sequential).
__device__ __forceinline__ void item_range(const MmaJob &J, int &i0, int &i1)
{
    const int per = (J.n_items + gridDim.x - 1) / gridDim.x;
    i0 = blockIdx.x * per;
    i1 = min(J.n_items, i0 + per);
}

template <int GPW>
__global__ void __launch_bounds__(kThreads, 1) k_mxfp4_mma(MmaJob J)
{
    extern __shared__ __align__(128) unsigned char smem[];
    const int S = J.stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + S;
    float *red = reinterpret_cast<float *>(smem + 256);          // [kCW warps][32 lanes][4]
    unsigned char *stage0 = smem + 256 + kCW * 32 * 4 * 4;        // 128-aligned
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rowbytes = J.in >> 1;
    const int ngrp = J.in >> 5;
    const int pitch = J.pitch;
    const int rt = J.rt;
    const int tile_rows = 16 * rt;
    const int codes_bytes = tile_rows * pitch;
    int i_beg, i_end;
    item_range(J, i_beg, i_end);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], kCW); }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kCW) {
        // ------------------------------------------------------------- producer ----
        if (lane == 0) {
            int it = 0;
            for (int item = i_beg; item < i_end; item++) {
                K3ExpertQ q; int beg, end, blk;
                if (!job_item(J, item, q, beg, end, blk)) continue;
                const int s = it % S;
                if (it >= S && !mbar_wait(&empty[s], ((it / S) - 1) & 1)) {
                    k3_raise(K3D_ETIMEOUT, K3_SITE_MXFP4);
                    abort_flag = 1;
                    break;
                }
                unsigned char *st = stage0 + (size_t)s * J.stage_bytes;
                const uint32_t tx = (uint32_t)tile_rows * (rowbytes + ngrp);
                mbar_expect_tx(&full[s], tx);
                if (J.mode == MODE_GATEUP) {
                    const int i0 = blk * 8;               // rt == 1
                    for (int r = 0; r < 8; r++) {
                        bulk_g2s(st + r * pitch, q.p1 + (size_t)(i0 + r) * rowbytes, rowbytes, &full[s]);
                        bulk_g2s(st + (r + 8) * pitch, q.p3 + (size_t)(i0 + r) * rowbytes, rowbytes, &full[s]);
                    }
                    bulk_g2s(st + codes_bytes, q.s1 + (size_t)i0 * ngrp, 8u * ngrp, &full[s]);
                    bulk_g2s(st + codes_bytes + 8 * ngrp, q.s3 + (size_t)i0 * ngrp, 8u * ngrp, &full[s]);
                } else {
                    const int r0 = blk * tile_rows;
                    for (int r = 0; r < tile_rows; r++)
                        bulk_g2s(st + r * pitch, q.p2 + (size_t)(r0 + r) * rowbytes, rowbytes, &full[s]);
                    bulk_g2s(st + codes_bytes, q.s2 + (size_t)r0 * ngrp, (uint32_t)tile_rows * ngrp, &full[s]);
                }
                it++;
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers ----
    const int qrow = lane >> 2, c = lane & 3;
    const int wpt = kCW / rt;                 // warps per 16-row tile
    const int tile = warp / wpt;              // this warp's tile within the stage
    const int wk = warp % wpt;                // this warp's K slice
    const int gpw = ngrp / wpt;               // == GPW when specialised
    const int g0 = wk * gpw;
    const int lm_row = tile * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
    const int lm_goff = (lane >> 4);
    // B fragments of the current quad for this warp's K slice, kept across items
    uint4 breg[GPW > 0 ? GPW : 1];
    int cached_v0 = -2, cached_v1 = -2, cached_v2 = -2, cached_v3 = -2;
    int it = 0;
    for (int item = i_beg; item < i_end; item++) {
        K3ExpertQ q; int beg, end, blk;
        if (!job_item(J, item, q, beg, end, blk)) continue;
        const int s = it % S;
        // the wait is bounded; its outcome is made collective (a named barrier over the
        // consumer warps, which every one of them reaches in bounded time) so that no
        // warp can be left waiting at a later barrier for a warp that gave up
        if (!mbar_wait(&full[s], (it / S) & 1)) {
            if (lane == 0) k3_raise(K3D_ETIMEOUT, K3_SITE_MXFP4);
            atomicExch(&abort_flag, 1);
        }
        named_sync(1, kCW * 32);
        if (*(volatile int *)&abort_flag) return;
        const unsigned char *st = stage0 + (size_t)s * J.stage_bytes;
        const unsigned char *sc = st + codes_bytes + (size_t)tile * 16 * ngrp;
        const uint32_t lm_base = smem_u32(st + lm_row * pitch + lm_goff * 16);

        for (int p0 = beg; p0 < end; p0 += 4) {
            int a_of[4], v_of[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int a = (p0 + k < end) ? work_assign(J.w, p0 + k) : -1;
                a_of[k] = a;
                v_of[k] = a < 0 ? -1 : (J.x_by_assign ? a : a / J.w.K);
            }
            const int bv = v_of[qrow >> 1];
            const __half *bsrc = bv < 0 ? nullptr
                                        : J.xb + ((size_t)bv * 2 + (qrow & 1)) * J.in + 8 * c;
            if (GPW > 0) {
                if (v_of[0] != cached_v0 || v_of[1] != cached_v1 || v_of[2] != cached_v2 ||
                    v_of[3] != cached_v3) {
#pragma unroll
                    for (int j = 0; j < (GPW > 0 ? GPW : 1); j++)
                        breg[j] = bsrc ? *reinterpret_cast<const uint4 *>(bsrc + 32 * (g0 + j))
                                       : make_uint4(0, 0, 0, 0);
                    cached_v0 = v_of[0]; cached_v1 = v_of[1]; cached_v2 = v_of[2]; cached_v3 = v_of[3];
                }
            }
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            const float zero[4] = {0.f, 0.f, 0.f, 0.f};
            const int jmax = GPW > 0 ? GPW : gpw;
#pragma unroll
            for (int j = 0; j < jmax; j += 2) {
                const int g = g0 + j;
                uint32_t w4[4];
                ldsm_x4(w4, lm_base + g * 16);
                float sq[2], sq8[2];
                e8m0x2(*reinterpret_cast<const uint16_t *>(sc + qrow * ngrp + g), sq[0], sq[1]);
                e8m0x2(*reinterpret_cast<const uint16_t *>(sc + (qrow + 8) * ngrp + g), sq8[0], sq8[1]);
#pragma unroll
                for (int gg = 0; gg < 2; gg++) {
                    uint32_t hq[4], hq8[4];
                    cvt8(w4[2 * gg], hq);
                    cvt8(w4[2 * gg + 1], hq8);
                    uint4 bb;
                    if (GPW > 0) bb = breg[(j + gg) % (GPW > 0 ? GPW : 1)];
                    else bb = bsrc ? *reinterpret_cast<const uint4 *>(bsrc + 32 * (g + gg))
                                   : make_uint4(0, 0, 0, 0);
                    const uint32_t a0[4] = {hq[0], hq8[0], hq[1], hq8[1]};
                    const uint32_t a1[4] = {hq[2], hq8[2], hq[3], hq8[3]};
                    float d0[4], d1[4];
                    mma_16816(d0, a0, bb.x, bb.y, zero);
                    mma_16816(d1, a1, bb.z, bb.w, d0);
                    acc[0] = fmaf(d1[0], sq[gg], acc[0]);
                    acc[1] = fmaf(d1[1], sq[gg], acc[1]);
                    acc[2] = fmaf(d1[2], sq8[gg], acc[2]);
                    acc[3] = fmaf(d1[3], sq8[gg], acc[3]);
                }
            }
            // reduction of the K slices of each tile, then the epilogue on the tile's
            // first warp
            float4 *rw = reinterpret_cast<float4 *>(red) + warp * 32 + lane;
            *rw = make_float4(acc[0], acc[1], acc[2], acc[3]);
            named_sync(1, kCW * 32);
            if (wk == 0) {
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int w = 0; w < wpt; w++) {
                    const float4 v = reinterpret_cast<const float4 *>(red)[(tile * wpt + w) * 32 + lane];
                    t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
                }
                const int a = a_of[c];
                if (a >= 0) {
                    const float xs = J.xsc[v_of[c]];
                    const float r0v = (t.x + t.y) * xs;
                    const float r8v = (t.z + t.w) * xs;
                    if (J.mode == MODE_GATEUP) {
                        J.out[(size_t)a * J.rows + blk * 8 + qrow] = silu_f(r0v) * r8v;
                    } else {
                        float *o = J.out + (size_t)a * J.rows + (size_t)blk * tile_rows + tile * 16;
                        o[qrow] = r0v;
                        o[qrow + 8] = r8v;
                    }
                }
            }
            named_sync(1, kCW * 32);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        it++;
    }
}

// Split fp32 vectors into f16 hi/lo pieces after a power-of-two normalisation.
// One CTA per vector: xb [nvec][2][n], xsc [nvec].
__global__ void k_xsplit(__half *xb, float *xsc, const float *x, int n, size_t ld)
{
    __shared__ float red[32];
    const float *xv = x + blockIdx.x * ld;
    float m = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(xv[i]));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_max(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float mx = red[0];
    // e with mx * 2^-e < 1; non-finite or zero vectors keep e = 0
    int e = 0;
    if (mx > 0.f && mx <= 3.0e38f) e = ilogbf(mx) + 1;
    const float inv = ldexpf(1.0f, -e);
    __half *hi = xb + (size_t)blockIdx.x * 2 * n;
    __half *lo = hi + n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = xv[i] * inv;
        const __half h = __float2half_rn(v);
        hi[i] = h;
        lo[i] = __float2half_rn(v - __half2float(h));
    }
    if (threadIdx.x == 0) xsc[blockIdx.x] = ldexpf(1.0f, e);
}

// Shared memory: a head (barriers + the B-fragment exchange) then S stages of rt
// 16-row tiles, each row in/2 packed bytes padded by 16, then the tiles' scales.
static constexpr int kHead = 256 + kCW * 32 * 4 * 4;
static constexpr int kBudget = 220 * 1024 - kHead;
static int stage_bytes_for(int in, int rt)
{
    return ((16 * rt * (in / 2 + 16) + 16 * rt * (in / 32)) + 127) & ~127;
}

// Tiles per stage for a shape, or 0 when the tensor-core kernel cannot run it: every
// consumer warp takes an even number of 32-element groups of one 16-row tile, and the
// ring holds at least two stages (three when a smaller tile allows it).
static int mma_plan(int in, int rows, int mode)
{
    if (in % 32 != 0 || in > 16384 || in < 64) return 0;
    const int ngrp = in / 32;
    if (mode == MODE_GATEUP) {
        if (rows % 8 != 0) return 0;
        if (kBudget / stage_bytes_for(in, 1) < 2) return 0;
        return (ngrp % kCW == 0 && (ngrp / kCW) % 2 == 0) ? 1 : 0;
    }
    int fallback = 0;
    for (int rt = 4; rt >= 1; rt /= 2) {
        const int wpt = kCW / rt;
        if (rows % (16 * rt) != 0 || ngrp % wpt != 0 || (ngrp / wpt) % 2 != 0) continue;
        const int S = kBudget / stage_bytes_for(in, rt);
        if (S >= 3) return rt;
        if (S >= 2 && fallback == 0) fallback = rt;
    }
    return fallback;
}

bool mma_supported(int in, int rows, int mode) { return mma_plan(in, rows, mode) > 0; }

int xsplit(__half *xb, float *xsc, const float *x, int n, int nvec, size_t ld, cudaStream_t s)
{
    if (nvec <= 0) return K3D_OK;
    k_xsplit<<<nvec, 256, 0, s>>>(xb, xsc, x, n, ld);
    note_launch();
    return check_launch("xsplit");
}

// Launch for a MoE work list (or a single expert in single mode).
int mxfp4_mma_launch(int mode, const MoeWork &w, int umax, int in, int rows, const __half *xb,
                     const float *xsc, int x_by_assign, float *out, cudaStream_t st)
{
    MmaJob J;
    J.w = w;
    J.mode = mode;
    J.in = in;
    J.rows = rows;
    const int ngrp = in / 32;
    // gate/up: one 16-row tile (8 gate + 8 up rows) per stage; down: up to 4 tiles so a
    // stage carries ~64 KB whatever the row length
    const int rt = mma_plan(in, rows, mode);
    if (rt == 0) return fail(K3D_EINVAL, "mxfp4 mma: unsupported shape in=%d rows=%d", in, rows);
    const int wpt = kCW / rt;
    J.rt = rt;
    J.nblk = mode == MODE_GATEUP ? rows / 8 : rows / (16 * rt);
    J.n_items = umax * J.nblk;
    J.xb = xb;
    J.xsc = xsc;
    J.x_by_assign = x_by_assign;
    J.out = out;
    J.pitch = in / 2 + 16;
    J.stage_bytes = stage_bytes_for(in, rt);
    const int head = kHead;
    int S = kBudget / J.stage_bytes;
    if (S > 8) S = 8;
    if (S < 2) return fail(K3D_EINVAL, "mxfp4 mma: stage of %d bytes does not fit", J.stage_bytes);
    J.stages = S;
    const size_t smem = (size_t)head + (size_t)S * J.stage_bytes;
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) {
        allow_smem_max(k_mxfp4_mma<14>);
        allow_smem_max(k_mxfp4_mma<16>);
        allow_smem_max(k_mxfp4_mma<0>);
        init |= dev_bit();
    }
    int grid = sm_count();
    if (grid > J.n_items) grid = J.n_items;
    if (grid < 1) return K3D_OK;
    const int gpw = ngrp / wpt;
    if (gpw == 14) k_mxfp4_mma<14><<<grid, kThreads, smem, st>>>(J);
    else if (gpw == 16) k_mxfp4_mma<16><<<grid, kThreads, smem, st>>>(J);
    else k_mxfp4_mma<0><<<grid, kThreads, smem, st>>>(J);
    note_launch();
    return check_launch("mxfp4 mma");
}

}  // namespace k3
