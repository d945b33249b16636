// k3_moe.cu -- MXFP4 routed experts (SwiGLU) and the MoE layer at the benchmark shapes:
// k3d_expert_swiglu (config 0) and k3d_moe_swiglu (config 1).
//
// Follows k3_moe / moe_prefill_chunk (k3_ops.c:556-656, 717-825):
//   1. route every token (k3_router semantics, bit-identical indices and weights);
//   2. group the (token, slot) assignments by expert, so each selected expert's bytes
//      are read from HBM once per step however many tokens chose it (the CPU's
//      "fetch each unique expert once" of moe_prefill_chunk);
//   3. gate/up GEMVs with SiLU(g)*u fused into the epilogue, per expert;
//   4. down GEMV per expert into a per-assignment contribution buffer;
//   5. per token, sum contributions in the ORIGINAL top-k order (acc += w_j * edn_j
//      with separate multiply and add, k3_ops.c:641-642 / 806-810), then add the
//      unweighted shared expert.
// BASELINE shapes have no latent projection and use SiLU where the released model uses
// SiTU; the CPU reference-semantics path (k3_moe in k3_refops.cu) keeps SiTU and the
// latent MoE.
//
// Expert parallelism: only experts in [expert_lo, expert_hi) are computed here; the
// combine treats the others as zero and the caller sums the partial outputs over ranks.
#include <algorithm>
#include <vector>

#include "k3_mxfp4.cuh"
#include "k3_moe.cuh"
#include "k3_ops.cuh"

namespace k3 {

// ---- prep: group assignments by expert (one CTA) --------------------------------
__global__ void __launch_bounds__(1024) k_moe_prep(const int *idx, int TK, int n_experts,
                                                   int lo, int hi, int *n_active,
                                                   int *act_expert, int *act_off, int *assign,
                                                   int *zero, int nzero)
{
    pdl_wait();
    pdl_trigger();
    extern __shared__ int sm[];
    group_assignments(idx, TK, n_experts, lo, hi, n_active, act_expert, act_off, assign, sm, zero, nzero);
}

// ---- gate/up + SiLU*mul -------------------------------------------------------------
// Work item = (active expert u, block of IPC intermediate indices). Persistent grid.
template <int NCHMAX>
__global__ void __launch_bounds__(256, 2) k_moe_gate_up(float *act, const float *x, MoeWork w,
                                                        int hidden, int inter, int nblk,
                                                        int n_items, int ipc)
{
    extern __shared__ float4 xs[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nch = hidden >> 5;
    const int pcols = hidden >> 1, ngrp = hidden >> 5;
    int staged_tok = -1;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int u = item / nblk, blk = item % nblk;
        K3ExpertQ q; int beg = 0, end = 0; bool ok;
        work_item(w, u, q, beg, end, ok);
        if (!ok) continue;
        if (bad_align(q.p1, q.p3)) { if (threadIdx.x == 0) k3_raise(K3D_EINVAL, K3_SITE_MOE); continue; }
        for (int p = beg; p < end; p++) {
            const int a = work_assign(w, p);
            const int t = a / w.K;
            if (t != staged_tok) {
                __syncthreads();
                stage_x_mxfp4(xs, x + (size_t)t * hidden, hidden);
                __syncthreads();
                staged_tok = t;
            }
            for (int i = blk * ipc + warp; i < min(inter, (blk + 1) * ipc); i += 8) {
                const unsigned char *pr[2] = {q.p1 + (size_t)i * pcols, q.p3 + (size_t)i * pcols};
                const unsigned char *sr[2] = {q.s1 + (size_t)i * ngrp, q.s3 + (size_t)i * ngrp};
                float acc[2];
                mxfp4_rows_partial<2, NCHMAX>(acc, pr, sr, xs, nch);
                const float g = warp_sum(acc[0]);
                const float uu = warp_sum(acc[1]);
                if (lane == 0) act[(size_t)a * inter + i] = silu_f(g) * uu;
            }
        }
    }
}

// ---- down ---------------------------------------------------------------------------
// Work item = (active expert u, block of RPC output rows). contrib[a][r] = W_down[r] . act[a]
template <int R, int NCHMAX>
__global__ void __launch_bounds__(256, 2) k_moe_down(float *contrib, const float *act, MoeWork w,
                                                     int hidden, int inter, int nblk,
                                                     int n_items, int rpc)
{
    extern __shared__ float4 xs[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nch = inter >> 5;
    const int pcols = inter >> 1, ngrp = inter >> 5;
    int staged_a = -1;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int u = item / nblk, blk = item % nblk;
        K3ExpertQ q; int beg = 0, end = 0; bool ok;
        work_item(w, u, q, beg, end, ok);
        if (!ok) continue;
        if (bad_align(q.p2, q.p2)) { if (threadIdx.x == 0) k3_raise(K3D_EINVAL, K3_SITE_MOE); continue; }
        for (int p = beg; p < end; p++) {
            const int a = work_assign(w, p);
            if (a != staged_a) {
                __syncthreads();
                stage_x_mxfp4(xs, act + (size_t)a * inter, inter);
                __syncthreads();
                staged_a = a;
            }
            const int r_end = min(hidden, (blk + 1) * rpc);
            for (int r0 = blk * rpc + warp * R; r0 < r_end; r0 += 8 * R) {
                const unsigned char *pr[R];
                const unsigned char *sr[R];
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const int rr = min(r0 + r, hidden - 1);
                    pr[r] = q.p2 + (size_t)rr * pcols;
                    sr[r] = q.s2 + (size_t)rr * ngrp;
                }
                float acc[R];
                mxfp4_rows_partial<R, NCHMAX>(acc, pr, sr, xs, nch);
#pragma unroll
                for (int r = 0; r < R; r++) {
                    const float v = warp_sum(acc[r]);
                    if (lane == 0 && r0 + r < r_end) contrib[(size_t)a * hidden + r0 + r] = v;
                }
            }
        }
    }
}

// ---- ordered combine ------------------------------------------------------------------
// early: the routing (idx, wts, pos_of) and the residual were written on this stream at
// least two kernels back (the expert passes ran in between), so they are read before the
// programmatic wait. The shared expert's output is read after it: it comes from the side
// stream, and a captured graph turns that join into a programmatic edge too, which lets
// this kernel start before the side stream's last kernel has finished.
__global__ void k_moe_combine(float *out, const float *contrib, int ks, size_t slice_stride,
                              const int *idx, const float *wts, const float *sh_out, int hidden,
                              int K, int lo, int hi, int accumulate, const int *pos_of, int early)
{
    const int t = blockIdx.y;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (!early) {
        pdl_wait();
        pdl_trigger();
    }
    if (r >= hidden) {
        if (early) { pdl_wait(); pdl_trigger(); }
        return;
    }
    float *o = out + (size_t)t * hidden + r;
    const float prev = accumulate ? *o : 0.0f;
    float acc = 0.0f;
    // top-k slots in groups of 8: the group's expert ids, weights and contributions are all
    // loaded before the ordered sum, so the loads overlap instead of chaining; the slices
    // go in groups of 4 whose 8 x 4 loads are all issued before they are added.
    for (int j0 = 0; j0 < K; j0 += 8) {
        int e[8];
        float w[8], v[8];
        const float *c[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int a = t * K + min(j0 + k, K - 1);
            e[k] = __ldg(idx + a);
            w[k] = __ldg(wts + a);
            // contributions by assignment, or by grouped position (only this rank's experts
            // have one: another rank's slot reads row 0 and is not added)
            const bool local = e[k] >= lo && e[k] < hi;
            const int row = !pos_of ? a : (local ? __ldcg(pos_of + a) : 0);
            c[k] = contrib + (size_t)row * hidden + r;
        }
        if (early && j0 == 0) {
            pdl_wait();
            pdl_trigger();
        }
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = c[k][0];
        for (int s0 = 1; s0 < ks; s0 += 4) {
            float t4[4][8];
#pragma unroll
            for (int i = 0; i < 4; i++)
                if (s0 + i < ks) {
#pragma unroll
                    for (int k = 0; k < 8; k++) t4[i][k] = c[k][(size_t)(s0 + i) * slice_stride];
                }
#pragma unroll
            for (int i = 0; i < 4; i++)
                if (s0 + i < ks) {
#pragma unroll
                    for (int k = 0; k < 8; k++) v[k] += t4[i][k];
                }
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            if (j0 + k >= K || e[k] < lo || e[k] >= hi) continue;
            acc = __fadd_rn(acc, __fmul_rn(w[k], v[k]));
        }
    }
    if (sh_out) acc = __fadd_rn(acc, sh_out[(size_t)t * hidden + r]);   // after the wait (K >= 1)
    *o = accumulate ? __fadd_rn(prev, acc) : acc;
}

// ---- host side -------------------------------------------------------------------------
template <typename K>
static void allow_smem(K kern)
{
    allow_smem_max(kern);
}

static int nchmax_for(int n)
{
    const int per = (n / 32 + 31) / 32;
    if (per <= 1) return 1;
    if (per <= 2) return 2;
    if (per <= 4) return 4;
    if (per <= 7) return 7;
    if (per <= 8) return 8;
    return -1;
}

static int persistent_grid(int items)
{
    int g = sm_count() * 2;
    if (items < g) g = items;
    return g < 1 ? 1 : g;
}

static const int kIPC = 32;   // intermediate indices per gate/up work item
static const int kRPC = 64;   // down rows per work item

static int launch_gate_up(float *act, const float *x, const MoeWork &w, int hidden, int inter,
                          int umax, cudaStream_t s)
{
    const int nblk = (inter + kIPC - 1) / kIPC;
    const int items = umax * nblk;
    const size_t smem = (size_t)hidden * sizeof(float);
    const int g = persistent_grid(items);
    switch (nchmax_for(hidden)) {
#define K3_GU(N) case N: { static bool i = false; if (!i) { allow_smem(k_moe_gate_up<N>); i = true; } \
        k_moe_gate_up<N><<<g, 256, smem, s>>>(act, x, w, hidden, inter, nblk, items, kIPC); break; }
        K3_GU(1) K3_GU(2) K3_GU(4) K3_GU(7) K3_GU(8)
#undef K3_GU
    default: return fail(K3D_EINVAL, "expert hidden=%d exceeds 8192", hidden);
    }
    note_launch();
    return check_launch("moe gate/up");
}

static int launch_down(float *contrib, const float *act, const MoeWork &w, int hidden, int inter,
                       int umax, cudaStream_t s)
{
    const int nblk = (hidden + kRPC - 1) / kRPC;
    const int items = umax * nblk;
    const size_t smem = (size_t)inter * sizeof(float);
    const int g = persistent_grid(items);
    switch (nchmax_for(inter)) {
#define K3_DN(N) case N: { static bool i = false; if (!i) { allow_smem(k_moe_down<4, N>); i = true; } \
        k_moe_down<4, N><<<g, 256, smem, s>>>(contrib, act, w, hidden, inter, nblk, items, kRPC); break; }
        K3_DN(1) K3_DN(2) K3_DN(4) K3_DN(7) K3_DN(8)
#undef K3_DN
    default: return fail(K3D_EINVAL, "expert inter=%d exceeds 8192", inter);
    }
    note_launch();
    return check_launch("moe down");
}

static size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

// Which expert kernel runs (k3d_set_expert_kernel): 0 chooses the tcgen05 block-scaled
// kernel whenever the shapes allow (gate/up, act split and down as three launches), 1 forces
// the mma.sync kernel, 2 the CUDA-core kernels, 3 the tcgen05 kernel with B in every stage,
// 4 the same as 0 but decode-sized work lists as ONE launch (k_mxfp4_fused).
static int g_expert_kernel = 0;
static const int kUmmaMaxTK = 64;     // assignments per call for the tcgen05 path

// Buffers of one run_experts call; the tcgen05 ones are null when the workspace has none.
struct ExpertBufs {
    float *act, *contrib;                  // CUDA-core / mma.sync: [TK][inter], [TK][hidden]
    __half *xb_x; float *xs_x; __half *xb_a; float *xs_a;   // mma.sync activation splits
    uint8_t *bq_x, *bs_x, *bq_a, *bs_a;    // tcgen05: E2M1 pieces of x and of act
    float *part_gu, *part_d;               // tcgen05: K-slice partials
    uint8_t *bqg_x, *bsg_x, *bqg_a, *bsg_a;   // tcgen05 grouped: pieces of x and act by group
    UmmaGroups grp;                        // tcgen05 grouped: the groups (null when absent)
    int *fcnt;                             // tcgen05 fused pass: its counters (null when absent)
    int fcnt_n;                            // their count (ints)
};

// Where the per-assignment contributions ended up: contrib[s * slice + a * hidden + r].
struct ExpertOut {
    const float *contrib;
    int ks;
    size_t slice;
    const int *pos_of;       // grouped pass: contributions are by position; pos_of[a] = row
};

static bool umma_shapes(int hidden, int inter)
{
    return umma_supported(hidden, inter, 0) && umma_supported(inter, hidden, 1);
}

// The tcgen05 buffers exist in a workspace when the kernel can run: checkpoint-layout
// experts up to kUmmaMaxTK assignments (beyond that the grouped mma.sync kernel reads each
// expert once for all its tokens), tiled experts always.
static bool umma_eligible(int hidden, int inter, int TK, int layout)
{
    return umma_shapes(hidden, inter) && (layout == 1 || TK <= kUmmaMaxTK);
}

// K slices the partial buffers are sized for: every stage up to kUmmaMaxTK assignments,
// one slice beyond (there are enough items to fill the GPU without splitting K).
static int umma_ks_cap(int K, int TK)
{
    return TK <= kUmmaMaxTK ? K / 512 : 1;
}

// The grouped tcgen05 pass (several tokens of an expert share each weight stage) for
// batches: tiled experts, more than kUmmaMaxTK assignments, unless kind 3 turns it off.
static bool grouped_eligible(int hidden, int inter, int TK, int layout)
{
    return layout == 1 && TK > kUmmaMaxTK && umma_shapes(hidden, inter);
}

// True when run_experts takes the tcgen05 path.
static bool use_umma(const ExpertBufs &B, int hidden, int inter, int TK, int layout)
{
    return (layout == 1 || g_expert_kernel == 0 || g_expert_kernel >= 3) && B.bq_x &&
           umma_eligible(hidden, inter, TK, layout);
}

static bool use_grouped(const ExpertBufs &B, int TK, int layout, int hidden, int inter)
{
    return g_expert_kernel != 3 && B.bqg_x && grouped_eligible(hidden, inter, TK, layout);
}

// gate/up -> act -> down -> contributions for a work list. tcgen05 block-scaled MMA
// (k3_mxfp4_umma.cu) when the workspace carries its buffers and the kernel choice allows,
// else the mma.sync kernel (k3_mxfp4_mma.cu), else the CUDA-core kernels. `count` is the
// device count of local assignments (MoE) or null (single expert, one assignment).
// x_split: the caller already wrote x's tcgen05 B operand (umma_bsplit into B.bq_x/bs_x).
// cnt_zeroed: B.fcnt was zeroed by the grouping that wrote this work list (the fused launch
// needs its counters at zero).
static int run_experts(const MoeWork &mw, const int *idx, const int *count, int umax,
                       const float *x, int T, int TK, int hidden, int inter, int layout,
                       const ExpertBufs &B, ExpertOut &O, cudaStream_t st, bool x_split = false,
                       bool cnt_zeroed = false)
{
    O.contrib = B.contrib;
    O.ks = 1;
    O.slice = 0;
    const int topk = mw.single_mode ? 1 : mw.K;
    if (layout == 1 && (!B.bq_x || !umma_eligible(hidden, inter, TK, 1)))
        return fail(K3D_EINVAL, "tiled experts need hidden and inter multiples of 512");
    O.pos_of = nullptr;
    if (!mw.single_mode && count && use_grouped(B, TK, layout, hidden, inter)) {
        // groups of up to four tokens of one expert share each weight stage; one K chunk
        // per slice (items ordered (group, chunk, tile), B resident across a run); partials
        // by position
        const int ks_gu = hidden / 512, ks_d = inter / 512;
        const size_t sl_gu = (size_t)TK * 2 * inter, sl_d = (size_t)TK * hidden;
        K3_TRY(umma_make_groups(mw, B.grp, st));
        K3_TRY(umma_bsplit_group_x(B.bqg_x, B.bsg_x, x, hidden, mw.assign, topk, B.grp, TK, st));
        prof_begin("experts.gateup");
        K3_TRY(umma_launch_grouped(0, mw, B.grp, TK, hidden, inter, ks_gu, B.bqg_x, B.bsg_x, B.part_gu, 2 * inter,
                                   sl_gu, st));
        prof_end("experts.gateup");
        K3_TRY(umma_bsplit_swiglu_group(B.bqg_a, B.bsg_a, B.part_gu, ks_gu, sl_gu, inter, B.grp, TK, st));
        prof_begin("experts.down");
        K3_TRY(umma_launch_grouped(1, mw, B.grp, TK, inter, hidden, ks_d, B.bqg_a, B.bsg_a, B.part_d, hidden, sl_d,
                                   st));
        prof_end("experts.down");
        O.contrib = B.part_d;
        O.ks = ks_d;
        O.slice = sl_d;
        O.pos_of = B.grp.pos_of;
        return K3D_OK;
    }
    if (!mw.single_mode && count && cnt_zeroed && B.fcnt && layout == 1 && g_expert_kernel == 4 &&
        use_umma(B, hidden, inter, TK, layout) && umma_fused_ok(TK, hidden, inter)) {
        // decode-sized work lists: gate/up, act split and down in one launch; partials and
        // operands as in the three-launch resident path below
        const size_t sl_gu = (size_t)TK * 2 * inter, sl_d = (size_t)TK * hidden;
        if (!x_split) K3_TRY(umma_bsplit(B.bq_x, B.bs_x, x, hidden, T, hidden, st));
        prof_begin("experts.fused");
        K3_TRY(umma_launch_fused(mw, idx, count, TK, hidden, inter, B.bq_x, B.bs_x, topk, B.part_gu, sl_gu,
                                 B.bq_a, B.bs_a, B.part_d, sl_d, B.fcnt, st));
        prof_end("experts.fused");
        O.contrib = B.part_d;
        O.ks = inter / 512;
        O.slice = sl_d;
        return K3D_OK;
    }
    if (use_umma(B, hidden, inter, TK, layout)) {
        // tiled experts keep B resident across the stages of a run (one K chunk per item);
        // kind 3 keeps B in every stage
        const int resident = layout == 1 && g_expert_kernel != 3 && TK <= kUmmaMaxTK;
        const int ks_gu = resident ? hidden / 512
                                   : std::min(umma_slices(TK, hidden, inter, 0), umma_ks_cap(hidden, TK));
        const int ks_d = resident ? inter / 512
                                  : std::min(umma_slices(TK, inter, hidden, 1), umma_ks_cap(inter, TK));
        const size_t sl_gu = (size_t)TK * 2 * inter, sl_d = (size_t)TK * hidden;
        if (!x_split) K3_TRY(umma_bsplit(B.bq_x, B.bs_x, x, hidden, T, hidden, st));
        prof_begin("experts.gateup");
        // the gate/up work list comes from the router just before (MoE); the down pass's
        // does not depend on the split just before it, nor does a single expert's
        K3_TRY(umma_launch(0, layout, mw, idx, count, TK, hidden, inter, ks_gu, B.bq_x, B.bs_x, topk,
                           B.part_gu, 2 * inter, sl_gu, st, mw.single_mode ? 1 : 0, resident));
        prof_end("experts.gateup");
        K3_TRY(umma_bsplit_swiglu(B.bq_a, B.bs_a, B.part_gu, ks_gu, sl_gu, inter, count, TK, st));
        prof_begin("experts.down");
        K3_TRY(umma_launch(1, layout, mw, idx, count, TK, inter, hidden, ks_d, B.bq_a, B.bs_a, 1,
                           B.part_d, hidden, sl_d, st, 1, resident));
        prof_end("experts.down");
        O.contrib = B.part_d;
        O.ks = ks_d;
        O.slice = sl_d;
        return K3D_OK;
    }
    if (g_expert_kernel <= 1 && mma_supported(hidden, inter, 0) && mma_supported(inter, hidden, 1) &&
        B.xb_x && B.xb_a) {
        K3_TRY(xsplit(B.xb_x, B.xs_x, x, hidden, T, hidden, st));
        prof_begin("experts.gateup");
        K3_TRY(mxfp4_mma_launch(0, mw, umax, hidden, inter, B.xb_x, B.xs_x, 0, B.act, st));
        prof_end("experts.gateup");
        K3_TRY(xsplit(B.xb_a, B.xs_a, B.act, inter, TK, inter, st));
        prof_begin("experts.down");
        K3_TRY(mxfp4_mma_launch(1, mw, umax, inter, hidden, B.xb_a, B.xs_a, 1, B.contrib, st));
        prof_end("experts.down");
        return K3D_OK;
    }
    prof_begin("experts.gateup");
    K3_TRY(launch_gate_up(B.act, x, mw, hidden, inter, umax, st));
    prof_end("experts.gateup");
    prof_begin("experts.down");
    K3_TRY(launch_down(B.contrib, B.act, mw, hidden, inter, umax, st));
    prof_end("experts.down");
    return K3D_OK;
}

// Workspace carve-up for k3d_moe_swiglu.
struct MoeWs {
    int *idx; float *wts; void *router; int *n_active; int *act_expert; int *act_off;
    int *assign; float *sh_act; float *sh_out;
    ExpertBufs eb;
    size_t total;
};

// The expert buffers of run_experts for T token vectors and TK assignments.
template <class Take>
static void expert_bufs_layout(ExpertBufs &eb, const K3dMoeShape *s, size_t T, size_t TK, Take &take)
{
    eb.act = (float *)take(TK * s->inter * sizeof(float));
    eb.contrib = (float *)take(TK * s->hidden * sizeof(float));
    eb.xb_x = (__half *)take(T * 2 * s->hidden * sizeof(__half));
    eb.xs_x = (float *)take(T * sizeof(float));
    eb.xb_a = (__half *)take(TK * 2 * s->inter * sizeof(__half));
    eb.xs_a = (float *)take(TK * sizeof(float));
    if (umma_eligible(s->hidden, s->inter, (int)TK, s->expert_layout)) {
        // the grouped pass keeps one slice per K chunk at any count
        const bool grp = grouped_eligible(s->hidden, s->inter, (int)TK, s->expert_layout);
        const size_t cap_gu = grp ? (size_t)s->hidden / 512 : (size_t)umma_ks_cap(s->hidden, (int)TK);
        const size_t cap_d = grp ? (size_t)s->inter / 512 : (size_t)umma_ks_cap(s->inter, (int)TK);
        eb.bq_x = (uint8_t *)take(T * umma_bq_bytes(s->hidden));
        eb.bs_x = (uint8_t *)take(T * umma_bs_bytes(s->hidden));
        eb.bq_a = (uint8_t *)take(TK * umma_bq_bytes(s->inter));
        eb.bs_a = (uint8_t *)take(TK * umma_bs_bytes(s->inter));
        eb.part_gu = (float *)take(cap_gu * TK * 2 * s->inter * sizeof(float));
        eb.part_d = (float *)take(cap_d * TK * s->hidden * sizeof(float));
        if (s->expert_layout == 1 && !grp) {
            eb.fcnt_n = (int)umma_fused_cnt_ints((int)TK, s->inter);
            eb.fcnt = (int *)take((size_t)eb.fcnt_n * sizeof(int));
        } else {
            eb.fcnt = nullptr;
            eb.fcnt_n = 0;
        }
    } else {
        eb.bq_x = eb.bs_x = eb.bq_a = eb.bs_a = nullptr;
        eb.part_gu = eb.part_d = nullptr;
        eb.fcnt = nullptr;
        eb.fcnt_n = 0;
    }
    if (grouped_eligible(s->hidden, s->inter, (int)TK, s->expert_layout)) {
        // at most one group per assignment
        eb.bqg_x = (uint8_t *)take(TK * umma_bq_group_bytes(s->hidden));
        eb.bsg_x = (uint8_t *)take(TK * umma_bs_bytes(s->hidden));
        eb.bqg_a = (uint8_t *)take(TK * umma_bq_group_bytes(s->inter));
        eb.bsg_a = (uint8_t *)take(TK * umma_bs_bytes(s->inter));
        eb.grp.ng = (int *)take(16);
        eb.grp.p0 = (int *)take(TK * sizeof(int));
        eb.grp.n = (int *)take(TK * sizeof(int));
        eb.grp.e = (int *)take(TK * sizeof(int));
        eb.grp.pos_of = (int *)take(TK * sizeof(int));
    } else {
        eb.bqg_x = eb.bsg_x = eb.bqg_a = eb.bsg_a = nullptr;
        eb.grp = UmmaGroups{nullptr, nullptr, nullptr, nullptr, nullptr};
    }
}

static MoeWs moe_ws_layout(const K3dMoeShape *s, int T, void *base)
{
    MoeWs L;
    const size_t TK = (size_t)T * s->topk;
    size_t off = 0;
    char *b = (char *)base;
    auto take = [&](size_t bytes) { char *p = b + off; off += align256(bytes); return (void *)p; };
    L.idx = (int *)take(TK * sizeof(int));
    L.wts = (float *)take(TK * sizeof(float));
    L.router = take(router_ws_bytes(T, s->n_experts));
    L.n_active = (int *)take(4 * sizeof(int));
    L.act_expert = (int *)take((size_t)s->n_experts * sizeof(int));
    L.act_off = (int *)take(((size_t)s->n_experts + 1) * sizeof(int));
    L.assign = (int *)take(TK * sizeof(int));
    L.sh_act = (float *)take((size_t)T * (s->shared_inter > 0 ? s->shared_inter : 1) * sizeof(float));
    L.sh_out = (float *)take((size_t)T * s->hidden * sizeof(float));
    expert_bufs_layout(L.eb, s, (size_t)T, TK, take);
    L.total = off;
    return L;
}

static int check_shape(const K3dMoeShape *s, int T)
{
    if (!s) return fail(K3D_EINVAL, "null MoE shape");
    if (T < 1) return fail(K3D_EINVAL, "MoE T=%d", T);
    if (s->hidden % 32 || s->inter % 32 || s->hidden > 8192 || s->inter > 8192)
        return fail(K3D_EINVAL, "MoE hidden=%d inter=%d must be multiples of 32 up to 8192",
                    s->hidden, s->inter);
    if (s->topk < 1 || s->topk > K3_MAX_TOPK || s->topk > s->n_experts)
        return fail(K3D_EBOUND, "MoE topk=%d (n_experts=%d, max %d)", s->topk, s->n_experts,
                    K3_MAX_TOPK);
    if (s->expert_lo < 0 || s->expert_hi > s->n_experts || s->expert_lo > s->expert_hi)
        return fail(K3D_EINVAL, "MoE expert range [%d, %d)", s->expert_lo, s->expert_hi);
    if (s->n_experts > 8192) return fail(K3D_EINVAL, "MoE n_experts=%d > 8192", s->n_experts);
    if (s->shared_inter > 0 && (s->shared_inter % 8))
        return fail(K3D_EINVAL, "shared_inter=%d must be a multiple of 8", s->shared_inter);
    if (s->expert_layout != 0 && s->expert_layout != 1)
        return fail(K3D_EINVAL, "expert_layout=%d (0 checkpoint, 1 tiled)", s->expert_layout);
    if (s->expert_layout == 1 && !umma_shapes(s->hidden, s->inter))
        return fail(K3D_EINVAL, "tiled experts need hidden=%d and inter=%d multiples of 512",
                    s->hidden, s->inter);
    return K3D_OK;
}

// pinned host copy of the last call's active-expert count (copied asynchronously, so the
// value survives the caller freeing its workspace)
static int *g_last_unique_pinned = nullptr;
static bool g_last_unique_valid = false;

// Single-expert workspace: the mma.sync / CUDA-core buffers, then the tcgen05 ones.
struct ExpertWs {
    ExpertBufs eb;
    size_t total;
};

static ExpertWs expert_ws_layout(int hidden, int inter, void *base)
{
    ExpertWs L;
    size_t off = 0;
    char *b = (char *)base;
    auto take = [&](size_t bytes) { char *p = b + off; off += align256(bytes); return (void *)p; };
    L.eb.act = (float *)take((size_t)inter * sizeof(float));
    L.eb.contrib = nullptr;
    L.eb.xb_x = (__half *)take((size_t)2 * hidden * sizeof(__half));
    L.eb.xs_x = (float *)take(sizeof(float));
    L.eb.xb_a = (__half *)take((size_t)2 * inter * sizeof(__half));
    L.eb.xs_a = (float *)take(sizeof(float));
    if (umma_eligible(hidden, inter, 1, 0)) {
        L.eb.bq_x = (uint8_t *)take(umma_bq_bytes(hidden));
        L.eb.bs_x = (uint8_t *)take(umma_bs_bytes(hidden));
        L.eb.bq_a = (uint8_t *)take(umma_bq_bytes(inter));
        L.eb.bs_a = (uint8_t *)take(umma_bs_bytes(inter));
        L.eb.part_gu = (float *)take((size_t)(hidden / 512) * 2 * inter * sizeof(float));
        L.eb.part_d = (float *)take((size_t)(inter / 512) * hidden * sizeof(float));
    } else {
        L.eb.bq_x = L.eb.bs_x = L.eb.bq_a = L.eb.bs_a = nullptr;
        L.eb.part_gu = L.eb.part_d = nullptr;
    }
    L.eb.bqg_x = L.eb.bsg_x = L.eb.bqg_a = L.eb.bsg_a = nullptr;   // one expert: no groups
    L.eb.grp = UmmaGroups{nullptr, nullptr, nullptr, nullptr, nullptr};
    L.total = off;
    return L;
}

// ---- Mode A: all-to-all expert parallelism ------------------------------------------
// Every rank routes ITS OWN tokens; the row of each (token, slot) assignment goes to the
// rank of its expert (expert e on rank e / (n_experts / nranks)), which runs its local
// experts over everything it received, one assignment per row, and sends the results
// back; the tokens' rank sums them in top-k order with the shared expert. Rows travel as
// fp32, so a token's result does not depend on where its experts ran.

// Host dispatch plan: cnt[r] rows for rank r, its rows from off[r] on in the send buffer,
// each rank's rows in assignment order; pos[a] = row of assignment a. -1 on a bad id.
static int a2a_plan_host(const int *idx, int TK, int n_experts, int nranks, int *cnt, int *off, int *pos)
{
    if (nranks < 1 || n_experts < nranks || n_experts % nranks) return -1;
    const int per = n_experts / nranks;
    for (int r = 0; r < nranks; r++) cnt[r] = 0;
    for (int a = 0; a < TK; a++) {
        if (idx[a] < 0 || idx[a] >= n_experts) return -1;
        cnt[idx[a] / per]++;
    }
    for (int r = 0, o = 0; r < nranks; r++) { off[r] = o; o += cnt[r]; }
    std::vector<int> cur(off, off + nranks);
    for (int a = 0; a < TK; a++) pos[a] = cur[idx[a] / per]++;
    return 0;
}

// Send rows: row pos[a] = x[a / K], and its expert id. grid TK, 256 threads.
__global__ void k_a2a_pack(float *sendbuf, int *send_ids, const float *x, const int *idx, const int *pos,
                           int K, int hidden)
{
    pdl_wait();
    pdl_trigger();
    const int a = blockIdx.x;
    const int row = pos[a];
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)(a / K) * hidden);
    float4 *dst = reinterpret_cast<float4 *>(sendbuf + (size_t)row * hidden);
    for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) send_ids[row] = idx[a];
}

// dst[a] = src[pos_of[a]] (rows of hidden floats). grid = rows, 256 threads.
__global__ void k_gather_rows(float *dst, const float *src, const int *pos_of, int hidden)
{
    pdl_wait();
    pdl_trigger();
    const int a = blockIdx.x;
    const float4 *s4 = reinterpret_cast<const float4 *>(src + (size_t)__ldcg(pos_of + a) * hidden);
    float4 *d4 = reinterpret_cast<float4 *>(dst + (size_t)a * hidden);
    for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) d4[i] = __ldcg(s4 + i);
}

// out[t] (+)= sum over slots k, in top-k order, of w[t][k] * back[pos[t K + k]], then the
// shared expert: the arithmetic of k_moe_combine. grid (ceil(hidden / 256), T).
__global__ void k_a2a_combine(float *out, const float *back, const int *pos, const float *wts,
                              const float *sh_out, int hidden, int K, int accumulate)
{
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.y;
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= hidden) return;
    float acc = 0.0f;
    for (int k = 0; k < K; k++) {
        const int a = t * K + k;
        acc = __fadd_rn(acc, __fmul_rn(wts[a], back[(size_t)pos[a] * hidden + r]));
    }
    if (sh_out) acc = __fadd_rn(acc, sh_out[(size_t)t * hidden + r]);
    float *o = out + (size_t)t * hidden + r;
    *o = accumulate ? __fadd_rn(*o, acc) : acc;
}

// Device-planned dispatch (k3d_moe_swiglu_a2a_dev): send row (r, p) = x[a / K] for the
// p-th assignment a (in assignment order) whose expert rank r owns, in rank r's region of
// cap = t_max * topk rows; meta[r][0] = that region's row count, meta[r][1 + p] = the
// expert id; pos[a] = r * cap + p. CTA a counts the earlier assignments bound for its rank
// itself (TK <= a few thousand), CTA 0 also writes every region's count. grid TK, 256
// threads.
__global__ void k_a2a_pack_dev(float *send, int *meta, int *pos, const float *x, const int *idx, int TK,
                               int K, int hidden, int per, int nranks, int cap)
{
    pdl_wait();
    pdl_trigger();
    __shared__ int s_cnt[8 * 32];
    const int a = blockIdx.x, tid = threadIdx.x;
    const int e = idx[a];
    const bool ok = e >= 0 && e < per * nranks;
    const int r = ok ? e / per : 0;
    int c = 0;
    for (int b = tid; b < a; b += blockDim.x) {
        const int eb = idx[b];
        c += (eb >= 0 && eb < per * nranks ? eb / per : 0) == r;
    }
    c = __reduce_add_sync(0xffffffffu, c);
    if ((tid & 31) == 0) s_cnt[tid >> 5] = c;
    if (a == 0)
        for (int q = tid; q < nranks; q += blockDim.x) s_cnt[32 + q] = 0;
    __syncthreads();
    int p = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) p += s_cnt[w];
    if (a == 0) {
        for (int b = tid; b < TK; b += blockDim.x) {
            const int eb = idx[b];
            atomicAdd(&s_cnt[32 + (eb >= 0 && eb < per * nranks ? eb / per : 0)], 1);
        }
        __syncthreads();
        for (int q = tid; q < nranks; q += blockDim.x) meta[(size_t)q * (cap + 1)] = s_cnt[32 + q];
    }
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)(a / K) * hidden);
    float4 *dst = reinterpret_cast<float4 *>(send + ((size_t)r * cap + p) * hidden);
    for (int i = tid; i < hidden / 4; i += blockDim.x) dst[i] = src[i];
    if (tid == 0) {
        meta[(size_t)r * (cap + 1) + 1 + p] = ok ? e : -1;
        pos[a] = r * cap + p;
    }
}

// Received rows: ids[s * cap + p] = the expert id of row p from rank s, or -1 past that
// rank's count (skipped by the grouping). grid ceil(nranks * cap / 256), 256 threads.
__global__ void k_a2a_mask_dev(int *ids, const int *meta, int nranks, int cap)
{
    pdl_wait();
    pdl_trigger();
    const int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= nranks * cap) return;
    const int s = a / cap, p = a % cap;
    const int *m = meta + (size_t)s * (cap + 1);
    ids[a] = p < m[0] ? m[1 + p] : -1;
}

// dst[a] = src[pos_of[a]] for the rows with an expert id (ids[a] >= 0); zero rows for the
// others (their pos_of is not written). grid = rows, 256 threads.
__global__ void k_gather_rows_masked(float *dst, const float *src, const int *pos_of, const int *ids, int hidden)
{
    pdl_wait();
    pdl_trigger();
    const int a = blockIdx.x;
    float4 *d4 = reinterpret_cast<float4 *>(dst + (size_t)a * hidden);
    if (__ldcg(ids + a) < 0) {
        for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) d4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    const float4 *s4 = reinterpret_cast<const float4 *>(src + (size_t)__ldcg(pos_of + a) * hidden);
    for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) d4[i] = __ldcg(s4 + i);
}

// Workspace of k3d_moe_swiglu_a2a: at most t_max tokens on any rank, so a rank receives at
// most nranks * t_max * topk rows. The device-planned form uses fixed regions of cap =
// t_max * topk rows per rank in its send, receive and return buffers.
struct A2aWs {
    int *idx; float *wts; void *router; float *sh_act, *sh_out;
    int *pos, *cnt_s, *cnt_r;
    float *sendbuf, *recvbuf, *back;
    int *send_ids, *recv_ids;
    int *n_active, *act_expert, *act_off, *assign;
    float *send_dev, *back_dev;
    int *meta_s, *meta_r;
    ExpertBufs eb;
    size_t total;
};

static A2aWs a2a_ws_layout(const K3dMoeShape *s, int t_max, int nranks, void *base)
{
    A2aWs L;
    const size_t TK = (size_t)t_max * s->topk, R = (size_t)nranks * TK;
    size_t off = 0;
    char *b = (char *)base;
    auto take = [&](size_t bytes) { char *p = b + off; off += align256(bytes); return (void *)p; };
    L.idx = (int *)take(TK * sizeof(int));
    L.wts = (float *)take(TK * sizeof(float));
    L.router = take(router_ws_bytes(t_max, s->n_experts));
    L.sh_act = (float *)take((size_t)t_max * (s->shared_inter > 0 ? s->shared_inter : 1) * sizeof(float));
    L.sh_out = (float *)take((size_t)t_max * s->hidden * sizeof(float));
    L.pos = (int *)take(TK * sizeof(int));
    L.cnt_s = (int *)take((size_t)nranks * sizeof(int));
    L.cnt_r = (int *)take((size_t)nranks * sizeof(int));
    L.sendbuf = (float *)take(TK * s->hidden * sizeof(float));
    L.send_ids = (int *)take(TK * sizeof(int));
    L.recvbuf = (float *)take(R * s->hidden * sizeof(float));
    L.recv_ids = (int *)take(R * sizeof(int));
    L.back = (float *)take(TK * s->hidden * sizeof(float));
    L.n_active = (int *)take(4 * sizeof(int));
    L.act_expert = (int *)take((size_t)s->n_experts * sizeof(int));
    L.act_off = (int *)take(((size_t)s->n_experts + 1) * sizeof(int));
    L.assign = (int *)take(R * sizeof(int));
    L.send_dev = (float *)take(R * s->hidden * sizeof(float));
    L.back_dev = (float *)take(R * s->hidden * sizeof(float));
    L.meta_s = (int *)take((size_t)nranks * (TK + 1) * sizeof(int));
    L.meta_r = (int *)take((size_t)nranks * (TK + 1) * sizeof(int));
    expert_bufs_layout(L.eb, s, R, R, take);
    L.total = off;
    return L;
}

// Pinned host scratch of the plan (grows; Mode A synchronises the host anyway).
static int *a2a_host_ints(size_t n)
{
    static int *buf = nullptr;
    static size_t cap = 0;
    if (n <= cap) return buf;
    if (buf) cudaFreeHost(buf);
    buf = nullptr;
    cap = 0;
    if (cudaMallocHost(&buf, n * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        fail(K3D_ENOMEM, "moe a2a: %zu pinned host ints", n);
        return nullptr;
    }
    cap = n;
    return buf;
}

}  // namespace k3

using namespace k3;

extern "C" {

int k3d_a2a_plan(const int *idx, int TK, int n_experts, int nranks, int *cnt, int *off, int *pos)
{
    if (!idx || !cnt || !off || !pos || TK < 0) return fail(K3D_EINVAL, "k3d_a2a_plan null pointer");
    if (a2a_plan_host(idx, TK, n_experts, nranks, cnt, off, pos))
        return fail(K3D_EINVAL, "k3d_a2a_plan: %d experts over %d ranks, or an expert id out of range",
                    n_experts, nranks);
    return K3D_OK;
}

size_t k3d_moe_a2a_ws_bytes(const K3dMoeShape *s, int t_max, int nranks)
{
    if (!s || t_max < 1 || nranks < 1) return 0;
    return a2a_ws_layout(s, t_max, nranks, nullptr).total + 256;
}

int k3d_moe_swiglu_a2a(float *out, const float *x, const K3dMoeW *w, const K3dMoeShape *s, int T,
                       int t_max, int accumulate, int *idx, float *wts, void *ws, size_t ws_bytes)
{
    K3_TRY(ensure_ctx());
    K3_TRY(check_shape(s, T));
    const int G = k3d_ep_size(), rank = k3d_ep_rank();
    if (!out || !x || !w || !ws || !w->router_w || !w->experts)
        return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a null pointer");
    if (T > t_max) return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a: T=%d above t_max=%d", T, t_max);
    if (s->n_experts % G) return fail(K3D_EINVAL, "moe a2a: %d experts over %d ranks", s->n_experts, G);
    const int per = s->n_experts / G;
    if (s->expert_lo != rank * per || s->expert_hi != (rank + 1) * per)
        return fail(K3D_EINVAL, "moe a2a: rank %d owns experts [%d, %d), not [%d, %d)", rank, rank * per,
                    (rank + 1) * per, s->expert_lo, s->expert_hi);
    if (s->shared_inter > 0 && s->add_shared && (!w->sh_gate || !w->sh_up || !w->sh_down))
        return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a shared expert weights missing");
    if (ws_bytes < k3d_moe_a2a_ws_bytes(s, t_max, G)) return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a workspace too small");
    if (((uintptr_t)x | (uintptr_t)ws) & 15u) return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a alignment");
    cudaStream_t st = stream();
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs != cudaStreamCaptureStatusNone)
        return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a synchronises the host and cannot be captured");
    A2aWs L = a2a_ws_layout(s, t_max, G, ws);
    const int K = s->topk, TK = T * K;
    int *I = idx ? idx : L.idx;
    float *Wt = wts ? wts : L.wts;
    int *h = a2a_host_ints((size_t)2 * TK + 4 * (size_t)G + 4);
    if (!h) return k3d_status();
    int *h_idx = h, *h_pos = h + TK, *h_cnt = h + 2 * TK, *h_off = h_cnt + G, *h_rcnt = h_off + G,
        *h_roff = h_rcnt + G;

    // the shared expert of this rank's tokens, on the side stream (joined before the combine)
    const bool shared = s->shared_inter > 0 && s->add_shared;
    cudaStream_t sst = (!profiling() && side_stream()) ? side_stream() : st;
    if (shared) {
        if (sst != st && (cudaEventRecord(side_event(0), st) != cudaSuccess ||
                          cudaStreamWaitEvent(sst, side_event(0), 0) != cudaSuccess))
            return fail(K3D_ECUDA, "moe a2a: fork to the side stream");
        prof_begin("moe.shared");
        K3_TRY(gemv_bf16_swiglu(L.sh_act, x, w->sh_gate, w->sh_up, s->hidden, s->shared_inter, T, sst));
        K3_TRY(gemv_bf16(L.sh_out, L.sh_act, w->sh_down, s->shared_inter, s->hidden, T, 0, sst));
        prof_end("moe.shared");
        if (sst != st && cudaEventRecord(side_event(1), sst) != cudaSuccess)
            return fail(K3D_ECUDA, "moe a2a: side stream join event");
    }
    prof_begin("moe.router");
    K3_TRY(router_bf16(I, Wt, x, w->router_w, w->router_bias, T, s->hidden, s->n_experts, K, s->renorm,
                       s->routed_scale, L.router, st));
    prof_end("moe.router");

    // plan on the host: the routing decides how many rows go to each rank
    prof_begin("ep.dispatch");
    if (cudaMemcpyAsync(h_idx, I, (size_t)TK * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(K3D_ECUDA, "moe a2a: routing to the host");
    K3_TRY(device_flag_status());
    if (a2a_plan_host(h_idx, TK, s->n_experts, G, h_cnt, h_off, h_pos))
        return fail(K3D_EBOUND, "moe a2a: expert id out of range");
    if (cudaMemcpyAsync(L.pos, h_pos, (size_t)TK * sizeof(int), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(L.cnt_s, h_cnt, (size_t)G * sizeof(int), cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail(K3D_ECUDA, "moe a2a: plan to the device");
    // the row counts every rank sends here
    {
        std::vector<size_t> c4(G, sizeof(int)), o4(G);
        for (int r = 0; r < G; r++) o4[r] = (size_t)r * sizeof(int);
        K3_TRY(ep_exchange(L.cnt_s, c4.data(), o4.data(), L.cnt_r, c4.data(), o4.data(), st));
    }
    if (cudaMemcpyAsync(h_rcnt, L.cnt_r, (size_t)G * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(K3D_ECUDA, "moe a2a: receive counts to the host");
    long long R = 0;
    for (int r = 0; r < G; r++) {
        if (h_rcnt[r] < 0) return fail(K3D_EBOUND, "moe a2a: rank %d sends %d rows", r, h_rcnt[r]);
        h_roff[r] = (int)R;
        R += h_rcnt[r];
    }
    if (R > (long long)G * t_max * K)
        return fail(K3D_EBOUND, "moe a2a: %lld rows received, room for %lld", R, (long long)G * t_max * K);
    if (TK > 0) {
        launch_pdl(k_a2a_pack, dim3(TK), dim3(256), 0, st, L.sendbuf, L.send_ids, x, (const int *)I,
                   (const int *)L.pos, K, s->hidden);
        note_launch();
        K3_TRY(check_launch("moe a2a pack"));
    }
    const size_t rowb = (size_t)s->hidden * sizeof(float);
    std::vector<size_t> sb(G), so(G), rb(G), ro(G), si(G), soi(G), ri(G), roi(G);
    for (int r = 0; r < G; r++) {
        sb[r] = (size_t)h_cnt[r] * rowb;   so[r] = (size_t)h_off[r] * rowb;
        rb[r] = (size_t)h_rcnt[r] * rowb;  ro[r] = (size_t)h_roff[r] * rowb;
        si[r] = (size_t)h_cnt[r] * 4;      soi[r] = (size_t)h_off[r] * 4;
        ri[r] = (size_t)h_rcnt[r] * 4;     roi[r] = (size_t)h_roff[r] * 4;
    }
    K3_TRY(ep_exchange(L.send_ids, si.data(), soi.data(), L.recv_ids, ri.data(), roi.data(), st));
    K3_TRY(ep_exchange(L.sendbuf, sb.data(), so.data(), L.recvbuf, rb.data(), ro.data(), st));
    prof_end("ep.dispatch");

    // this rank's experts over the rows it received: one assignment per row
    const float *ybuf = L.recvbuf;    // unused when R = 0
    if (R > 0) {
        const size_t smem = 2 * (size_t)s->n_experts * sizeof(int);
        launch_pdl(k_moe_prep, dim3(1), dim3(1024), smem, st, (const int *)L.recv_ids, (int)R, s->n_experts,
                   s->expert_lo, s->expert_hi, L.n_active, L.act_expert, L.act_off, L.assign, L.eb.fcnt,
                   L.eb.fcnt_n);
        note_launch();
        K3_TRY(check_launch("moe a2a prep"));
        MoeWork mw{};
        mw.table = w->experts;
        mw.n_active = L.n_active;
        mw.act_expert = L.act_expert;
        mw.act_off = L.act_off;
        mw.assign = L.assign;
        mw.K = 1;
        mw.n_experts = s->n_experts;
        ExpertOut O{L.eb.contrib, 1, 0};
        const int umax = (int)std::min<long long>(R, per);
        prof_begin("moe.experts");
        K3_TRY(run_experts(mw, L.recv_ids, L.n_active + 1, umax, L.recvbuf, (int)R, (int)R, s->hidden,
                           s->inter, s->expert_layout, L.eb, O, st));
        prof_end("moe.experts");
        ybuf = O.contrib;
        if (O.pos_of) {
            // grouped pass: K slices by position; summed, then gathered into received-row
            // order (the rows received are no longer needed: their buffer takes the result)
            const float *src = O.contrib;
            if (O.ks > 1) {
                K3_TRY(umma_slice_sum(L.eb.contrib, O.contrib, O.ks, O.slice, (int)(R * s->hidden), st));
                src = L.eb.contrib;
            }
            launch_pdl(k_gather_rows, dim3((unsigned)R), dim3(256), 0, st, L.recvbuf, src, O.pos_of, s->hidden);
            note_launch();
            K3_TRY(check_launch("moe a2a gather"));
            ybuf = L.recvbuf;
        } else if (O.ks > 1) {
            K3_TRY(umma_slice_sum(L.eb.contrib, O.contrib, O.ks, O.slice, (int)(R * s->hidden), st));
            ybuf = L.eb.contrib;
        }
    }
    // results back to the tokens' ranks, into the rows they were sent from
    prof_begin("ep.combine");
    K3_TRY(ep_exchange(ybuf, rb.data(), ro.data(), L.back, sb.data(), so.data(), st));
    prof_end("ep.combine");
    if (shared && sst != st && cudaStreamWaitEvent(st, side_event(1), 0) != cudaSuccess)
        return fail(K3D_ECUDA, "moe a2a: join from the side stream");
    dim3 grid((s->hidden + 255) / 256, T);
    launch_pdl(k_a2a_combine, dim3(grid), dim3(256), 0, st, out, (const float *)L.back, (const int *)L.pos,
               (const float *)Wt, shared ? (const float *)L.sh_out : nullptr, s->hidden, K, accumulate);
    note_launch();
    return check_launch("moe a2a combine");
}

size_t k3d_expert_ws_bytes(int hidden, int inter)
{
    return expert_ws_layout(hidden, inter, nullptr).total + 256;
}

int k3d_set_expert_kernel(int kind)
{
    if (kind < 0 || kind > 4) return fail(K3D_EINVAL, "k3d_set_expert_kernel(%d): 0 to 4", kind);
    g_expert_kernel = kind;
    return K3D_OK;
}

int k3d_expert_swiglu(float *y, const float *x, const K3ExpertQ *e, int hidden, int inter,
                      void *ws, size_t ws_bytes)
{
    K3_TRY(ensure_ctx());
    if (!y || !x || !e || !ws) return fail(K3D_EINVAL, "k3d_expert_swiglu null pointer");
    if (hidden % 32 || inter % 32 || hidden > 8192 || inter > 8192)
        return fail(K3D_EINVAL, "k3d_expert_swiglu hidden=%d inter=%d", hidden, inter);
    if (ws_bytes < k3d_expert_ws_bytes(hidden, inter))
        return fail(K3D_EINVAL, "k3d_expert_swiglu workspace too small");
    const uintptr_t al = (uintptr_t)e->p1 | (uintptr_t)e->p3 | (uintptr_t)e->p2 | (uintptr_t)e->s1 |
                         (uintptr_t)e->s3 | (uintptr_t)e->s2 | (uintptr_t)x | (uintptr_t)ws;
    if (al & 15u) return fail(K3D_EINVAL, "k3d_expert_swiglu pointers must be 16-byte aligned");
    MoeWork w{};
    w.single = *e;
    w.single_mode = 1;
    w.ntok_single = 1;
    w.K = 1;
    ExpertWs L = expert_ws_layout(hidden, inter, ws);
    L.eb.contrib = y;      // the contribution of the single assignment is y itself
    cudaStream_t s = stream();
    prof_begin("expert.swiglu");
    ExpertOut O;
    K3_TRY(run_experts(w, nullptr, nullptr, 1, x, 1, 1, hidden, inter, 0, L.eb, O, s));
    if (O.contrib != y) K3_TRY(umma_slice_sum(y, O.contrib, O.ks, O.slice, hidden, s));
    prof_end("expert.swiglu");
    return K3D_OK;
}

size_t k3d_moe_ws_bytes(const K3dMoeShape *s, int T)
{
    if (!s || T < 1) return 0;
    return moe_ws_layout(s, T, nullptr).total + 256;
}

int k3d_moe_swiglu(float *out, const float *x, const K3dMoeW *w, const K3dMoeShape *s, int T,
                   int accumulate, int *idx, float *wts, void *ws, size_t ws_bytes)
{
    K3_TRY(ensure_ctx());
    K3_TRY(check_shape(s, T));
    if (!out || !x || !w || !ws || !w->router_w || !w->experts)
        return fail(K3D_EINVAL, "k3d_moe_swiglu null pointer");
    if (s->shared_inter > 0 && s->add_shared && (!w->sh_gate || !w->sh_up || !w->sh_down))
        return fail(K3D_EINVAL, "k3d_moe_swiglu shared expert weights missing");
    if (ws_bytes < k3d_moe_ws_bytes(s, T)) return fail(K3D_EINVAL, "k3d_moe_swiglu workspace too small");
    if (((uintptr_t)x | (uintptr_t)ws) & 15u) return fail(K3D_EINVAL, "k3d_moe_swiglu alignment");
    MoeWs L = moe_ws_layout(s, T, ws);
    cudaStream_t st = stream();
    int *I = idx ? idx : L.idx;
    float *Wt = wts ? wts : L.wts;
    const int K = s->topk;
    const int TK = T * K;

    // Neither the tcgen05 B operand of x nor the shared expert depends on the router: both
    // run on the side stream, in parallel with routing (a parallel branch when the stream
    // is captured into a graph); the routed experts wait for the split, the combine for the
    // shared expert. With the section timers on they run in line, so that each section's
    // time is measured on its own.
    const bool shared = s->shared_inter > 0 && s->add_shared;
    const int umax = TK < (s->expert_hi - s->expert_lo) ? TK : (s->expert_hi - s->expert_lo);
    const bool early_split = umax > 0 && use_umma(L.eb, s->hidden, s->inter, TK, s->expert_layout) &&
                             !use_grouped(L.eb, TK, s->expert_layout, s->hidden, s->inter);
    cudaStream_t sst = (!profiling() && side_stream()) ? side_stream() : st;
    if ((shared || early_split) && sst != st) {
        if (cudaEventRecord(side_event(0), st) != cudaSuccess ||
            cudaStreamWaitEvent(sst, side_event(0), 0) != cudaSuccess)
            return fail(K3D_ECUDA, "moe: fork to the side stream");
    }
    if (early_split) {
        K3_TRY(umma_bsplit(L.eb.bq_x, L.eb.bs_x, x, s->hidden, T, s->hidden, sst));
        if (sst != st && cudaEventRecord(side_event(2), sst) != cudaSuccess)
            return fail(K3D_ECUDA, "moe: side stream split event");
    }
    if (shared) {
        prof_begin("moe.shared");
        K3_TRY(gemv_bf16_swiglu(L.sh_act, x, w->sh_gate, w->sh_up, s->hidden, s->shared_inter, T, sst));
        K3_TRY(gemv_bf16(L.sh_out, L.sh_act, w->sh_down, s->shared_inter, s->hidden, T, 0, sst));
        prof_end("moe.shared");
        if (sst != st && cudaEventRecord(side_event(1), sst) != cudaSuccess)
            return fail(K3D_ECUDA, "moe: side stream join event");
    }
    prof_begin("moe.router");
    RouterGroup grp{L.n_active, L.act_expert, L.act_off, L.assign, s->expert_lo, s->expert_hi, 0};
    grp.zero = L.eb.fcnt;
    grp.nzero = L.eb.fcnt_n;
    K3_TRY(router_bf16(I, Wt, x, w->router_w, w->router_bias, T, s->hidden, s->n_experts, K,
                       s->renorm, s->routed_scale, L.router, st, &grp));
    prof_end("moe.router");
    if (!grp.done) {
        const size_t smem = 2 * (size_t)s->n_experts * sizeof(int);
        launch_pdl(k_moe_prep, dim3(1), dim3(1024), smem, st, I, TK, s->n_experts, s->expert_lo, s->expert_hi,
                                          L.n_active, L.act_expert, L.act_off, L.assign, L.eb.fcnt, L.eb.fcnt_n);
        note_launch();
        K3_TRY(check_launch("moe prep"));
    }
    MoeWork mw{};
    mw.table = w->experts;
    mw.n_active = L.n_active;
    mw.act_expert = L.act_expert;
    mw.act_off = L.act_off;
    mw.assign = L.assign;
    mw.K = K;
    mw.n_experts = s->n_experts;
    ExpertOut O{L.eb.contrib, 1, 0};
    if (early_split && sst != st && cudaStreamWaitEvent(st, side_event(2), 0) != cudaSuccess)
        return fail(K3D_ECUDA, "moe: join of the split from the side stream");
    if (umax > 0) {
        prof_begin("moe.experts");
        K3_TRY(run_experts(mw, I, L.n_active + 1, umax, x, T, TK, s->hidden, s->inter,
                           s->expert_layout, L.eb, O, st, early_split, true));
        prof_end("moe.experts");
    }
    if (shared && sst != st && cudaStreamWaitEvent(st, side_event(1), 0) != cudaSuccess)
        return fail(K3D_ECUDA, "moe: join from the side stream");
    dim3 grid((s->hidden + 255) / 256, T);
    launch_pdl(k_moe_combine, dim3(grid), dim3(256), 0, st, out, O.contrib, O.ks, O.slice, I, Wt, shared ? L.sh_out : nullptr,
                                        s->hidden, K, s->expert_lo, s->expert_hi, accumulate, O.pos_of,
                                        umax > 0 ? 1 : 0);
    note_launch();
    K3_TRY(check_launch("moe combine"));
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs == cudaStreamCaptureStatusNone) {
        if (!g_last_unique_pinned && cudaMallocHost(&g_last_unique_pinned, sizeof(int)) != cudaSuccess) {
            cudaGetLastError();
            g_last_unique_pinned = nullptr;
        }
        if (g_last_unique_pinned) {
            cudaMemcpyAsync(g_last_unique_pinned, L.n_active, sizeof(int), cudaMemcpyDeviceToHost, st);
            g_last_unique_valid = true;
        }
    }
    return K3D_OK;
}

int k3d_moe_last_unique(void)
{
    if (!g_last_unique_valid || !g_last_unique_pinned) return -1;
    cudaStreamSynchronize(stream());
    return *g_last_unique_pinned;
}

}  // extern "C"

// Mode A planned on the device: the same rows and arithmetic as k3d_moe_swiglu_a2a, but the
// dispatch plan (which rank, which row) is computed by k_a2a_pack_dev and every exchange
// moves fixed regions of cap = T * topk rows per pair, whatever the routing, so no size
// reaches the host and the whole layer can be captured into a CUDA graph. The price is
// traffic: each pair exchanges cap rows both ways instead of the rows routed to it.
extern "C" int k3d_moe_swiglu_a2a_dev(float *out, const float *x, const K3dMoeW *w, const K3dMoeShape *s,
                                      int T, int accumulate, int *idx, float *wts, void *ws, size_t ws_bytes)
{
    K3_TRY(ensure_ctx());
    K3_TRY(check_shape(s, T));
    const int G = k3d_ep_size(), rank = k3d_ep_rank();
    if (!out || !x || !w || !ws || !w->router_w || !w->experts)
        return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a_dev null pointer");
    if (s->n_experts % G) return fail(K3D_EINVAL, "moe a2a: %d experts over %d ranks", s->n_experts, G);
    const int per = s->n_experts / G;
    if (s->expert_lo != rank * per || s->expert_hi != (rank + 1) * per)
        return fail(K3D_EINVAL, "moe a2a: rank %d owns experts [%d, %d), not [%d, %d)", rank, rank * per,
                    (rank + 1) * per, s->expert_lo, s->expert_hi);
    if (s->shared_inter > 0 && s->add_shared && (!w->sh_gate || !w->sh_up || !w->sh_down))
        return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a_dev shared expert weights missing");
    if (ws_bytes < k3d_moe_a2a_ws_bytes(s, T, G)) return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a_dev workspace too small");
    if (((uintptr_t)x | (uintptr_t)ws) & 15u) return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a_dev alignment");
    if (s->hidden % 4) return fail(K3D_EINVAL, "k3d_moe_swiglu_a2a_dev: hidden %% 4");
    cudaStream_t st = stream();
    A2aWs L = a2a_ws_layout(s, T, G, ws);
    const int K = s->topk, TK = T * K, cap = TK, R = G * cap;
    int *I = idx ? idx : L.idx;
    float *Wt = wts ? wts : L.wts;

    const bool shared = s->shared_inter > 0 && s->add_shared;
    cudaStream_t sst = (!profiling() && side_stream()) ? side_stream() : st;
    if (shared) {
        if (sst != st && (cudaEventRecord(side_event(0), st) != cudaSuccess ||
                          cudaStreamWaitEvent(sst, side_event(0), 0) != cudaSuccess))
            return fail(K3D_ECUDA, "moe a2a: fork to the side stream");
        prof_begin("moe.shared");
        K3_TRY(gemv_bf16_swiglu(L.sh_act, x, w->sh_gate, w->sh_up, s->hidden, s->shared_inter, T, sst));
        K3_TRY(gemv_bf16(L.sh_out, L.sh_act, w->sh_down, s->shared_inter, s->hidden, T, 0, sst));
        prof_end("moe.shared");
        if (sst != st && cudaEventRecord(side_event(1), sst) != cudaSuccess)
            return fail(K3D_ECUDA, "moe a2a: side stream join event");
    }
    prof_begin("moe.router");
    K3_TRY(router_bf16(I, Wt, x, w->router_w, w->router_bias, T, s->hidden, s->n_experts, K, s->renorm,
                       s->routed_scale, L.router, st));
    prof_end("moe.router");

    prof_begin("ep.dispatch");
    launch_pdl(k_a2a_pack_dev, dim3(TK), dim3(256), 0, st, L.send_dev, L.meta_s, L.pos, x, (const int *)I, TK, K,
               s->hidden, per, G, cap);
    note_launch();
    K3_TRY(check_launch("moe a2a pack"));
    const size_t rowb = (size_t)s->hidden * sizeof(float), metab = (size_t)(cap + 1) * sizeof(int);
    std::vector<size_t> rb(G, (size_t)cap * rowb), ro(G), mb(G, metab), mo(G);
    for (int r = 0; r < G; r++) { ro[r] = (size_t)r * cap * rowb; mo[r] = (size_t)r * metab; }
    K3_TRY(ep_exchange(L.meta_s, mb.data(), mo.data(), L.meta_r, mb.data(), mo.data(), st));
    K3_TRY(ep_exchange(L.send_dev, rb.data(), ro.data(), L.recvbuf, rb.data(), ro.data(), st));
    launch_pdl(k_a2a_mask_dev, dim3((R + 255) / 256), dim3(256), 0, st, L.recv_ids, (const int *)L.meta_r, G, cap);
    note_launch();
    K3_TRY(check_launch("moe a2a mask"));
    prof_end("ep.dispatch");

    // this rank's experts over the rows it may have received: one assignment per row, the
    // rows past a sender's count carry id -1 and stay out of the work list
    const size_t smem = 2 * (size_t)s->n_experts * sizeof(int);
    launch_pdl(k_moe_prep, dim3(1), dim3(1024), smem, st, (const int *)L.recv_ids, R, s->n_experts, s->expert_lo,
               s->expert_hi, L.n_active, L.act_expert, L.act_off, L.assign, L.eb.fcnt, L.eb.fcnt_n);
    note_launch();
    K3_TRY(check_launch("moe a2a prep"));
    MoeWork mw{};
    mw.table = w->experts;
    mw.n_active = L.n_active;
    mw.act_expert = L.act_expert;
    mw.act_off = L.act_off;
    mw.assign = L.assign;
    mw.K = 1;
    mw.n_experts = s->n_experts;
    ExpertOut O{L.eb.contrib, 1, 0};
    const int umax = std::min(R, per);
    prof_begin("moe.experts");
    K3_TRY(run_experts(mw, L.recv_ids, L.n_active + 1, umax, L.recvbuf, R, R, s->hidden, s->inter,
                       s->expert_layout, L.eb, O, st));
    prof_end("moe.experts");
    const float *ybuf = O.contrib;
    if (O.pos_of) {
        const float *src = O.contrib;
        if (O.ks > 1) {
            K3_TRY(umma_slice_sum(L.eb.contrib, O.contrib, O.ks, O.slice, (int)((size_t)R * s->hidden), st));
            src = L.eb.contrib;
        }
        launch_pdl(k_gather_rows_masked, dim3((unsigned)R), dim3(256), 0, st, L.recvbuf, src, O.pos_of,
                   (const int *)L.recv_ids, s->hidden);
        note_launch();
        K3_TRY(check_launch("moe a2a gather"));
        ybuf = L.recvbuf;
    } else if (O.ks > 1) {
        K3_TRY(umma_slice_sum(L.eb.contrib, O.contrib, O.ks, O.slice, (int)((size_t)R * s->hidden), st));
        ybuf = L.eb.contrib;
    }
    // results back: the region of rows received from rank r returns to rank r
    prof_begin("ep.combine");
    K3_TRY(ep_exchange(ybuf, rb.data(), ro.data(), L.back_dev, rb.data(), ro.data(), st));
    prof_end("ep.combine");
    if (shared && sst != st && cudaStreamWaitEvent(st, side_event(1), 0) != cudaSuccess)
        return fail(K3D_ECUDA, "moe a2a: join from the side stream");
    dim3 grid((s->hidden + 255) / 256, T);
    launch_pdl(k_a2a_combine, dim3(grid), dim3(256), 0, st, out, (const float *)L.back_dev, (const int *)L.pos,
               (const float *)Wt, shared ? (const float *)L.sh_out : nullptr, s->hidden, K, accumulate);
    note_launch();
    return check_launch("moe a2a combine");
}
