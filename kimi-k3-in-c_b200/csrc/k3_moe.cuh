// k3_moe.cuh -- the expert work list shared by the MoE kernels (k3_moe.cu) and the
// tensor-core MXFP4 expert kernels (k3_mxfp4_mma.cu).
#pragma once
#include "k3_common.cuh"

namespace k3 {

struct MoeWork {
    const K3ExpertQ *table;     // device table, indexed by expert id (MoE mode)
    K3ExpertQ single;           // the one expert (single mode)
    const int *n_active;        // device: number of active (local, selected) experts
    const int *act_expert;      // device [n_active]
    const int *act_off;         // device [n_active + 1] into assign
    const int *assign;          // device: assignment ids a = t*K + j, grouped by expert
    int single_mode;
    int ntok_single;            // single mode: assignments a = 0..ntok-1, token t = a
    int K;                      // top-k (token t = a / K)
    int n_experts;              // MoE mode: size of the expert table
};

__device__ __forceinline__ void work_item(const MoeWork &w, int u, K3ExpertQ &q, int &beg,
                                          int &end, bool &ok)
{
    if (w.single_mode) {
        q = w.single; beg = 0; end = w.ntok_single; ok = (u == 0);
        return;
    }
    const int na = __ldg(w.n_active);
    ok = u < na;
    if (!ok) return;
    const int e = __ldg(w.act_expert + u);
    q = w.table[e];
    beg = __ldg(w.act_off + u);
    end = __ldg(w.act_off + u + 1);
}

__device__ __forceinline__ int work_assign(const MoeWork &w, int p)
{
    return w.single_mode ? p : __ldg(w.assign + p);
}

// Groups the T*K routed assignments by expert (k3_ops.c:717-825, "fetch each unique
// expert once"): n_active[0] = active experts in [lo, hi), n_active[1] = their
// assignments; act_expert[u] in increasing id order with act_off[u] into assign, which
// lists the assignment ids a = t*K + j of each expert. Any block size >= 32; `sm` holds
// 2 * n_experts ints. idx is read through L2 (it may have been written by other CTAs of
// the same grid).
// zero/nzero: a region zeroed on the way (the fused expert pass's counters).
// idx_local: idx is this CTA's shared-memory copy (read with plain loads), not global
__device__ __forceinline__ void group_assignments(const int *idx, int TK, int n_experts, int lo,
                                                  int hi, int *n_active, int *act_expert,
                                                  int *act_off, int *assign, int *sm,
                                                  int *zero = nullptr, int nzero = 0,
                                                  bool idx_local = false)
{
    for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
    int *cnt = sm;                 // [n_experts]
    int *cur = sm + n_experts;     // [n_experts]
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int a = threadIdx.x; a < TK; a += blockDim.x) {
        const int e = idx_local ? idx[a] : __ldcg(idx + a);
        if (e >= lo && e < hi && e < n_experts && e >= 0) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const int per = (n_experts + 31) / 32;
        const int e0 = min(n_experts, lane * per), e1 = min(n_experts, e0 + per);
        int sc = 0, sf = 0;
        for (int e = e0; e < e1; e++) { sc += cnt[e]; sf += cnt[e] > 0; }
        int ic = sc, iff = sf;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int vc = __shfl_up_sync(0xffffffffu, ic, o);
            const int vf = __shfl_up_sync(0xffffffffu, iff, o);
            if (lane >= o) { ic += vc; iff += vf; }
        }
        int off = ic - sc, u = iff - sf;
        for (int e = e0; e < e1; e++) {
            cur[e] = off;
            if (cnt[e] > 0) { act_expert[u] = e; act_off[u] = off; u++; }
            off += cnt[e];
        }
        if (lane == 31) { n_active[0] = iff; n_active[1] = ic; act_off[iff] = ic; }
    }
    __syncthreads();
    for (int a = threadIdx.x; a < TK; a += blockDim.x) {
        const int e = idx_local ? idx[a] : __ldcg(idx + a);
        if (e >= lo && e < hi && e < n_experts && e >= 0) {
            const int p = atomicAdd(&cur[e], 1);
            assign[p] = a;
        }
    }
}

__device__ __forceinline__ bool bad_align(const void *a, const void *b)
{
    return (((uintptr_t)a | (uintptr_t)b) & 15u) != 0;
}

}  // namespace k3
