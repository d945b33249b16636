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

__device__ __forceinline__ bool bad_align(const void *a, const void *b)
{
    return (((uintptr_t)a | (uintptr_t)b) & 15u) != 0;
}

}  // namespace k3
