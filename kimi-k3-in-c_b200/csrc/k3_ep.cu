// k3_ep.cu -- expert parallelism plumbing over NCCL: one process per GPU, experts
// [n*E/G, (n+1)*E/G) on rank n. The combine of a replicated-activation decode step is an
// in-place sum of the per-rank partial MoE outputs (ncclAllReduce on the library stream,
// so it orders after the expert kernels and can be captured into a CUDA graph).
// Mode A (all-to-all dispatch and combine of data-parallel tokens) exchanges rows with
// grouped send/recv (ep_exchange). The CPU engine is single-process and has no counterpart.
#include <nccl.h>

#include "k3_common.cuh"

namespace k3 {
namespace {
ncclComm_t g_comm = nullptr;
int g_rank = 0, g_size = 1;
}  // namespace
}  // namespace k3

namespace k3 {

// Grouped point-to-point exchange on the library stream: to each rank r, scnt[r] bytes of
// `send` from byte soff[r]; from it, rcnt[r] bytes into `recv` at byte roff[r]. Both sides
// of a pair agree on the size (the receive counts come from an earlier exchange of the
// send counts), so zero-byte pairs are skipped on both. One rank: a device copy.
int ep_exchange(const void *send, const size_t *scnt, const size_t *soff, void *recv,
                const size_t *rcnt, const size_t *roff, cudaStream_t st)
{
    if (g_size == 1) {
        if (scnt[0] != rcnt[0]) return fail(K3D_EINVAL, "ep exchange: %zu bytes sent, %zu expected", scnt[0], rcnt[0]);
        if (scnt[0] && cudaMemcpyAsync((char *)recv + roff[0], (const char *)send + soff[0], scnt[0],
                                       cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return fail(K3D_ECUDA, "ep exchange copy");
        return K3D_OK;
    }
    if (!g_comm) return fail(K3D_ENCCL, "ep exchange before k3d_ep_init");
    ncclResult_t r = ncclGroupStart();
    for (int p = 0; p < g_size && r == ncclSuccess; p++) {
        if (scnt[p]) r = ncclSend((const char *)send + soff[p], scnt[p], ncclInt8, p, g_comm, st);
        if (r == ncclSuccess && rcnt[p]) r = ncclRecv((char *)recv + roff[p], rcnt[p], ncclInt8, p, g_comm, st);
    }
    const ncclResult_t e = ncclGroupEnd();
    if (r == ncclSuccess) r = e;
    if (r != ncclSuccess) return fail(K3D_ENCCL, "ep exchange: %s", ncclGetErrorString(r));
    return K3D_OK;
}

int ep_allreduce_max_u64(unsigned long long *buf, size_t n, cudaStream_t st)
{
    if (g_size == 1) return K3D_OK;
    if (!g_comm) return fail(K3D_ENCCL, "ep max before k3d_ep_init");
    ncclResult_t r = ncclAllReduce(buf, buf, n, ncclUint64, ncclMax, g_comm, st);
    if (r != ncclSuccess) return fail(K3D_ENCCL, "ncclAllReduce max: %s", ncclGetErrorString(r));
    return K3D_OK;
}

}  // namespace k3

using namespace k3;

extern "C" {

int k3d_ep_unique_id(unsigned char id[128])
{
    if (!id) return fail(K3D_EINVAL, "k3d_ep_unique_id null");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    ncclUniqueId u;
    ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) return fail(K3D_ENCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
    memcpy(id, &u, sizeof u);
    return K3D_OK;
}

int k3d_ep_init(int rank, int nranks, const unsigned char id[128])
{
    K3_TRY(ensure_ctx());
    if (!id || nranks < 1 || rank < 0 || rank >= nranks)
        return fail(K3D_EINVAL, "k3d_ep_init rank=%d nranks=%d", rank, nranks);
    if (g_comm) return fail(K3D_EINVAL, "k3d_ep_init called twice");
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    ncclResult_t r = ncclCommInitRank(&g_comm, nranks, u, rank);
    if (r != ncclSuccess) {
        g_comm = nullptr;
        return fail(K3D_ENCCL, "ncclCommInitRank: %s", ncclGetErrorString(r));
    }
    g_rank = rank;
    g_size = nranks;
    return K3D_OK;
}

int k3d_ep_finalize(void)
{
    if (!g_comm) return K3D_OK;
    cudaStreamSynchronize(stream());
    ncclCommDestroy(g_comm);
    g_comm = nullptr;
    g_rank = 0;
    g_size = 1;
    return K3D_OK;
}

int k3d_ep_rank(void) { return g_rank; }
int k3d_ep_size(void) { return g_size; }

int k3d_ep_allreduce_f32(float *buf, size_t n)
{
    K3_TRY(ensure_ctx());
    if (g_size == 1) return K3D_OK;
    if (!g_comm) return fail(K3D_ENCCL, "k3d_ep_allreduce_f32 before k3d_ep_init");
    prof_begin("ep.combine");
    ncclResult_t r = ncclAllReduce(buf, buf, n, ncclFloat32, ncclSum, g_comm, stream());
    prof_end("ep.combine");
    if (r != ncclSuccess) return fail(K3D_ENCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
    return K3D_OK;
}

}  // extern "C"
