// k3_ep.cu -- expert parallelism plumbing over NCCL: one process per GPU, experts
// [n*E/G, (n+1)*E/G) on rank n. The combine of a replicated-activation decode step is an
// in-place sum of the per-rank partial MoE outputs (ncclAllReduce on the library stream,
// so it orders after the expert kernels and can be captured into a CUDA graph).
// Mode A (all-to-all dispatch and combine of data-parallel tokens) exchanges rows with
// grouped send/recv (ep_exchange). The CPU engine is single-process and has no counterpart.
#include <nccl.h>

#include <cstdint>
#include <cstring>
#include <vector>

#include "k3_common.cuh"

namespace k3 {
namespace {
ncclComm_t g_comm = nullptr;
int g_rank = 0, g_size = 1;

// ------------------------------------------------------ NVLink push combine (Mode R)
// Every rank owns one receive buffer, exported with CUDA IPC and mapped by every other rank
// (k3d_ep_peer_init). Layout: flags [kEpMaxRanks sources][kEpSlices] as one 128-byte line
// each, then data [2 parities][kEpMaxRanks sources][max_n] fp32.
constexpr int kEpSlices = 32;             // CTAs of one combine; slice i of the vector each
constexpr int kEpMaxRanks = 8;
constexpr size_t kEpFlagBytes = (size_t)kEpMaxRanks * kEpSlices * 128;
struct PeerBufs {
    char *local = nullptr;                // this rank's buffer
    char *peer[kEpMaxRanks] = {};         // every rank's buffer as mapped here (peer[me] = local)
    unsigned *epoch = nullptr;            // [kEpSlices]: combines completed, per slice (device)
    size_t max_n = 0;                     // floats per slot
};
PeerBufs g_pb;
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

struct EpPeers {
    float *data[kEpMaxRanks];             // rank r's data region
    unsigned *flags[kEpMaxRanks];         // rank r's flag lines
};

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// h[j] (+)= sum over ranks r = 0..nr-1 of part_r[j], the same on every rank. CTA i owns
// slice i of the vector: it stores its slice of this rank's partial into slot (parity, me)
// of every rank's buffer (plain stores through NVLink), publishes it with one release flag
// per destination, waits for the flags of slice i from every rank (bounded), and sums the
// nr slots in rank order. The parity alternates with the call count: a rank can be at most
// one call ahead of another (it cannot finish a call without the other's contribution), so
// two generations of slots never collide. Per-slice call counters (epoch) live on each
// device and advance identically on every rank.
__global__ void __launch_bounds__(256) k_ep_push_sum(float *h, const float *part, int n, const __grid_constant__ EpPeers P, int me,
                                                     int nr, unsigned *epoch, size_t max_n, int accumulate)
{
    __shared__ unsigned s_e;
    __shared__ int s_ok;
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x;
    const int per = ((n + (int)gridDim.x - 1) / (int)gridDim.x + 3) & ~3;
    const int s0 = min(n, i * per), s1 = min(n, s0 + per);
    if (threadIdx.x == 0) { s_e = epoch[i] + 1u; s_ok = 1; }
    __syncthreads();
    const unsigned e = s_e;
    const size_t par = e & 1u;
    for (int r = 0; r < nr; r++) {
        float *dst = P.data[r] + (par * kEpMaxRanks + (size_t)me) * max_n;
        for (int j = s0 + 4 * (int)threadIdx.x; j < s1; j += 4 * blockDim.x) {
            if (j + 3 < s1) {
                *reinterpret_cast<float4 *>(dst + j) = *reinterpret_cast<const float4 *>(part + j);
            } else {
                for (int t = j; t < s1; t++) dst[t] = part[t];
            }
        }
    }
    __threadfence_system();
    __syncthreads();
    if ((int)threadIdx.x < nr)
        st_release_sys(P.flags[threadIdx.x] + ((size_t)me * kEpSlices + i) * 32, e);
    if ((int)threadIdx.x < nr) {
        const unsigned *f = P.flags[me] + ((size_t)threadIdx.x * kEpSlices + i) * 32;
        const long long t0 = clock64(), lim = k3_wait_cycles;
        while ((int)(ld_acquire_sys(f) - e) < 0) {
            if (clock64() - t0 > lim) {
                k3_raise_at(K3D_ETIMEOUT, K3_SITE_EP, (int)threadIdx.x, i, (int)e);
                s_ok = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (!s_ok) return;                    // a rank did not arrive; the status says which
    const float *src = P.data[me] + par * kEpMaxRanks * max_n;
    for (int j = s0 + (int)threadIdx.x; j < s1; j += blockDim.x) {
        float v = __ldcg(src + j);
        for (int r = 1; r < nr; r++) v += __ldcg(src + (size_t)r * max_n + j);
        h[j] = accumulate ? h[j] + v : v;
    }
    if (threadIdx.x == 0) epoch[i] = e;
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

// The same sum in one pass per element (the default): every element travels as one 8-byte
// word, its float bits in the low half and the slice's call count in the high half, stored
// to slot (parity, me) of every rank with one single-copy-atomic store; the receiver polls
// each source's word until its tag shows this call, so a word carries its own arrival flag
// and there is no fence, no separate flag store and no barrier. Same sum order (rank 0
// first) and the same per-slice counts as k_ep_push_sum, hence the same bits.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long *p, unsigned long long v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(256) k_ep_push_sum_ll(float *h, const float *part, int n, const __grid_constant__ EpPeers P,
                                                        int me, int nr, unsigned *epoch, size_t max_n, int accumulate)
{
    __shared__ unsigned s_e;
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x;
    const int per = ((n + (int)gridDim.x - 1) / (int)gridDim.x + 3) & ~3;
    const int s0 = min(n, i * per), s1 = min(n, s0 + per);
    if (threadIdx.x == 0) s_e = epoch[i] + 1u;
    __syncthreads();
    const unsigned e = s_e;
    const size_t par = e & 1u;
    for (int j = s0 + (int)threadIdx.x; j < s1; j += blockDim.x) {
        const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(part[j]);
        for (int r = 0; r < nr; r++) {
            unsigned long long *dst = reinterpret_cast<unsigned long long *>(P.data[r]) + (par * kEpMaxRanks + (size_t)me) * max_n;
            st_relaxed_sys_u64(dst + j, w);
        }
    }
    const unsigned long long *src = reinterpret_cast<const unsigned long long *>(P.data[me]) + par * kEpMaxRanks * max_n;
    const long long lim = k3_wait_cycles;
    bool timed_out = false;
    for (int j = s0 + (int)threadIdx.x; j < s1; j += blockDim.x) {
        float v = 0.0f;
        for (int r = 0; r < nr; r++) {
            const unsigned long long *q = src + (size_t)r * max_n + j;
            unsigned long long w = ld_relaxed_sys_u64(q);
            if ((unsigned)(w >> 32) != e && !timed_out) {
                const long long t0 = clock64();
                do {
                    __nanosleep(32);
                    w = ld_relaxed_sys_u64(q);
                    if (clock64() - t0 > lim) {
                        k3_raise_at(K3D_ETIMEOUT, K3_SITE_EP, r, i, (int)e);
                        timed_out = true;
                        break;
                    }
                } while ((unsigned)(w >> 32) != e);
            }
            const float x = __uint_as_float((unsigned)w);
            v = r == 0 ? x : v + x;
        }
        h[j] = accumulate ? h[j] + v : v;
    }
    __syncthreads();
    if (threadIdx.x == 0) epoch[i] = e;
}

// which combine kernel k3d_ep_combine_add launches: 0 one tagged word per element, 1 data
// then a release flag per slice
static int g_ep_combine_kind = 0;

int k3d_ep_peer_init(size_t max_floats)
{
    K3_TRY(ensure_ctx());
    if (g_size == 1) return K3D_OK;
    if (!g_comm) return fail(K3D_ENCCL, "k3d_ep_peer_init before k3d_ep_init");
    if (g_size > kEpMaxRanks) return fail(K3D_EINVAL, "k3d_ep_peer_init: %d ranks (at most %d)", g_size, kEpMaxRanks);
    if (g_pb.local && g_pb.max_n >= max_floats) return K3D_OK;
    if (g_pb.local) return fail(K3D_EINVAL, "k3d_ep_peer_init: already set up for %zu floats", g_pb.max_n);
    const size_t max_n = (max_floats + 63) & ~(size_t)63;
    // data: [2 parities][kEpMaxRanks sources][max_n] 8-byte words (the flag protocol uses the
    // first half of the region as floats with the same indexing)
    const size_t bytes = kEpFlagBytes + 2 * (size_t)kEpMaxRanks * max_n * sizeof(unsigned long long);
    cudaStream_t st = stream();
    if (cudaMalloc(&g_pb.local, bytes) != cudaSuccess || cudaMalloc(&g_pb.epoch, kEpSlices * sizeof(unsigned)) != cudaSuccess) {
        cudaGetLastError();
        return fail(K3D_ENOMEM, "k3d_ep_peer_init: %zu bytes", bytes);
    }
    if (cudaMemsetAsync(g_pb.local, 0, bytes, st) != cudaSuccess ||
        cudaMemsetAsync(g_pb.epoch, 0, kEpSlices * sizeof(unsigned), st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(K3D_ECUDA, "k3d_ep_peer_init: clearing the buffer");
    // every rank's IPC handle to every rank (an all-gather over the NCCL communicator)
    cudaIpcMemHandle_t mine;
    if (cudaIpcGetMemHandle(&mine, g_pb.local) != cudaSuccess) return fail(K3D_ECUDA, "cudaIpcGetMemHandle");
    char *dh = nullptr;
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    if (cudaMalloc(&dh, hb * (g_size + 1)) != cudaSuccess) return fail(K3D_ENOMEM, "ipc handle staging");
    std::vector<cudaIpcMemHandle_t> all(g_size);
    bool ok = cudaMemcpyAsync(dh, &mine, hb, cudaMemcpyHostToDevice, st) == cudaSuccess &&
              ncclAllGather(dh, dh + hb, hb, ncclInt8, g_comm, st) == ncclSuccess &&
              cudaMemcpyAsync(all.data(), dh + hb, hb * g_size, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
              cudaStreamSynchronize(st) == cudaSuccess;
    cudaFree(dh);
    if (!ok) return fail(K3D_ENCCL, "k3d_ep_peer_init: handle exchange");
    for (int r = 0; r < g_size; r++) {
        if (r == g_rank) { g_pb.peer[r] = g_pb.local; continue; }
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
            return fail(K3D_ECUDA, "cudaIpcOpenMemHandle (rank %d)", r);
        g_pb.peer[r] = (char *)p;
    }
    g_pb.max_n = max_n;
    // no rank pushes before every rank has mapped every buffer
    float *one = nullptr;
    if (cudaMalloc(&one, sizeof(float)) != cudaSuccess) return fail(K3D_ENOMEM, "ep barrier");
    ok = ncclAllReduce(one, one, 1, ncclFloat32, ncclSum, g_comm, st) == ncclSuccess &&
         cudaStreamSynchronize(st) == cudaSuccess;
    cudaFree(one);
    return ok ? K3D_OK : fail(K3D_ENCCL, "k3d_ep_peer_init: barrier");
}

int k3d_ep_combine_add(float *h, const float *partial, size_t n, int accumulate)
{
    K3_TRY(ensure_ctx());
    cudaStream_t st = stream();
    if (g_size == 1) {
        if (accumulate) return k3d_add_f32(h, partial, n);
        return h == partial ? K3D_OK : k3d_copy(h, partial, n * sizeof(float));
    }
    if (!g_pb.local || n > g_pb.max_n || (((uintptr_t)h | (uintptr_t)partial) & 15u)) {
        // the NCCL form: an in-place sum of the partials, then the residual add
        if (!g_comm) return fail(K3D_ENCCL, "k3d_ep_combine_add before k3d_ep_init");
        prof_begin("ep.combine");
        ncclResult_t r = ncclAllReduce(partial, (void *)partial, n, ncclFloat32, ncclSum, g_comm, st);
        prof_end("ep.combine");
        if (r != ncclSuccess) return fail(K3D_ENCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
        if (accumulate) return k3d_add_f32(h, partial, n);
        return h == partial ? K3D_OK : k3d_copy(h, partial, n * sizeof(float));
    }
    if (n > (size_t)INT32_MAX) return fail(K3D_EINVAL, "k3d_ep_combine_add: n=%zu", n);
    EpPeers P;
    for (int r = 0; r < kEpMaxRanks; r++) {
        P.data[r] = r < g_size ? (float *)(g_pb.peer[r] + kEpFlagBytes) : nullptr;
        P.flags[r] = r < g_size ? (unsigned *)g_pb.peer[r] : nullptr;
    }
    prof_begin("ep.combine");
    if (g_ep_combine_kind == 0)
        launch_pdl(k_ep_push_sum_ll, dim3(kEpSlices), dim3(256), 0, st, h, partial, (int)n, P, g_rank, g_size,
                   g_pb.epoch, g_pb.max_n, accumulate);
    else
        launch_pdl(k_ep_push_sum, dim3(kEpSlices), dim3(256), 0, st, h, partial, (int)n, P, g_rank, g_size,
                   g_pb.epoch, g_pb.max_n, accumulate);
    note_launch();
    prof_end("ep.combine");
    return check_launch("ep push combine");
}

int k3d_ep_finalize(void)
{
    if (!g_comm) return K3D_OK;
    cudaStreamSynchronize(stream());
    for (int r = 0; r < kEpMaxRanks; r++) {
        if (g_pb.peer[r] && r != g_rank) cudaIpcCloseMemHandle(g_pb.peer[r]);
        g_pb.peer[r] = nullptr;
    }
    if (g_pb.local) cudaFree(g_pb.local);
    if (g_pb.epoch) cudaFree(g_pb.epoch);
    g_pb = PeerBufs{};
    ncclCommDestroy(g_comm);
    g_comm = nullptr;
    g_rank = 0;
    g_size = 1;
    return K3D_OK;
}

int k3d_set_ep_combine(int kind)
{
    if (kind < 0 || kind > 1) return fail(K3D_EINVAL, "k3d_set_ep_combine(%d): 0 or 1", kind);
    g_ep_combine_kind = kind;
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
