// k3_gemm_tc.cu -- the bf16 weight product of a batch on the fifth-generation tensor
// cores: Y[T][rows] (+)= X[T][in] . W^T for bf16 W [rows][in] (every bf16 projection of
// the model) and fp32 X, for batches of more than four tokens (decode of a batch; a
// single token or up to four stream the weights through the CUDA-core GEMV instead).
// Per token this is k3_matmul_bf16 (k3_ops.c:1108-1213), which accumulates in double; here
// the accumulation is fp32 in tensor memory.
//
// OPERANDS. A = a 128-row weight tile (M = 128), K-major, brought in by a 2-D TMA load
// (cp.async.bulk.tensor, no multicast) with the 128-byte swizzle, 64 K elements (one
// swizzle row of 128 bytes) per stage. B = the tokens: X does not fit bf16, so each token
// is written as hi = bf16(x) and lo = bf16(x - hi) (x - hi - lo is below 2^-16 |x|), and B
// holds the hi rows of the Tp tokens (T rounded up to 16, so that the epilogue's 16-column
// loads stay inside each half; padding rows zero) then their lo rows: N = 2 Tp <= 256. A
// product of bf16 values is exact in fp32; the epilogue adds the hi and lo columns of a
// token. kind::f16, bf16 x bf16, fp32 accumulators (tcgen05.mma,
// one thread issues 4 MMAs of K = 16 per stage).
//
// WORK. The units (weight tile, 64-element K chunk) of all the tiles, tile-major, are cut
// into one contiguous range per CTA (one CTA per SM at most); a CTA's range covers parts
// of one or a few tiles ("segments"), each accumulated in tensor memory and stored as a
// partial [T][128]. A second kernel sums each tile's partials in CTA order (deterministic)
// and writes Y (plain, accumulating, or silu(gate) * up for a gate/up pair).
//
// ROLES (192 threads): warp 0 lane 0 issues the copies into a ring of stages (the weight
// tiles of the first stages before waiting for the previous kernel: weights never depend
// on it); warp 1 allocates tensor memory and lane 0 issues the MMAs; warps 2-5 drain the
// accumulators (two buffers, so one segment's epilogue overlaps the next one's MMAs).
// Every wait is bounded (k3_bulk.cuh): on time-out the kernel records K3D_ETIMEOUT, all
// roles leave, in-flight tensor-core work is drained and tensor memory freed.
#include <cuda.h>

#include <mutex>
#include <unordered_map>

#include "k3_bulk.cuh"
#include "k3_ops.cuh"

namespace k3 {
namespace gtc {

using namespace bulk;

constexpr int kKC = 64;                   // K elements per stage
constexpr int kTileA = 128 * 128;         // 16 KB: 128 rows x 128 bytes
constexpr int kMaxTok = 128;              // tokens per pass (N = 2 x 128 = 256)
constexpr int kMaxMats = 8;
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kHeader = 1024;
constexpr int kSmemBudget = 226 * 1024;

struct __align__(64) Args {
    CUtensorMap tm[kMaxMats];             // weights of each matrix: bf16 [rows][in]
    int tile0[kMaxMats + 1];              // first global tile of each matrix
    int nmat;
    const uint8_t *bq;                    // B operand [nch][N rows x 128 B], swizzled
    float *part;                          // partials [grid][smax][T][128]
    int nch, N, T, Tp, U, smax, stages, stage_bytes, tmem_cols;
};

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major SWIZZLE_128B: 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t a)
{
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: fp32 D, bf16 A and B, both K-major, M = 128, N.
__device__ __forceinline__ uint32_t idesc_bf16(int N)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum) : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar) : "memory");
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float v[16])
{
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// 2-D TMA load of one weight tile: x = K element (a multiple of 64), y = first row.
__device__ __forceinline__ void tma_tile(uint32_t dst, const CUtensorMap *tm, int x, int y, uint32_t bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
                 "[%0], [%1, {%2, %3}], [%4];"
                 :: "r"(dst), "l"(tm), "r"(x), "r"(y), "r"(bar) : "memory");
}

__device__ __forceinline__ int unit_begin(int c, int grid, int U)
{
    return (int)((long long)c * U / grid);
}

// Which matrix a global tile belongs to.
__device__ __forceinline__ int mat_of(const Args &a, int tile)
{
    int j = 0;
    while (j + 1 < a.nmat && tile >= a.tile0[j + 1]) j++;
    return j;
}

__global__ void __launch_bounds__(kThreads, 1) k_gemm_tc(const __grid_constant__ Args a)
{
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = saddr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char *gbase = smem_raw + (base - raw);
    const uint32_t b_full = base;                          // [kMaxStages]
    const uint32_t b_empty = base + 8 * kMaxStages;        // [kMaxStages]
    const uint32_t b_accf = base + 16 * kMaxStages;        // [2]
    const uint32_t b_acce = b_accf + 16;                   // [2]
    const uint32_t b_drain = b_acce + 16;
    volatile int *abort = reinterpret_cast<volatile int *>(gbase + 512);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + 520);
    const uint32_t stage0 = base + kHeader;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) { mbar_init(b_full + 8 * s, 1); mbar_init(b_empty + 8 * s, 1); }
        for (int i = 0; i < 2; i++) { mbar_init(b_accf + 8 * i, 1); mbar_init(b_acce + 8 * i, 4); }
        mbar_init(b_drain, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(saddr(tmem_slot)), "r"(a.tmem_cols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int u0 = unit_begin(blockIdx.x, gridDim.x, a.U), u1 = unit_begin(blockIdx.x + 1, gridDim.x, a.U);
    const int first_tile = u0 / a.nch;
    const uint32_t btile = (uint32_t)a.N * 128u;
    const uint32_t tx = (uint32_t)kTileA + btile;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            // the first stages' weight tiles before waiting for the kernel that writes B
            const int pre = min(S, u1 - u0);
            for (int h = 0; h < pre; h++) {
                const int u = u0 + h, tile = u / a.nch, j = mat_of(a, tile);
                const uint32_t sb = stage0 + (uint32_t)h * a.stage_bytes, fb = b_full + 8 * h;
                mbar_expect_tx(fb, tx);
                tma_tile(sb, &a.tm[j], (u % a.nch) * kKC, (tile - a.tile0[j]) * 128, fb);
            }
            pdl_wait();
            for (int h = 0; h < pre; h++) {
                const int u = u0 + h;
                const uint32_t sb = stage0 + (uint32_t)h * a.stage_bytes, fb = b_full + 8 * h;
                g2s(sb + kTileA, a.bq + (size_t)(u % a.nch) * btile, btile, fb);
            }
            for (int u = u0 + pre, g = pre; u < u1; u++, g++) {
                const int st = g % S;
                if (!mbar_wait(b_empty + 8 * st, ((g / S) - 1) & 1, abort, K3_SITE_GEMV, 20, g)) break;
                const int tile = u / a.nch, j = mat_of(a, tile);
                const uint32_t sb = stage0 + (uint32_t)st * a.stage_bytes, fb = b_full + 8 * st;
                mbar_expect_tx(fb, tx);
                tma_tile(sb, &a.tm[j], (u % a.nch) * kKC, (tile - a.tile0[j]) * 128, fb);
                g2s(sb + kTileA, a.bq + (size_t)(u % a.nch) * btile, btile, fb);
            }
        }
    } else {
        pdl_wait();
        pdl_trigger();
        if (warp == 1) {
            // ----------------------------------------------------------- MMA issuer
            if (lane == 0) {
                const uint32_t id = idesc_bf16(a.N);
                int g = 0, nseg = 0;
                bool stop = false;
                for (int u = u0; u < u1 && !stop; nseg++) {
                    const int seg_end = min(u1, (u / a.nch + 1) * a.nch);
                    const int buf = nseg & 1;
                    if (nseg >= 2 && !mbar_wait(b_acce + 8 * buf, ((nseg >> 1) - 1) & 1, abort, K3_SITE_GEMV, 21, nseg)) break;
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)(buf * a.N);
                    const int seg_start = u;
                    for (; u < seg_end; u++, g++) {
                        const int st = g % S;
                        if (!mbar_wait(b_full + 8 * st, (g / S) & 1, abort, K3_SITE_GEMV, 22, g)) { stop = true; break; }
                        tc_fence_after();
                        const uint32_t sa = stage0 + (uint32_t)st * a.stage_bytes, sb = sa + kTileA;
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            tc_mma(d, desc_sw128(sa + 32u * k), desc_sw128(sb + 32u * k), id,
                                   (u != seg_start || k > 0) ? 1u : 0u);
                        tc_commit(b_empty + 8 * st);
                    }
                    if (!stop) tc_commit(b_accf + 8 * buf);
                }
            }
            __syncwarp();
        } else {
            // ------------------------------------------------------------- epilogue
            const int q = warp & 3;                // tensor-memory lane quadrant
            const int row = q * 32 + lane;         // row of the tile
            int nseg = 0;
            for (int u = u0; u < u1; nseg++) {
                const int tile = u / a.nch;
                const int seg_end = min(u1, (tile + 1) * a.nch);
                const int buf = nseg & 1;
                if (!mbar_wait(b_accf + 8 * buf, (nseg >> 1) & 1, abort, K3_SITE_GEMV, 23, nseg)) break;
                tc_fence_after();
                float *dst = a.part + ((size_t)(blockIdx.x * a.smax + (tile - first_tile)) * a.T) * 128 + row;
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * a.N);
                for (int t0 = 0; t0 < a.T; t0 += 16) {
                    float hi[16], lo[16];
                    tc_ld16(tbase + (uint32_t)t0, hi);
                    tc_ld16(tbase + (uint32_t)(a.Tp + t0), lo);
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        if (t0 + i < a.T) dst[(size_t)(t0 + i) * 128] = hi[i] + lo[i];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(b_acce + 8 * buf);
                u = seg_end;
            }
        }
    }
    __syncthreads();
    if (warp == 1 && lane == 0) {
        // every MMA issued above has completed once this barrier flips
        tc_commit(b_drain);
        const long long t0 = clock64();
        while (!mbar_try(b_drain, 0)) {
            if (clock64() - t0 > kSpinLimit) { k3_raise_at(K3D_ETIMEOUT, K3_SITE_GEMV, 24, 0, (int)blockIdx.x); break; }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem), "r"(a.tmem_cols) : "memory");
    }
}

// B operand of the tokens: for chunk c (64 K elements), N rows of 128 bytes in the
// SWIZZLE_128B layout: row r < Tp the bf16 of token r, row Tp + r its remainder (x - hi
// rounded to bf16); rows of tokens >= T are zero. One thread per 16-byte unit.
__global__ void k_split_hilo(uint8_t *bq, const float *x, int in, int T, int Tp, int nch)
{
    pdl_wait();
    pdl_trigger();
    const int N = 2 * Tp;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)nch * N * 8) return;
    const int j = (int)(i & 7), r = (int)((i >> 3) % N), c = (int)(i / (8LL * N));
    const int t = r < Tp ? r : r - Tp;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (t < T) {
        const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * in + c * kKC + j * 8);
        const float4 p = src[0], q = src[1];
        const float v[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
        uint16_t h[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const uint16_t hb = f32_to_bf16_bits(v[e]);
            h[e] = r < Tp ? hb : f32_to_bf16_bits(v[e] - bf16_to_f32(hb));
        }
#pragma unroll
        for (int e = 0; e < 4; e++) w[e] = (uint32_t)h[2 * e] | ((uint32_t)h[2 * e + 1] << 16);
    }
    *reinterpret_cast<uint4 *>(bq + (size_t)c * N * 128 + (size_t)r * 128 + (((j ^ (r & 7)) & 7) << 4)) =
        make_uint4(w[0], w[1], w[2], w[3]);
}

struct RedArgs {
    float *y[kMaxMats];
    int rows[kMaxMats];
    int tile0[kMaxMats + 1];
    int nmat, swiglu, accumulate;
    const float *part;
    int T, nch, U, grid, smax;
};

// Sum over the CTAs covering tile m (units [m nch, (m+1) nch)) of their partials, in CTA
// order; tr = this thread's row of the tile.
__device__ __forceinline__ float tile_sum(const RedArgs &r, int m, int t, int tr)
{
    const long long lo = (long long)m * r.nch, hi = lo + r.nch;
    int c = (int)(lo * r.grid / r.U);
    while (c > 0 && (long long)c * r.U / r.grid > lo) c--;
    while (c + 1 < r.grid && (long long)(c + 1) * r.U / r.grid <= lo) c++;
    float s = 0.0f;
    for (; c < r.grid; c++) {
        const long long cb = (long long)c * r.U / r.grid;
        if (cb >= hi) break;
        const int seg = m - (int)(cb / r.nch);
        s += __ldcg(r.part + ((size_t)(c * r.smax + seg) * r.T + t) * 128 + tr);
    }
    return s;
}

// grid (output tiles, ceil(T / 8)), 128 threads: one row of a tile, eight tokens.
__global__ void k_gemm_reduce(RedArgs r)
{
    pdl_wait();
    pdl_trigger();
    const int m = blockIdx.x, tr = threadIdx.x;
    int j = 0;
    while (j + 1 < r.nmat && m >= r.tile0[j + 1]) j++;
    const int row = (m - r.tile0[j]) * 128 + tr;
    if (row >= r.rows[j]) return;
    const int t1 = min(r.T, (int)(blockIdx.y + 1) * 8);
    for (int t = blockIdx.y * 8; t < t1; t++) {
        float v = tile_sum(r, m, t, tr);
        if (r.swiglu) {
            // gate tiles are matrix 0, the same rows of up are matrix 1
            const float u = tile_sum(r, r.tile0[1] + (m - r.tile0[0]), t, tr);
            v = silu_f(v) * u;
        }
        float *o = r.y[j] + (size_t)t * r.rows[j] + row;
        *o = r.accumulate ? *o + v : v;
    }
}

// --------------------------------------------------------------------------- host ----
typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encoder()
{
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiled)p;
        else
            cudaGetLastError();
    });
    return fn;
}

// The tensor map of a weight matrix (box 64 K x 128 rows, 128-byte swizzle; rows past the
// end read as zero), encoded once per (pointer, shape).
static bool weight_map(CUtensorMap *m, const uint16_t *W, int in, int rows)
{
    struct Key {
        const void *p; int in, rows;
        bool operator==(const Key &o) const { return p == o.p && in == o.in && rows == o.rows; }
    };
    struct Hash {
        size_t operator()(const Key &k) const { return std::hash<const void *>()(k.p) ^ ((size_t)k.in << 20) ^ k.rows; }
    };
    static std::mutex mu;
    static std::unordered_map<Key, CUtensorMap, Hash> cache;
    std::lock_guard<std::mutex> lk(mu);
    const Key key{W, in, rows};
    auto it = cache.find(key);
    if (it != cache.end()) { *m = it->second; return true; }
    EncodeTiled enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)in, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)in * 2};
    const cuuint32_t box[2] = {kKC, 128};
    const cuuint32_t es[2] = {1, 1};
    CUtensorMap t;
    if (enc(&t, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void *)W, dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    cache.emplace(key, t);
    *m = t;
    return true;
}

// One pass over at most kMaxTok tokens.
static int gemm_pass(int nmat, const uint16_t *const *W, float *const *Y, const int *rows, const float *x,
                     int in, int T, int accumulate, int swiglu, cudaStream_t st)
{
    Args a;
    RedArgs r;
    const int Tp = (T + 15) & ~15, N = 2 * Tp, nch = in / kKC;
    a.nmat = r.nmat = nmat;
    int tiles = 0;
    for (int j = 0; j < nmat; j++) {
        if (!weight_map(&a.tm[j], W[j], in, rows[j]))
            return fail(K3D_ECUDA, "gemm: tensor map of a %d x %d bf16 matrix", rows[j], in);
        a.tile0[j] = r.tile0[j] = tiles;
        tiles += (rows[j] + 127) / 128;
        r.y[j] = Y[j];
        r.rows[j] = rows[j];
    }
    a.tile0[nmat] = r.tile0[nmat] = tiles;
    const int U = tiles * nch;
    const int grid = U < sm_count() ? U : sm_count();
    const int per = (U + grid - 1) / grid;
    const int smax = per / nch + 2;
    const int stage_bytes = kTileA + N * 128;
    int stages = (kSmemBudget - kHeader - 1024) / stage_bytes;
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < 2) return fail(K3D_EINVAL, "gemm: N=%d leaves fewer than two stages", N);
    int tcols = 32;
    while (tcols < 2 * N) tcols <<= 1;
    // scratch slot by stream: the library stream and the side stream may both run one
    const int slot = st == stream() ? 1 : 4;
    const size_t bq_bytes = (size_t)nch * N * 128;
    const size_t part_bytes = (size_t)grid * smax * T * 128 * sizeof(float);
    uint8_t *ws = (uint8_t *)scratch(bq_bytes + part_bytes + 256, slot);
    if (!ws) return k3d_status();
    a.bq = ws;
    a.part = (float *)(ws + ((bq_bytes + 255) & ~(size_t)255));
    a.nch = r.nch = nch;
    a.N = N;
    a.T = r.T = T;
    a.Tp = Tp;
    a.U = r.U = U;
    a.smax = r.smax = smax;
    a.stages = stages;
    a.stage_bytes = stage_bytes;
    a.tmem_cols = tcols;
    r.grid = grid;
    r.part = a.part;
    r.swiglu = swiglu;
    r.accumulate = accumulate;
    const size_t smem = 1024 + kHeader + (size_t)stages * stage_bytes;
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) {
        if (cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget) != cudaSuccess)
            return fail(K3D_ECUDA, "gemm smem attribute");
        init |= dev_bit();
    }
    const long long units = (long long)nch * N * 8;
    launch_pdl(k_split_hilo, dim3((unsigned)((units + 255) / 256)), dim3(256), 0, st, ws, x, in, T, Tp, nch);
    launch_pdl(k_gemm_tc, dim3(grid), dim3(kThreads), smem, st, a);
    const int out_tiles = swiglu ? a.tile0[1] : tiles;
    launch_pdl(k_gemm_reduce, dim3(out_tiles, (T + 7) / 8), dim3(128), 0, st, r);
    note_launch(3);
    return check_launch("gemm tc");
}

}  // namespace gtc

// Batched bf16 product on the tensor cores (see the file comment). swiglu: two matrices
// (gate, up) of the same rows; Y[0] receives silu(gate) * up. Requirements: in a multiple
// of 64, W 16-byte aligned, x 16-byte aligned.
int gemm_bf16_tc(int nmat, const uint16_t *const *W, float *const *Y, const int *rows, const float *x,
                 int in, int T, int accumulate, int swiglu, cudaStream_t st)
{
    using namespace gtc;
    if (nmat < 1 || nmat > kMaxMats || T < 1 || in % kKC || (swiglu && (nmat != 2 || rows[0] != rows[1])))
        return fail(K3D_EINVAL, "gemm: %d matrices, T=%d, in=%d", nmat, T, in);
    if ((uintptr_t)x & 15u) return fail(K3D_EINVAL, "gemm: unaligned x");
    for (int j = 0; j < nmat; j++)
        if (((uintptr_t)W[j] & 15u) || rows[j] < 1) return fail(K3D_EINVAL, "gemm: matrix %d", j);
    for (int t0 = 0; t0 < T; t0 += kMaxTok) {
        const int Tc = T - t0 < kMaxTok ? T - t0 : kMaxTok;
        float *Yc[kMaxMats];
        for (int j = 0; j < nmat; j++) Yc[j] = Y[j] + (size_t)t0 * rows[j];
        if (swiglu) Yc[1] = Yc[0];
        K3_TRY(gemm_pass(nmat, W, Yc, rows, x + (size_t)t0 * in, in, Tc, accumulate, swiglu, st));
    }
    return K3D_OK;
}

}  // namespace k3
