// k3_mxfp4_umma.cu -- the MXFP4 expert GEMV on the fifth-generation tensor cores:
// tcgen05.mma.kind::mxf4.block_scale.block32 (E2M1 x E2M1 with one UE8M0 scale per 32
// elements on each operand, fp32 accumulation in tensor memory).
//
// WHAT IT COMPUTES: for each routed (token, expert) assignment, the gate/up rows of the
// expert against the token's activation (k3_ops.c:1380-1785 for the MXFP4 dot, 628-630
// for SwiGLU), then the down rows against silu(gate) * up. Weights are read in the
// checkpoint layout (codes [rows][in/2], low nibble = even element; scales [rows][in/32]),
// so no repacking step exists.
//
// THE ACTIVATION OPERAND. The tensor core takes B in E2M1 too, so each fp32 activation
// vector is written as a sum of 16 E2M1 "pieces" with their own per-32 E8M0 scales:
//   r_0 = x;  piece p = round_to_E2M1(r_p / 2^s_p);  r_{p+1} = r_p - piece_p * 2^s_p,
// with s_0 the smallest exponent that fits the block maximum of |r_0| into [0, 6], then
// s_1 = s_0 - 2 and s_{p+1} = s_p - 3: rounding to the E2M1 grid {0, .5, 1, 1.5, 2, 3, 4, 6}
// leaves |r_1| <= 2^s_0 (grid spacing 2 in [4, 6]) and, once |r_p / 2^s_p| <= 4,
// |r_{p+1}| <= 2^(s_p - 1) (spacing at most 1), so every scaled residual stays within
// [-4, 4] and 16 pieces leave a residual below 2^-46 of the block maximum (in practice 0:
// the ~9 pieces that hold a float's 24 bits take all of it). Every step is exact in fp32
// (a power-of-two scaling, and a subtraction of the nearest grid point, a multiple of
// ulp(r / 2^s) no larger than r / 2^s). The schedule needs one block maximum per block,
// not one per piece. The 16 pieces are the 16 columns of B (N = 16): one MMA produces the
// 16 partial dot products of a 128-row tile, and the epilogue adds them. E8M0 code 255 in the
// weights (NaN to the hardware) is replaced by 0 (2^-127) on its way to tensor memory; the
// CPU engine treats 255 as zero, and 2^-127 * 6 * |piece| is below any fp32 output ulp.
//
// DATA MOVEMENT AND ROLES (one CTA per SM, 9 warps):
//   warps 0-3  producers: cp.async 16-byte copies of the weight tile (128 rows x 512
//              K-elements per stage) and of the B tile into the SWIZZLE_128B K-major
//              layout the MMA descriptors describe, and of the scale rows. Nothing in
//              the loop waits on memory: a thread publishes a stage three stages later,
//              once its copies for it have landed (cp.async.wait_group), after moving its
//              scale row, cleaned of 255, into the 32x16-byte atom tcgen05.cp reads and
//              fencing the stage for the tensor core's proxy.
//   warp 4     allocates 128 tensor-memory columns; one thread issues tcgen05.cp (scales)
//              and tcgen05.mma (8 MMAs of K = 64 per stage) and commits stage release and
//              accumulator completion to mbarriers.
//   warps 5-8  epilogue: tcgen05.ld of the 128 x 16 accumulator (two buffers, so the
//              epilogue of one item overlaps the MMAs of the next), the piece sum, and the
//              store of the partial result.
// Work items are (assignment, 128-row tile, K slice); K slices are summed in a fixed order
// by the consumer (no atomics, results are deterministic). Every mbarrier wait is bounded:
// on timeout the kernel stores K3D_ETIMEOUT in the device error flag, all roles leave
// their loops, outstanding copies and MMAs are drained, and tensor memory is freed.
#include "k3_moe.cuh"
#include "k3_ops.cuh"

namespace k3 {
namespace umma {

constexpr int kStageK = 512;                 // K elements per stage
constexpr int kRowBytes = kStageK / 2;       // packed bytes of one row per stage
constexpr int kN = 16;                       // B columns (pieces)
constexpr int kOffB = 128 * kRowBytes;       // 32768: A is 2 SW128 blocks of 128 x 128 B
constexpr int kOffSFA = kOffB + kN * kRowBytes;  // 36864
constexpr int kOffSFB = kOffSFA + 4 * 512;       // 38912
constexpr int kOffRawA = kOffSFB + 4 * 512;      // 40960: scale rows as loaded, 128 x 16 B
constexpr int kStageBytes = kOffRawA + 128 * 16;  // 43008 (multiple of 1024)
constexpr int kTileA = 32768, kTileSF = 2048, kTileB = 4096;   // tiled-layout units per stage
constexpr int kStages = 5;
constexpr int kLag = 3;                      // producer publishes a stage kLag stages later
constexpr int kProducers = 128;
constexpr int kThreads = 288;
constexpr int kTmemCols = 128;               // acc 4 x 16 @0, SFA 2 x 16 @64, SFB 2 x 16 @96
constexpr uint32_t kSfaCol = 64, kSfbCol = 96;
constexpr long long kSpinLimit = 4000000000LL;   // drain waits: ~2 s at 1.9 GHz

enum { GATEUP = 0, DOWN = 1 };

struct Job {
    const K3ExpertQ *table;
    K3ExpertQ single;
    int single_mode;
    const int *assign;       // grouped position -> assignment id (MoE mode)
    const int *idx;          // [assignments] expert id
    const int *count;        // device count of local assignments (MoE), else null
    int count_host;          // count when `count` is null
    int mode;
    int K;                   // reduction length
    int ntiles;              // gate/up: inter / 64; down: rows / 128
    int ks;                  // K slices per tile
    int cps;                 // stages per slice
    int nch;                 // stages along the whole K (K / 512)
    int tiled;               // 1: experts in the tiled layout (k3d_expert_pretile)
    const uint8_t *bq;       // B pieces [vec][16][K/2]
    const uint8_t *bs;       // B scales [vec][16][K/32]
    int vec_div;             // vector of assignment a = a / vec_div (unless vec_pos)
    int vec_pos;             // 1: B vector = grouped position p (down: act pieces by position)
    int out_pos;             // 1: partial row block = p (gate/up), else the assignment a
    int n_experts;           // MoE mode: expert ids must lie in [0, n_experts)
    const int *g_p0, *g_n, *g_e;   // grouped items: first position, tokens (<= 4) and expert
                                   // of each group; the count is the number of groups
    int early;               // 1: the work list and the weights do not depend on the kernel
                             //    launched just before (only the B operand does): the work
                             //    list is read and the first stages' weights are requested
                             //    before waiting for that kernel
    float *part;             // [ks][cap][out_w]
    int out_w;               // gate/up: 2 * inter (gate rows then up rows); down: rows
    size_t slice_stride;     // floats per K slice
};

__device__ __forceinline__ uint32_t saddr(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(b), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint32_t b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(b) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t b, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(b), "r"(parity) : "memory");
    return ok != 0;
}

// try_wait that lets the hardware suspend the thread until the phase completes or about
// `ns` nanoseconds pass, so a waiting role does not take issue slots from the warps that
// share its scheduler.
__device__ __forceinline__ bool mbar_try_sleep(uint32_t b, uint32_t parity, uint32_t ns)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(b), "r"(parity), "r"(ns) : "memory");
    return ok != 0;
}

// Bounded wait; false when it gave up (time limit, or another role already aborted).
__device__ __forceinline__ bool mbar_wait(uint32_t b, uint32_t parity, volatile int *abort)
{
    if (mbar_try(b, parity)) return true;
    const long long t0 = clock64(), lim = k3_wait_cycles;
    while (!mbar_try_sleep(b, parity, 1000u)) {
        if (*abort) return false;
        if (clock64() - t0 > lim) {
            k3_raise(K3D_ETIMEOUT, K3_SITE_MXFP4);
            *abort = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(b), "r"(bytes) : "memory");
}

// 1-D bulk copy global -> shared, completing on an mbarrier (no multicast)
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// Bounded wait that ignores the abort flag: used to drain in-flight tensor-core work
// before tensor memory is freed.
__device__ __forceinline__ void mbar_drain(uint32_t b, uint32_t parity)
{
    const long long t0 = clock64();
    while (!mbar_try(b, parity)) {
        if (clock64() - t0 > kSpinLimit) { k3_raise(K3D_ETIMEOUT, K3_SITE_MXFP4); return; }
    }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major SWIZZLE_128B: 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t a)
{
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Descriptor of one 32-row x 16-byte scale atom (no swizzle; 8-row groups 128 B apart).
__device__ __forceinline__ uint64_t desc_sf(uint32_t a)
{
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 32) | ((uint64_t)1 << 46);
}

// Instruction descriptor: kind::mxf4, A and B E2M1 (format 1), UE8M0 scales, K-major
// operands, M = 128, N = 16, scale-factor byte ids for A and B.
template <int N>
__device__ __forceinline__ uint32_t idesc_mxf4(uint32_t sf_id)
{
    return (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
           ((uint32_t)(128 >> 4) << 24) | (sf_id << 29) | (sf_id << 4);
}

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t accum, uint32_t sfa, uint32_t sfb)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
                 :: "r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum), "r"(sfa), "r"(sfb)
                 : "memory");
}

__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc)
{
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" :: "r"(taddr), "l"(sdesc) : "memory");
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

// 0xFF bytes (E8M0 NaN) -> 0x00, bytewise on a 32-bit word
__device__ __forceinline__ uint32_t clean_e8m0(uint32_t w)
{
    const uint32_t lo7 = w & 0x7F7F7F7Fu;
    const uint32_t ff = ((lo7 + 0x01010101u) & w) & 0x80808080u;   // high bit set iff byte == 0xFF
    const uint32_t mask = (ff >> 7) * 0xFFu;
    return w & ~mask;
}

// Once this thread's copies for a stage have landed (checkpoint layout only): move its
// scale row into the 32x16-byte atom tcgen05.cp reads (row m of the 128-row operand at
// byte 16*(m%32) + 4*(m/32), blocks 4a..4a+3 in atom a), cleaned of 255, then make the
// stage's shared-memory writes visible to the tensor core.
__device__ __forceinline__ void publish(unsigned char *st, int tid)
{
    const uint4 v = *reinterpret_cast<const uint4 *>(st + kOffRawA + 16 * tid);
    uint32_t *atom = reinterpret_cast<uint32_t *>(st + kOffSFA + 16 * (tid & 31) + 4 * (tid >> 5));
    atom[0] = clean_e8m0(v.x);
    atom[128] = clean_e8m0(v.y);
    atom[256] = clean_e8m0(v.z);
    atom[384] = clean_e8m0(v.w);
    fence_async_smem();
}

// One work item as the roles need it, resolved once per round into shared memory so
// that no role's loop waits on a dependent chain of global loads (assignment -> expert id
// -> expert table entry).
struct ItemEnt {
    const uint8_t *c0, *c1, *s0, *s1;   // weight codes / scales (gate and up, or down twice)
    int out;                            // partial row block (position or assignment; grouped:
                                        // the first of nv consecutive positions)
    int tile, s;                        // 128-row tile, K slice
    int vec;                            // B operand vector (grouped: the group)
    int nv;                             // vectors of the item (1, or up to 4 when grouped)
    int pad[3];
};
static_assert(sizeof(ItemEnt) == 64, "item entry size");
constexpr int kMaxItems = 128;          // table entries per round
constexpr int kOffItems = 1024;         // after the barrier header
constexpr int kStage0 = kOffItems + kMaxItems * 64;   // 9216, 1024-aligned
constexpr int kAccBufs = 4;             // accumulator ring depth

// Stage geometry for NV activation vectors per item. NV = 1: one vector (the assignment's
// token) per item, B = 16 piece rows. NV = 4 (grouped): up to four tokens routed to the
// same expert share each weight stage; B stacks their pieces as 64 rows (row 16 v + p =
// piece p of slot v), one MMA of N = 64 per K step, and the scale atoms hold B row m at
// byte 16 (m % 32) + 4 (m / 32) + block (the layout of A's 128 rows).
template <int NV, int RES = 0>
struct Geo {
    static constexpr int kVec = NV;                             // vectors per item
    static constexpr int kBTile = NV * kTileB;                  // B tile per stage
    static constexpr int kB = kTileA;                           // 32768
    static constexpr int kSFA = kB + kBTile;
    static constexpr int kSFB = kSFA + kTileSF;
    static constexpr int kBytes = NV == 1 ? kStageBytes : kSFB + kTileSF;
    static constexpr int kNStages = NV == 1 ? kStages : 4;
    static constexpr int kCols = kN * NV;                       // MMA N, accumulator columns
    static constexpr int kTmem = NV == 1 ? kTmemCols : 512;
    static constexpr uint32_t kSfaCol = NV == 1 ? umma::kSfaCol : 256;
    static constexpr uint32_t kSfbCol = NV == 1 ? umma::kSfbCol : 288;
    static constexpr uint32_t kTx = kTileA + kTileSF + kBTile + kTileSF;
    static constexpr size_t kSmem = 1024 + kStage0 + (size_t)kNStages * kBytes;
    static_assert(kBytes % 1024 == 0, "stage alignment");
    static_assert(kAccBufs * kCols + 64 <= kTmem, "tensor memory");
};

// RES = 1 (resident B): one stage per item, items ordered (vector or group, K chunk,
// tile), so consecutive items share their B chunk: B and its scale atoms are loaded once
// per run of items into one of two slots beside the ring, and the ring's stages carry only
// the weight tile and its scales (34 KB), six of them for one vector (five when B rode
// along) and five for a group of four (four when B rode along); B's scales go to tensor
// memory once per run instead of once per stage.
template <int NV>
struct Geo<NV, 1> {
    static constexpr int kVec = NV;
    static constexpr int kSFA = kTileA;                         // 32768
    static constexpr int kBytes = kTileA + kTileSF;             // 34816
    static constexpr int kNStages = NV == 1 ? 6 : 5;
    static constexpr int kCols = kN * NV;
    static constexpr int kTmem = NV == 1 ? kTmemCols : 512;
    static constexpr uint32_t kSfaCol = NV == 1 ? umma::kSfaCol : 256;
    static constexpr uint32_t kSfbCol = NV == 1 ? umma::kSfbCol : 288;   // 16 columns per slot
    static constexpr uint32_t kTx = kTileA + kTileSF;
    static constexpr int kBTile = NV * kTileB;
    static constexpr int kBSlot = kBTile + kTileSF;             // B tile, then its atoms
    static constexpr int kBSlots = kStage0 + kNStages * kBytes; // offset of the two slots
    static constexpr size_t kSmem = 1024 + kBSlots + 2 * kBSlot;
    static_assert(kBytes % 1024 == 0 && kBSlots % 1024 == 0 && kBSlot % 1024 == 0, "alignment");
    static_assert(kSmem <= 232448, "shared memory");
    static_assert(kAccBufs * kCols <= (int)kSfaCol && kSfbCol + 32 <= (uint32_t)kTmem, "tensor memory");
};

template <int NV, int RES>
__device__ __forceinline__ ItemEnt decode(const Job &J, int item)
{
    ItemEnt it;
    it.s = item % J.ks;
    int rest, p;
    if (RES) {
        // (vector or group, K chunk, tile), tile fastest (one stage per item)
        it.tile = item % J.ntiles;
        rest = item / J.ntiles;
        it.s = rest % J.ks;
        p = rest / J.ks;
    } else {
        rest = item / J.ks;
        it.tile = rest % J.ntiles;
        p = rest / J.ntiles;
    }
    it.nv = 1;
    it.pad[0] = it.pad[1] = it.pad[2] = 0;
    if (NV > 1) {
        // p is a group: nv consecutive positions of one expert
        const int nv = __ldcg(J.g_n + p), e = __ldcg(J.g_e + p);
        if (e < 0 || e >= J.n_experts || nv < 1 || nv > NV) {
            k3_raise(K3D_EBOUND, K3_SITE_MXFP4);
            it.c0 = it.c1 = it.s0 = it.s1 = nullptr;
            it.out = it.tile = it.s = it.vec = 0;
            return it;
        }
        const K3ExpertQ q = J.table[e];
        if (J.mode == GATEUP) { it.c0 = q.p1; it.c1 = q.p3; it.s0 = q.s1; it.s1 = q.s3; }
        else { it.c0 = it.c1 = q.p2; it.s0 = it.s1 = q.s2; }
        it.out = __ldcg(J.g_p0 + p);
        it.vec = p;
        it.nv = nv;
        return it;
    }
    int a;
    K3ExpertQ q;
    if (J.single_mode) {
        a = p;
        q = J.single;
    } else {
        a = __ldcg(J.assign + p);
        const int e = (a >= 0 && a < J.count_host) ? __ldcg(J.idx + a) : -1;
        if (e < 0 || e >= J.n_experts) {
            // a corrupt work list: the item is skipped (no copies), the error recorded
            k3_raise(K3D_EBOUND, K3_SITE_MXFP4);
            it.c0 = it.c1 = it.s0 = it.s1 = nullptr;
            it.out = 0;
            it.tile = it.s = 0;
            it.vec = 0;
            return it;
        }
        q = J.table[e];
    }
    if (J.mode == GATEUP) { it.c0 = q.p1; it.c1 = q.p3; it.s0 = q.s1; it.s1 = q.s3; }
    else { it.c0 = it.c1 = q.p2; it.s0 = it.s1 = q.s2; }
    it.out = J.out_pos ? p : a;
    it.vec = J.vec_pos ? p : a / J.vec_div;
    return it;
}

__device__ __forceinline__ int item_count(const Job &J)
{
    const int n = J.count ? *(volatile const int *)J.count : J.count_host;
    return n * J.ntiles * J.ks;
}

__device__ __forceinline__ bool item_ok(const ItemEnt &it)
{
    return it.c0 && ((((uintptr_t)it.c0 | (uintptr_t)it.s0) & 15u) == 0);
}

// Tiled layout: the weight tile of one stage and its scale atoms, completing on `fb`.
template <int NV, int RES>
__device__ __forceinline__ void issue_weights(uint32_t sb, uint32_t fb, const Job &J, const ItemEnt &it,
                                              int chunk)
{
    const size_t tix = (size_t)chunk * J.ntiles + it.tile;
    bulk_g2s(sb, it.c0 + tix * kTileA, kTileA, fb);
    bulk_g2s(sb + Geo<NV, RES>::kSFA, it.s0 + tix * kTileSF, kTileSF, fb);
}

// The B tile of one stage and its scale atoms, completing on `fb`.
template <int NV>
__device__ __forceinline__ void issue_operand(uint32_t sb, uint32_t fb, const Job &J, const ItemEnt &it,
                                              int chunk)
{
    const size_t vix = (size_t)it.vec * J.nch + chunk;
    bulk_g2s(sb + Geo<NV>::kB, J.bq + vix * Geo<NV>::kBTile, Geo<NV>::kBTile, fb);
    bulk_g2s(sb + Geo<NV>::kSFB, J.bs + vix * kTileSF, kTileSF, fb);
}

// MMA issuer (one thread): the J.cps stages of each of `nr` items into the accumulator
// buffer of the item, releasing each stage and publishing each accumulator on its
// mbarrier. The stage and item positions carry across calls. False when a wait gave up.
template <int NV>
__device__ __forceinline__ bool mma_items(const Job &J, int nr, int &g_mma, int &n_mma, uint32_t tmem,
                                          uint32_t stage0, uint32_t b_full, uint32_t b_empty,
                                          uint32_t b_accf, uint32_t b_acce, volatile int *abort)
{
    using G = Geo<NV>;
    for (int k = 0; k < nr; k++, n_mma++) {
        const int buf = n_mma % kAccBufs;
        if (n_mma >= kAccBufs && !mbar_wait(b_acce + 8 * buf, ((n_mma / kAccBufs) - 1) & 1, abort))
            return false;
        tc_fence_after();
        const uint32_t dcol = tmem + (uint32_t)(buf * G::kCols);
        for (int c = 0; c < J.cps; c++) {
            const int st = g_mma % G::kNStages;
            if (!mbar_wait(b_full + 8 * st, (g_mma / G::kNStages) & 1, abort)) return false;
            tc_fence_after();
            const uint32_t sb = stage0 + (uint32_t)st * G::kBytes;
            const uint32_t sfa = tmem + G::kSfaCol + (uint32_t)((g_mma & 1) * 16);
            const uint32_t sfb = tmem + G::kSfbCol + (uint32_t)((g_mma & 1) * 16);
#pragma unroll
            for (int a4 = 0; a4 < 4; a4++) {
                tc_cp_sf(sfa + 4 * a4, desc_sf(sb + G::kSFA + 512 * a4));
                tc_cp_sf(sfb + 4 * a4, desc_sf(sb + G::kSFB + 512 * a4));
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t kb = (uint32_t)(j >> 2), off = (uint32_t)((j & 3) * 32);
                const uint64_t ad = desc_sw128(sb + kb * 16384u + off);
                const uint64_t bd = desc_sw128(sb + G::kB + kb * (uint32_t)(NV * 2048) + off);
                const uint32_t id = (uint32_t)((j & 1) * 2);
                // blocks 2j, 2j+1: the scales in atom j/2 (a scale address is a 4-column
                // group); the byte id picks the pair
                const uint32_t atom = (uint32_t)(4 * (j >> 1));
                tc_mma(dcol, ad, bd, idesc_mxf4<G::kCols>(id), (c > 0 || j > 0) ? 1u : 0u,
                       (sfa + atom) | (id << 30), (sfb + atom) | (id << 30));
            }
            tc_commit(b_empty + 8 * st);
            g_mma++;
        }
        tc_commit(b_accf + 8 * buf);
    }
    return true;
}

// Runs of items sharing a B chunk (the resident-B geometry): true when item `it` starts a
// new run after (vec, chunk).
__device__ __forceinline__ bool new_run(const ItemEnt &it, int vec, int chunk)
{
    return it.vec != vec || it.s != chunk;
}

// MMA issuer of the resident-B geometry: one stage per item; at the start of each run the
// previous run's B slot is released (a commit: it frees once that run's MMAs finish) and
// the new slot's scale atoms are copied to tensor memory after its B has landed.
template <int NV>
__device__ __forceinline__ bool mma_items_rb(const Job &J, const ItemEnt *items, int nr, int &g_mma, int &n_mma,
                                             int &rb_n, int &rb_vec, int &rb_chunk, uint32_t tmem,
                                             uint32_t stage0, uint32_t bslots, uint32_t b_full,
                                             uint32_t b_empty, uint32_t b_accf, uint32_t b_acce,
                                             uint32_t b_bfull, uint32_t b_bempty, volatile int *abort)
{
    using G = Geo<NV, 1>;
    for (int k = 0; k < nr; k++, n_mma++) {
        const ItemEnt &it = items[k];
        const int buf = n_mma % kAccBufs;
        if (n_mma >= kAccBufs && !mbar_wait(b_acce + 8 * buf, ((n_mma / kAccBufs) - 1) & 1, abort))
            return false;
        tc_fence_after();
        if (new_run(it, rb_vec, rb_chunk)) {
            if (rb_n > 0) tc_commit(b_bempty + 8 * ((rb_n - 1) & 1));
            const int slot = rb_n & 1;
            if (!mbar_wait(b_bfull + 8 * slot, (rb_n >> 1) & 1, abort)) return false;
            tc_fence_after();
            const uint32_t sfb = tmem + G::kSfbCol + (uint32_t)(slot * 16);
#pragma unroll
            for (int a4 = 0; a4 < 4; a4++)
                tc_cp_sf(sfb + 4 * a4, desc_sf(bslots + (uint32_t)(slot * G::kBSlot + G::kBTile + 512 * a4)));
            rb_n++;
            rb_vec = it.vec;
            rb_chunk = it.s;
        }
        const int slot = (rb_n - 1) & 1;
        const uint32_t bs = bslots + (uint32_t)(slot * G::kBSlot);
        const uint32_t sfb = tmem + G::kSfbCol + (uint32_t)(slot * 16);
        const uint32_t dcol = tmem + (uint32_t)(buf * G::kCols);
        const int st = g_mma % G::kNStages;
        if (!mbar_wait(b_full + 8 * st, (g_mma / G::kNStages) & 1, abort)) return false;
        tc_fence_after();
        const uint32_t sb = stage0 + (uint32_t)st * G::kBytes;
        const uint32_t sfa = tmem + G::kSfaCol + (uint32_t)((g_mma & 1) * 16);
#pragma unroll
        for (int a4 = 0; a4 < 4; a4++) tc_cp_sf(sfa + 4 * a4, desc_sf(sb + G::kSFA + 512 * a4));
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t kb = (uint32_t)(j >> 2), off = (uint32_t)((j & 3) * 32);
            const uint64_t ad = desc_sw128(sb + kb * 16384u + off);
            const uint64_t bd = desc_sw128(bs + kb * (uint32_t)(NV * 2048) + off);
            const uint32_t id = (uint32_t)((j & 1) * 2);
            const uint32_t atom = (uint32_t)(4 * (j >> 1));
            tc_mma(dcol, ad, bd, idesc_mxf4<G::kCols>(id), j > 0 ? 1u : 0u, (sfa + atom) | (id << 30),
                   (sfb + atom) | (id << 30));
        }
        tc_commit(b_empty + 8 * st);
        g_mma++;
        tc_commit(b_accf + 8 * buf);
    }
    return true;
}

// Epilogue warp of tensor-memory lane quadrant q: for each of `nr` items, its 32 rows of
// the 128 x 16 accumulator, summed over the 16 pieces and stored as the item's partial.
// False when a wait gave up.
template <int NV, int RES>
__device__ __forceinline__ bool epilogue_items(const Job &J, const ItemEnt *items, int nr, int &n_epi,
                                               uint32_t tmem, uint32_t b_accf, uint32_t b_acce,
                                               volatile int *abort, int q, int lane)
{
    using G = Geo<NV, RES>;
    const int m = q * 32 + lane;            // tile row
    for (int k = 0; k < nr; k++, n_epi++) {
        const ItemEnt &it = items[k];
        int row;
        if (J.mode == GATEUP) row = m < 64 ? it.tile * 64 + m : (J.out_w >> 1) + it.tile * 64 + (m - 64);
        else row = it.tile * 128 + m;
        float *dst = J.part + (size_t)it.s * J.slice_stride + (size_t)it.out * J.out_w + row;
        const int buf = n_epi % kAccBufs;
        if (!mbar_wait(b_accf + 8 * buf, (n_epi / kAccBufs) & 1, abort)) return false;
        tc_fence_after();
        float v[G::kCols];
#pragma unroll
        for (int u = 0; u < G::kVec; u++)
            tc_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * G::kCols + u * kN), v + u * kN);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(b_acce + 8 * buf);
        // each vector's 16 pieces, smallest first; vector u is position out + u
#pragma unroll
        for (int u = 0; u < G::kVec; u++) {
            if (u >= it.nv) break;
            float sum = v[u * kN + 15];
#pragma unroll
            for (int i = 14; i >= 0; i--) sum += v[u * kN + i];
            dst[(size_t)u * J.out_w] = sum;
        }
    }
    return true;
}

template <int NV, int RES>
__global__ void __launch_bounds__(kThreads, 1) k_mxfp4_umma(Job J)
{
    using G = Geo<NV, RES>;
    extern __shared__ unsigned char smem_raw[];
    // 1024-aligned base (the SWIZZLE_128B pattern is a function of the absolute address)
    const uint32_t raw = saddr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char *gbase = smem_raw + (base - raw);
    // header: barriers, abort flag, tensor-memory address slot
    const uint32_t b_full = base;                       // [8] x 8 (G::kNStages used)
    const uint32_t b_empty = base + 64;                 // [8] x 8
    const uint32_t b_accf = base + 128;                 // [kAccBufs] x 8
    const uint32_t b_acce = b_accf + 8 * kAccBufs;      // [kAccBufs] x 8
    const uint32_t b_drain = b_acce + 8 * kAccBufs;
    const uint32_t b_bfull = b_drain + 8;               // [2] x 8: resident B slots (NV = 0)
    const uint32_t b_bempty = b_bfull + 16;             // [2] x 8
    static_assert(G::kNStages <= 8, "barrier header");
    volatile int *abort = reinterpret_cast<volatile int *>(gbase + 512);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + 520);
    ItemEnt *items = reinterpret_cast<ItemEnt *>(gbase + kOffItems);
    const uint32_t stage0 = base + kStage0;
    unsigned char *gstage0 = gbase + kStage0;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::kNStages; s++) {
            mbar_init(b_full + 8 * s, J.tiled ? 1 : kProducers);
            mbar_init(b_empty + 8 * s, 1);
        }
        for (int i = 0; i < kAccBufs; i++) { mbar_init(b_accf + 8 * i, 1); mbar_init(b_acce + 8 * i, 4); }
        mbar_init(b_drain, 1);
        for (int i = 0; i < 2; i++) { mbar_init(b_bfull + 8 * i, 1); mbar_init(b_bempty + 8 * i, 1); }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(saddr(tmem_slot)), "r"(G::kTmem) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // programmatic dependent launch: the set-up above overlapped the kernel before this
    // one; unless the work list is independent of it, wait for it before reading the list
    if (!J.early) pdl_wait();

    const int total = item_count(J);
    const int i_beg = (int)((long long)blockIdx.x * total / gridDim.x);
    const int i_end = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    const int rowbytes = J.K >> 1;
    const int sfrow = J.K >> 5;

    // pipeline positions, carried across rounds
    int g_prod = 0;      // stages issued by this producer thread
    int g_mma = 0;       // stages consumed by the MMA thread
    int n_mma = 0;       // items issued by the MMA thread
    int n_epi = 0;       // items finished by this epilogue warp
    bool stop = false;
    // resident-B runs (RES = 1): runs begun and the current run's (vector, chunk), kept by
    // the producer and the MMA issuer each
    int rb_n = 0, rb_vec = -1, rb_chunk = -1;
    const uint32_t bslots = base + (uint32_t)(RES ? Geo<NV, 1>::kBSlots : 0);

    for (int r0 = i_beg; r0 < i_end; r0 += kMaxItems) {
        const int r1 = min(i_end, r0 + kMaxItems);
        for (int i = r0 + threadIdx.x; i < r1; i += blockDim.x) items[i - r0] = decode<NV, RES>(J, i);
        __syncthreads();
        const int nr = r1 - r0;
        const bool prefetch = J.early && J.tiled && r0 == i_beg;
        if (r0 == i_beg) {
            // early: everyone but the tiled producer (which first requests the weights of
            // its first stages) waits for the kernel before this one here
            if (J.early && !(prefetch && threadIdx.x == 0)) pdl_wait();
            pdl_trigger();
        }

        if (RES && warp < 4) {
          if constexpr (RES == 1) {
            // ------------------- producer, resident B: one thread; a run's B chunk and its
            // atoms once into a slot, each stage the weight tile and its scale atoms
            if (threadIdx.x == 0) {
                int pre = 0;
                if (prefetch) {
                    // early launch: the first stages' weights before the programmatic wait,
                    // three of the six: when every CTA has six 34 KB stages in flight (30 MB)
                    // as the wait returns, the B operand requested then lands only as they
                    // drain, about 4.5 us later (a plain-load copy of B waits as long); with
                    // three, B comes sooner and the stream starts earlier (down pass 23.0 ->
                    // 21.6 us in the stack; two and four measured slower than three)
                    pre = min(3, nr);
                    for (int h = 0; h < pre; h++) {
                        const ItemEnt &it = items[h];
                        if (!item_ok(it)) continue;
                        const int st = (g_prod + h) % G::kNStages;
                        const uint32_t fb = b_full + 8 * st;
                        mbar_expect_tx(fb, G::kTx);
                        issue_weights<NV, RES>(stage0 + (uint32_t)st * G::kBytes, fb, J, it, it.s);
                    }
                    pdl_wait();
                }
                for (int k = 0; k < nr && !stop; k++) {
                    const ItemEnt &it = items[k];
                    const bool aligned = item_ok(it);
                    if (!aligned) k3_raise(K3D_EINVAL, K3_SITE_MXFP4);
                    if (new_run(it, rb_vec, rb_chunk)) {
                        const int slot = rb_n & 1;
                        if (rb_n >= 2 && !mbar_wait(b_bempty + 8 * slot, ((rb_n >> 1) - 1) & 1, abort)) {
                            stop = true;
                            break;
                        }
                        const uint32_t bb = b_bfull + 8 * slot, dst = bslots + (uint32_t)(slot * G::kBSlot);
                        const size_t vix = (size_t)it.vec * J.nch + it.s;
                        mbar_expect_tx(bb, G::kBTile + kTileSF);
                        bulk_g2s(dst, J.bq + vix * G::kBTile, G::kBTile, bb);
                        bulk_g2s(dst + G::kBTile, J.bs + vix * kTileSF, kTileSF, bb);
                        rb_n++;
                        rb_vec = it.vec;
                        rb_chunk = it.s;
                    }
                    if (k < pre) { g_prod++; continue; }     // weights issued above
                    const int st = g_prod % G::kNStages;
                    if (g_prod >= G::kNStages &&
                        !mbar_wait(b_empty + 8 * st, ((g_prod / G::kNStages) - 1) & 1, abort)) {
                        stop = true;
                        break;
                    }
                    const uint32_t fb = b_full + 8 * st;
                    if (aligned) {
                        mbar_expect_tx(fb, G::kTx);
                        issue_weights<NV, RES>(stage0 + (uint32_t)st * G::kBytes, fb, J, it, it.s);
                    } else {
                        mbar_arrive(fb);
                    }
                    g_prod++;
                }
            }
          }
        } else if (warp < 4 && J.tiled) {
          if constexpr (RES == 0) {
            // ------------------------------------------ producer, tiled layout: one thread
            // streams each stage as four bulk copies (weight tile, its scale atoms, the B
            // tile and its scale atoms), all completing on the stage's mbarrier
            if (threadIdx.x == 0) {
                // early launch: the weight tiles and scale atoms of the first stages are
                // requested before waiting for the kernel that writes the B operand
                int pre = 0;
                if (prefetch) {
                    pre = min(G::kNStages, nr * J.cps);
                    for (int h = 0; h < pre; h++) {
                        const ItemEnt &it = items[h / J.cps];
                        if (!item_ok(it)) continue;
                        const uint32_t sb = stage0 + (uint32_t)((g_prod + h) % G::kNStages) * G::kBytes;
                        const uint32_t fb = b_full + 8 * ((g_prod + h) % G::kNStages);
                        mbar_expect_tx(fb, G::kTx);
                        issue_weights<NV, RES>(sb, fb, J, it, it.s * J.cps + h % J.cps);
                    }
                    pdl_wait();
                    for (int h = 0; h < pre; h++) {
                        const ItemEnt &it = items[h / J.cps];
                        const uint32_t fb = b_full + 8 * ((g_prod + h) % G::kNStages);
                        if (!item_ok(it)) {
                            k3_raise(K3D_EINVAL, K3_SITE_MXFP4);
                            mbar_arrive(fb);
                            continue;
                        }
                        const uint32_t sb = stage0 + (uint32_t)((g_prod + h) % G::kNStages) * G::kBytes;
                        issue_operand<NV>(sb, fb, J, it, it.s * J.cps + h % J.cps);
                    }
                }
                int h = 0;       // stage index within this round
                for (int k = 0; k < nr && !stop; k++) {
                    const ItemEnt &it = items[k];
                    const bool aligned = item_ok(it);
                    if (!aligned) k3_raise(K3D_EINVAL, K3_SITE_MXFP4);
                    for (int c = 0; c < J.cps; c++, h++) {
                        if (h < pre) { g_prod++; continue; }     // issued above
                        const int chunk = it.s * J.cps + c;
                        const int st = g_prod % G::kNStages;
                        if (g_prod >= G::kNStages &&
                            !mbar_wait(b_empty + 8 * st, ((g_prod / G::kNStages) - 1) & 1, abort)) {
                            stop = true;
                            break;
                        }
                        const uint32_t sb = stage0 + (uint32_t)st * G::kBytes;
                        const uint32_t fb = b_full + 8 * st;
                        if (aligned) {
                            mbar_expect_tx(fb, G::kTx);
                            issue_weights<NV, RES>(sb, fb, J, it, chunk);
                            issue_operand<NV>(sb, fb, J, it, chunk);
                        } else {
                            mbar_arrive(fb);
                        }
                        g_prod++;
                    }
                }
            }
          }
        } else if (warp < 4) {
          if constexpr (NV == 1 && RES == 0) {
            // -------------------------- producers, checkpoint layout: 128 threads, cp.async
            const int tid = threadIdx.x;
            const int g_round = g_prod;          // stages of this round are published here
            for (int k = 0; k < nr && !stop; k++) {
                const ItemEnt &it = items[k];
                const int r0w = J.mode == GATEUP ? it.tile * 64 : it.tile * 128;
                const bool aligned = it.c0 && it.c1 &&
                                     ((((uintptr_t)it.c0 | (uintptr_t)it.c1 | (uintptr_t)it.s0 |
                                        (uintptr_t)it.s1) & 15u) == 0);
                if (!aligned && tid == 0) k3_raise(K3D_EINVAL, K3_SITE_MXFP4);
                const size_t vbase = (size_t)it.vec * J.nch;
                for (int c = 0; c < J.cps; c++) {
                    const int chunk = it.s * J.cps + c;
                    const int st = g_prod % kStages;
                    if (g_prod >= kStages &&
                        !mbar_wait(b_empty + 8 * st, ((g_prod / kStages) - 1) & 1, abort)) {
                        stop = true;
                        break;
                    }
                    const uint32_t sb = stage0 + (uint32_t)st * kStageBytes;
                    if (aligned) {
                        // A: 128 rows x 16 chunks of 16 B into the SWIZZLE_128B layout; a
                        // warp reads 2 full row segments
#pragma unroll 4
                        for (int i = 0; i < 16; i++) {
                            const int qd = tid + kProducers * i;
                            const int r = qd >> 4, j = qd & 15;
                            const uint8_t *src_row = (J.mode == GATEUP && r >= 64)
                                ? it.c1 + (size_t)(r0w + r - 64) * rowbytes
                                : it.c0 + (size_t)(r0w + r) * rowbytes;
                            const uint32_t dst = sb + (uint32_t)((j >> 3) * 16384 + (r >> 3) * 1024 +
                                                                 (r & 7) * 128 + (((j & 7) ^ (r & 7)) << 4));
                            cp_async16(dst, src_row + (size_t)chunk * kRowBytes + j * 16);
                        }
                        // B tile and its scale atoms are stored ready-made: straight copies
                        const uint8_t *btile = J.bq + (vbase + chunk) * kTileB;
                        const uint8_t *bsf = J.bs + (vbase + chunk) * kTileSF;
                        cp_async16(sb + kOffB + 16 * tid, btile + 16 * tid);
                        cp_async16(sb + kOffB + 16 * (tid + kProducers), btile + 16 * (tid + kProducers));
                        cp_async16(sb + kOffSFB + 16 * tid, bsf + 16 * tid);
                        // the scale row as it is in memory; rearranged when the stage is
                        // published (below), so no load blocks this loop
                        const uint8_t *srow = (J.mode == GATEUP && tid >= 64)
                            ? it.s1 + (size_t)(r0w + tid - 64) * sfrow
                            : it.s0 + (size_t)(r0w + tid) * sfrow;
                        cp_async16(sb + kOffRawA + 16 * tid, srow + (size_t)chunk * 16);
                    }
                    cp_commit();
                    if (g_prod - g_round >= kLag) {
                        cp_wait<kLag>();
                        publish(gstage0 + (size_t)((g_prod - kLag) % kStages) * kStageBytes, tid);
                        mbar_arrive(b_full + 8 * ((g_prod - kLag) % kStages));
                    }
                    g_prod++;
                }
            }
            // publish the round's last stages before the round barrier
            cp_wait_all();
            const int h0 = max(g_round, g_prod - kLag);
            for (int h = h0; h < g_prod; h++) {
                publish(gstage0 + (size_t)(h % kStages) * kStageBytes, tid);
                mbar_arrive(b_full + 8 * (h % kStages));
            }
          }
        } else if (warp == 4) {
            // ----------------------------------------------------------- MMA issuer
            if (lane == 0 && !stop) {
                bool ok;
                if constexpr (RES == 1)
                    ok = mma_items_rb<NV>(J, items, nr, g_mma, n_mma, rb_n, rb_vec, rb_chunk, tmem, stage0, bslots,
                                      b_full, b_empty, b_accf, b_acce, b_bfull, b_bempty, abort);
                else
                    ok = mma_items<NV>(J, nr, g_mma, n_mma, tmem, stage0, b_full, b_empty, b_accf, b_acce, abort);
                if (!ok) stop = true;
            }
            __syncwarp();
        } else {
            // ------------------------------------------------------------- epilogue
            epilogue_items<NV, RES>(J, items, nr, n_epi, tmem, b_accf, b_acce, abort, warp & 3, lane);
        }
        __syncthreads();          // every role is done with this round's table
    }
    if (warp == 4 && lane == 0) {
        // every MMA and copy issued above has completed once this barrier flips
        tc_commit(b_drain);
        mbar_drain(b_drain, 0);
    }
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem), "r"(G::kTmem) : "memory");
    }
}

// ---------------------------------------------------------------- activation split
// The B operand of one vector, stored ready for the kernel's stages: for each 512-element
// chunk c, a 4 KB tile (16 piece rows x 256 bytes in the SWIZZLE_128B K-major layout) at
// bq + 4096 c, and 4 scale atoms at bs + 2048 c (piece p's scale for block 4a+i at byte
// 512 a + 16 p + i; every other byte of an atom is zero).
//
// One lane per element of a 32-element block. From the block maximum m of |x| (one redux
// on the bits: non-negative floats order like their bits):
//   s_0 = e - 2 if m <= 1.5 * 2^e else e - 1 (e = floor(log2 m)), so m / 2^s_0 lies in
//   (3, 6]; from the bits, the E8M0 code is s_0 + 127 = E - 2 + (mantissa > 0x400000);
//   the later codes follow the schedule s_1 = s_0 - 2, s_{p+1} = s_p - 3; every code is
//   clamped at 0 (blocks below 2^-80 or so share the smallest scale, 2^-127, which only
//   makes their scaled residuals smaller);
//   per piece, the E2M1 code of r / 2^s rounded to nearest even (e2m1_rne; the scaled value
//   never exceeds 6, so saturation never acts), its value q, and the residual
//   (r / 2^s - q) * 2^s.
// A block holding an inf or NaN gets scale code 255 (NaN) on every piece, zero codes.

// Round to the nearest E2M1 value, ties to the even code, for |v| <= 6 (saturating above,
// as the hardware conversion's satfinite does): the value and its 4-bit code (sign bit 8;
// zero always +0). Plain float arithmetic, exact at every step (a power-of-two scaling and
// an integer rounding), so it equals cvt.rn.satfinite.e2m1x2.f32 on this range, without
// branches.
__device__ __forceinline__ float e2m1_rne(float v, uint32_t &nib)
{
    // grid spacing 0.5 below 2, 1 below 4, 2 up to 6: scale to unit spacing, round to the
    // nearest integer (ties to even, which is the even code), scale back; no branches
    const float a = fabsf(v);
    const float up = a < 2.0f ? 2.0f : (a < 4.0f ? 1.0f : 0.5f);
    const float dn = a < 2.0f ? 0.5f : (a < 4.0f ? 1.0f : 2.0f);
    const float q = fminf(rintf(a * up) * dn, 6.0f);
    // the code from q's bits: 2 (exponent - 127) + top mantissa bit + 2 from 1 up, 1 for 0.5
    const uint32_t bits = __float_as_uint(q);
    const uint32_t code = q >= 1.0f ? 2u * ((bits >> 23) - 127u) + ((bits >> 22) & 1u) + 2u : (q > 0.0f ? 1u : 0u);
    nib = code ? (code | (v < 0.0f ? 8u : 0u)) : 0u;
    return code ? (v < 0.0f ? -q : q) : 0.0f;
}

// The 32 codes of one piece of a block (lane l holds element l's nibble) as the 16 bytes of
// its B row segment: lanes 0, 8, 16 and 24 return one 32-bit word each (bytes 0-3, 4-7, 8-11,
// 12-15; the low nibble of byte i is element 2i), the other lanes garbage: four 32-bit
// stores per piece instead of sixteen byte stores.
__device__ __forceinline__ uint32_t piece_word(uint32_t nib)
{
    const uint32_t b = nib | (__shfl_down_sync(0xffffffffu, nib, 1) << 4);
    return b | (__shfl_down_sync(0xffffffffu, b, 2) << 8) | (__shfl_down_sync(0xffffffffu, b, 4) << 16) |
           (__shfl_down_sync(0xffffffffu, b, 6) << 24);
}

// Piece p of one element's split: the E2M1 code (nibble) of the residual r at the
// schedule's scale, r replaced by what remains; lane p records the scale code.
__device__ __forceinline__ uint32_t split_piece(float &r, int code0, int p, int lane, int &my_code)
{
    const int code = max(0, p == 0 ? code0 : code0 + 1 - 3 * p);
    uint32_t nib;
    const float rs = __fmul_rn(r, __int_as_float((254 - code) << 23));   // r / 2^s, exact
    const float q = e2m1_rne(rs, nib);                                  // no -0 codes
    const float sc = code ? __int_as_float(code << 23) : __int_as_float(0x00400000);
    r = __fmul_rn(__fsub_rn(rs, q), sc);
    if (lane == p) my_code = code;
    return nib;
}

// NV vectors per B operand (the grouped layout, NV = 4): slot v's piece p is B row
// m = 16 v + p, at row m of each K block's (16 NV) x 128-byte SWIZZLE_128B image, and its
// scale at byte 16 (m % 32) + 4 (m / 32) + (block % 4) of the block's atom.
template <int NV>
__device__ __forceinline__ void split_block(uint8_t *bq, uint8_t *bs, float r, int blk, int v, int lane)
{
    const int c = blk >> 4, j = blk & 15;
    uint8_t *tile = bq + (size_t)c * (NV * kTileB) + (j >> 3) * (NV * 2048) + v * 2048;
    uint8_t *atom = bs + (size_t)c * kTileSF + (j >> 2) * 512;
    if ((j & 3) == 0 && v == 0) {
        // the zero bytes of this atom (its data bytes are written below by 4 blocks)
        if (NV == 1) {
            if (lane < 16) {
                uint32_t *z = reinterpret_cast<uint32_t *>(atom + 16 * lane + 4);
                z[0] = 0u; z[1] = 0u; z[2] = 0u;
            } else {
                *reinterpret_cast<uint4 *>(atom + 256 + 16 * (lane - 16)) = make_uint4(0, 0, 0, 0);
            }
        } else {
            *reinterpret_cast<uint2 *>(atom + 16 * lane + 8) = make_uint2(0u, 0u);   // words 2, 3
        }
    }
    int my_code = 255;                       // lane p < 16 keeps piece p's scale code
    if (__any_sync(0xffffffffu, !isfinite(r))) {
#pragma unroll 1
        for (int p = 0; p < kN; p++)
            if ((lane & 7) == 0)
                *reinterpret_cast<uint32_t *>(tile + (p >> 3) * 1024 + (p & 7) * 128 + (((j & 7) ^ (p & 7)) << 4) +
                                              (lane >> 1)) = 0u;
    } else {
        const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(r)));
        const int code0 = (int)(mb >> 23) - 2 + ((mb & 0x7fffffu) > 0x400000u ? 1 : 0);
        // the lane's 16 codes first, a chain of plain arithmetic with no warp operation in
        // it (a zero residual gives zero codes from there on, as the schedule wants), kept
        // as nibbles; then the 16 row words, whose shuffles are independent of one another
        uint32_t nlo = 0u, nhi = 0u;
#pragma unroll 4
        for (int p = 0; p < 8; p++) nlo |= split_piece(r, code0, p, lane, my_code) << (4 * p);
#pragma unroll 4
        for (int p = 8; p < kN; p++) nhi |= split_piece(r, code0, p, lane, my_code) << (4 * (p - 8));
#pragma unroll
        for (int p = 0; p < kN; p++) {
            const uint32_t w = piece_word(((p < 8 ? nlo : nhi) >> (4 * (p & 7))) & 15u);
            if ((lane & 7) == 0)
                *reinterpret_cast<uint32_t *>(tile + (p >> 3) * 1024 + (p & 7) * 128 + (((j & 7) ^ (p & 7)) << 4) +
                                              (lane >> 1)) = w;
        }
    }
    if (lane < kN) atom[16 * (16 * (v & 1) + lane) + 4 * (v >> 1) + (j & 3)] = (uint8_t)my_code;
}

// B operands of fp32 vectors: grid (ceil(K/32 / 8), nvec), 256 threads, a warp per block.
__global__ void k_bsplit(uint8_t *bq, uint8_t *bs, const float *x, int K, size_t ld)
{
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x * 8 + warp;
    if (blk >= K / 32) return;
    const int v = blockIdx.y;
    const int nch = K / kStageK;
    const float r = x[(size_t)v * ld + blk * 32 + lane];
    split_block<1>(bq + (size_t)v * nch * kTileB, bs + (size_t)v * nch * kTileSF, r, blk, 0, lane);
}

// silu(gate) * up of one element, gate and up summed over the K slices in slice order from
// the partials at pa[s * slice_stride] (gate) and pa[s * slice_stride + inter] (up). Loads
// go to L2 (the partials may have been written by other CTAs of the same launch) in groups
// of 16 slices, every load of a group issued before the ordered sums.
__device__ __forceinline__ float act_value(const float *pa, int ks, size_t slice_stride, int inter)
{
    float g = 0.0f, u = 0.0f;
    for (int s0 = 0; s0 < ks; s0 += 16) {
        float gv[16], uv[16];
#pragma unroll
        for (int i = 0; i < 16; i++) {
            if (s0 + i < ks) {
                gv[i] = __ldcg(pa + (size_t)(s0 + i) * slice_stride);
                uv[i] = __ldcg(pa + (size_t)(s0 + i) * slice_stride + inter);
            }
        }
#pragma unroll
        for (int i = 0; i < 16; i++) {
            if (s0 + i < ks) {
                g += gv[i];
                u += uv[i];
            }
        }
    }
    return silu_f(g) * u;
}

// B operands of act = silu(gate) * up, gate/up summed over the K slices of the gate/up
// pass in slice order; both indexed by grouped position p. grid (ceil(inter/32 / 8),
// positions). The count and the partials are loaded together (the partial rows of every
// position exist), so the block pays one memory latency.
__global__ void k_bsplit_swiglu(uint8_t *bq, uint8_t *bs, const float *part, int ks,
                                size_t slice_stride, int inter, const int *count, int count_host)
{
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = blockIdx.x * 8 + warp;
    const int p = blockIdx.y;
    if (blk >= inter / 32) return;
    const int n = count ? *count : count_host;
    const float act = act_value(part + (size_t)p * 2 * inter + blk * 32 + lane, ks, slice_stride, inter);
    if (p >= n) return;
    const int nch = inter / kStageK;
    split_block<1>(bq + (size_t)p * nch * kTileB, bs + (size_t)p * nch * kTileSF, act, blk, 0, lane);
}

// ------------------------------------------------------------ fused decode pass
// gate/up, the act split and down in ONE launch, for the decode shapes whose items fit
// one table per CTA (T * topk up to 16 at config 1). Both passes run back to back in every
// CTA's roles, with no kernel boundary between them:
//   warp 0 lane 0   weight producer: the ring streams the CTA's gate/up tiles, then its
//                   down tiles; the down weights do not depend on the gate/up results, so
//                   they fill the ring while the last gate/up stages finish;
//   warp 1 lane 0   B producer of the gate/up runs (x's pieces, one bulk copy per run);
//   warp 4          MMA issuer, as in k_mxfp4_umma;
//   warps 5-8       epilogue. After their gate/up items they publish the CTA's gate/up rows
//                   (one release per act chunk touched), then form the B operand of each
//                   of the CTA's down runs themselves: act = silu(gate) * up over the K
//                   slices (k_bsplit_swiglu's arithmetic) once every CTA's rows of that act
//                   chunk are out, split into the 16 E2M1 pieces straight into the run's
//                   shared-memory B slot; then the down items' epilogue.
// Cross-CTA dependencies go through counters in the workspace (zeroed by the router of the
// same layer, before this launch's programmatic wait returns):
//   cnt[p * nact + c]      gate/up rows of act chunk c of position p published (expected:
//                          4 epilogue warps x 8 tiles x the K slices);
//   cnt[2 * npos * nact]   abort word: a CTA whose wait ran out sets it, every waiter then
//                          gives up at once.
// A CTA only ever waits for gate/up work, which waits on nothing across CTAs, so progress
// needs no more co-residency than the scheduler eventually provides; every wait is bounded
// (k3_wait_cycles). Results are bit-identical to the three-launch form (kind 4).
struct FusedJob {
    Job A, B;          // gate/up and down, both in the resident-B geometry (one stage per item)
    int *cnt;          // counters, 2 * npos * nact + 1 ints
    int npos;          // positions the counters cover (the launch's npos_max)
    int nact;          // act chunks per position: inter / 512
    int arrivals;      // expected gate/up arrivals per (position, act chunk)
};
constexpr int kFusedCtr = 96;            // shared per-(position, act chunk) arrival counts

__device__ __forceinline__ int ld_acquire(const int *p)
{
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(int *p, int v)
{
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// Barrier of the 4 epilogue warps, bounded: a shared arrival count that every warp's lane 0
// bumps and then waits to reach 4 x gen (gen = this barrier's ordinal, counted by each warp
// alike). A hardware named barrier would wait forever for a warp that left on an abort;
// this one returns false on the abort flag or the time limit.
__device__ __forceinline__ bool epi_barrier(int *ctr, int gen, volatile int *abort, int lane)
{
    int ok = 1;
    __syncwarp();
    if (lane == 0) {
        __threadfence_block();
        atomicAdd(ctr, 1);
        const long long t0 = clock64(), lim = k3_wait_cycles;
        while (*(volatile int *)ctr < 4 * gen) {
            __nanosleep(32);
            if (*abort) { ok = 0; break; }
            if (clock64() - t0 > lim) {
                k3_raise(K3D_ETIMEOUT, K3_SITE_MXFP4);
                *abort = 1;
                ok = 0;
                break;
            }
        }
        __threadfence_block();
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

// Bounded wait for *p >= target (acquire); false when it gave up: this CTA's or another
// CTA's abort, or the time limit (which raises K3D_ETIMEOUT and sets both abort words).
__device__ __forceinline__ bool wait_count(const int *p, int target, volatile int *abort, int *gabort)
{
    if (ld_acquire(p) >= target) return true;
    const long long t0 = clock64(), lim = k3_wait_cycles;
    while (ld_acquire(p) < target) {
        if (*abort) return false;
        if (*(volatile int *)gabort) { *abort = 1; return false; }
        if (clock64() - t0 > lim) {
            k3_raise(K3D_ETIMEOUT, K3_SITE_MXFP4);
            *abort = 1;
            atomicExch(gabort, 1);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// Run identity of an item in the fused table: the pass, its B vector and its K chunk.
__device__ __forceinline__ bool fused_new_run(const ItemEnt &it, int pass, int key, int chunk)
{
    return ((pass << 24) | it.vec) != key || it.s != chunk;
}

// split_block<1> for the four blocks j0..j0+3 of one 512-element chunk (one scale atom, j0 a
// multiple of 4) at once: lane l holds element l of each block, and the four blocks' piece
// chains are independent, so they run side by side. Same bytes as four split_block<1> calls.
__device__ __forceinline__ void split_block4(uint8_t *bq, uint8_t *bs, const float r_in[4], int j0, int lane)
{
    uint8_t *atom = bs + (j0 >> 2) * 512;
    if (lane < 16) {
        uint32_t *z = reinterpret_cast<uint32_t *>(atom + 16 * lane + 4);
        z[0] = 0u; z[1] = 0u; z[2] = 0u;
    } else {
        *reinterpret_cast<uint4 *>(atom + 256 + 16 * (lane - 16)) = make_uint4(0, 0, 0, 0);
    }
    float r[4];
    int code0[4], my_code[4];
    bool fin[4];
#pragma unroll
    for (int b = 0; b < 4; b++) {
        r[b] = r_in[b];
        fin[b] = !__any_sync(0xffffffffu, !isfinite(r[b]));
        const uint32_t mb = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(r[b])));
        code0[b] = (int)(mb >> 23) - 2 + ((mb & 0x7fffffu) > 0x400000u ? 1 : 0);
        my_code[b] = 255;
    }
    bool live = true;              // some residual of the four blocks is not yet zero
    // a rolled loop: unrolled, the body is thousands of instructions that every SM fetches
    // once per call through the instruction cache, all at the same time
#pragma unroll 1
    for (int p = 0; p < kN; p++) {
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int j = j0 + b;
            uint32_t nib = 0u;
            int code = 255;
            if (fin[b]) code = max(0, p == 0 ? code0[b] : code0[b] + 1 - 3 * p);
            if (fin[b] && live) {
                const float rs = __fmul_rn(r[b], __int_as_float((254 - code) << 23));
                const float q = e2m1_rne(rs, nib);
                const float sc = code ? __int_as_float(code << 23) : __int_as_float(0x00400000);
                r[b] = __fmul_rn(__fsub_rn(rs, q), sc);
            }
            if (lane == p) my_code[b] = code;
            const uint32_t w = live ? piece_word(nib) : 0u;
            if ((lane & 7) == 0)
                *reinterpret_cast<uint32_t *>(bq + (j >> 3) * 2048 + (p >> 3) * 1024 + (p & 7) * 128 +
                                              (((j & 7) ^ (p & 7)) << 4) + (lane >> 1)) = w;
        }
        // the remaining pieces of a zero residual are zero codes (their scales still follow
        // the schedule)
        live = live && __any_sync(0xffffffffu, (fin[0] && r[0] != 0.0f) || (fin[1] && r[1] != 0.0f) ||
                                                (fin[2] && r[2] != 0.0f) || (fin[3] && r[3] != 0.0f));
    }
    if (lane < kN)
        *reinterpret_cast<uint32_t *>(atom + 16 * lane) = (uint32_t)(my_code[0] & 0xff) |
            ((uint32_t)(my_code[1] & 0xff) << 8) | ((uint32_t)(my_code[2] & 0xff) << 16) |
            ((uint32_t)(my_code[3] & 0xff) << 24);
}

__device__ __forceinline__ void fused_act_split(const FusedJob &F, int p, int c, unsigned char *tile, unsigned char *atoms,
                                            int q, int lane);

// The B operand of one down run (position p, act chunk c) formed by the 4 epilogue warps
// into the shared-memory slot at `slot` (pieces, then the scale atoms): each warp waits for
// the chunk's gate/up rows, then forms 4 of its 16 blocks (act = silu(gate) * up with the K
// slices summed in order, as act_value; the split of split_block). false when a wait gave up.
__device__ __forceinline__ bool fused_make_b(const FusedJob &F, int p, int c, unsigned char *tile,
                                             unsigned char *atoms, int q, int lane, volatile int *abort, int *gabort)
{
    const int *ca = F.cnt + (size_t)p * F.nact + c;
    int okw = 1;
    if (lane == 0) okw = wait_count(ca, F.arrivals, abort, gabort) ? 1 : 0;
    okw = __shfl_sync(0xffffffffu, okw, 0);
    if (!okw) return false;
    (void)ld_acquire(ca);                   // every lane acquires the gate/up stores
    fused_act_split(F, p, c, tile, atoms, q, lane);
    return true;
}

// act of the warp's 4 blocks of act chunk c of position p, split into `slot` (B pieces, then
// the scale atoms).
__device__ __forceinline__ void fused_act_split(const FusedJob &F, int p, int c, unsigned char *tile, unsigned char *atoms,
                                            int q, int lane)
{
    const int inter = F.nact * kStageK, ks = F.A.ks;
    const size_t ss = F.A.slice_stride;
    const float *pa = F.A.part + (size_t)p * 2 * inter + (size_t)(c * 16 + q * 4) * 32 + lane;
    // the four blocks' gate and up partials, all slices of a group of 8 in flight together
    float g[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < ks; s0 += 8) {
        float gv[4][8], uv[4][8];
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int b = 0; b < 4; b++)
                if (s0 + i < ks) {
                    gv[b][i] = __ldcg(pa + (size_t)(s0 + i) * ss + 32 * b);
                    uv[b][i] = __ldcg(pa + (size_t)(s0 + i) * ss + 32 * b + inter);
                }
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int b = 0; b < 4; b++)
                if (s0 + i < ks) {
                    g[b] += gv[b][i];
                    u[b] += uv[b][i];
                }
    }
    float act[4];
#pragma unroll
    for (int b = 0; b < 4; b++) act[b] = silu_f(g[b]) * u[b];
    split_block4(tile, atoms, act, q * 4, lane);
    // a bulk copy brings these bytes into the run's shared-memory slot
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

__global__ void __launch_bounds__(kThreads, 1) k_mxfp4_fused(const __grid_constant__ FusedJob F)
{
    using G = Geo<1, 1>;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = saddr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char *gbase = smem_raw + (base - raw);
    const uint32_t b_full = base, b_empty = base + 64, b_accf = base + 128;
    const uint32_t b_acce = b_accf + 8 * kAccBufs, b_drain = b_acce + 8 * kAccBufs;
    const uint32_t b_bfull = b_drain + 8, b_bempty = b_bfull + 16;
    volatile int *abort = reinterpret_cast<volatile int *>(gbase + 512);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + 520);
    int *s_n = reinterpret_cast<int *>(gbase + 528);            // na, nb, first items
    int *s_ctr = reinterpret_cast<int *>(gbase + 544);          // [kFusedCtr] arrivals
    int *s_epi = reinterpret_cast<int *>(gbase + 544 + 4 * kFusedCtr);   // epilogue barrier
    ItemEnt *items = reinterpret_cast<ItemEnt *>(gbase + kOffItems);
    const uint32_t stage0 = base + kStage0;
    const uint32_t bslots = base + (uint32_t)G::kBSlots;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *gabort = F.cnt + 2 * F.npos * F.nact;
    static_assert(544 + 4 * kFusedCtr + 4 <= kOffItems, "shared header");

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::kNStages; s++) { mbar_init(b_full + 8 * s, 1); mbar_init(b_empty + 8 * s, 1); }
        for (int i = 0; i < kAccBufs; i++) { mbar_init(b_accf + 8 * i, 1); mbar_init(b_acce + 8 * i, 4); }
        mbar_init(b_drain, 1);
        for (int i = 0; i < 2; i++) { mbar_init(b_bfull + 8 * i, 1); mbar_init(b_bempty + 8 * i, 1); }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i <= kFusedCtr; i += blockDim.x) s_ctr[i] = 0;   // and s_epi
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(saddr(tmem_slot)), "r"(G::kTmem) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();                      // the work lists and the counters' zeroing come from the router

    if (threadIdx.x == 0) {
        const int ta = item_count(F.A), tb = item_count(F.B);
        const int a0 = (int)((long long)blockIdx.x * ta / gridDim.x), a1 = (int)((long long)(blockIdx.x + 1) * ta / gridDim.x);
        const int b0 = (int)((long long)blockIdx.x * tb / gridDim.x), b1 = (int)((long long)(blockIdx.x + 1) * tb / gridDim.x);
        s_n[0] = a1 - a0;
        s_n[1] = b1 - b0;
        s_n[2] = a0;
        s_n[3] = b0;
    }
    __syncthreads();
    int na = s_n[0], nb = s_n[1];
    if (na + nb > kMaxItems || F.npos * F.nact > kFusedCtr) {   // the host sizes launches so that
        if (threadIdx.x == 0) k3_raise(K3D_EBOUND, K3_SITE_MXFP4);  // this cannot happen
        na = nb = 0;
    }
    for (int i = threadIdx.x; i < na + nb; i += blockDim.x)
        items[i] = i < na ? decode<1, 1>(F.A, s_n[2] + i) : decode<1, 1>(F.B, s_n[3] + i - na);
    __syncthreads();
    pdl_trigger();
    const int n = na + nb;

    if (warp == 0) {
        // ------------------------------------------------------------ weight producer
        if (lane == 0) {
            int g = 0;
            for (int k = 0; k < n; k++) {
                const ItemEnt &it = items[k];
                const int st = g % G::kNStages;
                if (g >= G::kNStages && !mbar_wait(b_empty + 8 * st, ((g / G::kNStages) - 1) & 1, abort)) break;
                const uint32_t fb = b_full + 8 * st;
                if (item_ok(it)) {
                    mbar_expect_tx(fb, G::kTx);
                    issue_weights<1, 1>(stage0 + (uint32_t)st * G::kBytes, fb, k < na ? F.A : F.B, it, it.s);
                } else {
                    k3_raise(K3D_EINVAL, K3_SITE_MXFP4);
                    mbar_arrive(fb);
                }
                g++;
            }
            // no copy may land after the CTA exits: wait for the last stages issued (each
            // earlier one was consumed before its slot was reused)
            for (int h = max(0, g - G::kNStages); h < g; h++)
                mbar_drain(b_full + 8 * (h % G::kNStages), (h / G::kNStages) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------- B producer, gate/up runs
        if (lane == 0) {
            int rb = 0, key = -1, chunk = -1;
            for (int k = 0; k < na; k++) {
                const ItemEnt &it = items[k];
                if (!fused_new_run(it, 0, key, chunk)) continue;
                const int slot = rb & 1;
                if (rb >= 2 && !mbar_wait(b_bempty + 8 * slot, ((rb >> 1) - 1) & 1, abort)) break;
                const uint32_t bb = b_bfull + 8 * slot, dst = bslots + (uint32_t)(slot * G::kBSlot);
                const size_t vix = (size_t)it.vec * F.A.nch + it.s;
                mbar_expect_tx(bb, G::kBTile + kTileSF);
                bulk_g2s(dst, F.A.bq + vix * G::kBTile, G::kBTile, bb);
                bulk_g2s(dst + G::kBTile, F.A.bs + vix * kTileSF, kTileSF, bb);
                rb++;
                key = it.vec;
                chunk = it.s;
            }
            for (int h = max(0, rb - 2); h < rb; h++) mbar_drain(b_bfull + 8 * (h & 1), (h >> 1) & 1);
        }
    } else if (warp == 4) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int g = 0, rb = 0, key = -1, chunk = -1;
            for (int k = 0; k < n; k++) {
                const ItemEnt &it = items[k];
                const int pass = k < na ? 0 : 1;
                const int buf = k % kAccBufs;
                if (k >= kAccBufs && !mbar_wait(b_acce + 8 * buf, ((k / kAccBufs) - 1) & 1, abort)) break;
                tc_fence_after();
                if (fused_new_run(it, pass, key, chunk)) {
                    if (rb > 0) tc_commit(b_bempty + 8 * ((rb - 1) & 1));
                    const int slot = rb & 1;
                    if (!mbar_wait(b_bfull + 8 * slot, (rb >> 1) & 1, abort)) break;
                    tc_fence_after();
                    const uint32_t sfb = tmem + G::kSfbCol + (uint32_t)(slot * 16);
#pragma unroll
                    for (int a4 = 0; a4 < 4; a4++)
                        tc_cp_sf(sfb + 4 * a4, desc_sf(bslots + (uint32_t)(slot * G::kBSlot + G::kBTile + 512 * a4)));
                    rb++;
                    key = (pass << 24) | it.vec;
                    chunk = it.s;
                }
                const int slot = (rb - 1) & 1;
                const uint32_t bs = bslots + (uint32_t)(slot * G::kBSlot);
                const uint32_t sfb = tmem + G::kSfbCol + (uint32_t)(slot * 16);
                const uint32_t dcol = tmem + (uint32_t)(buf * G::kCols);
                const int st = g % G::kNStages;
                if (!mbar_wait(b_full + 8 * st, (g / G::kNStages) & 1, abort)) break;
                tc_fence_after();
                const uint32_t sb = stage0 + (uint32_t)st * G::kBytes;
                const uint32_t sfa = tmem + G::kSfaCol + (uint32_t)((g & 1) * 16);
#pragma unroll
                for (int a4 = 0; a4 < 4; a4++) tc_cp_sf(sfa + 4 * a4, desc_sf(sb + G::kSFA + 512 * a4));
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const uint32_t kb = (uint32_t)(j >> 2), off = (uint32_t)((j & 3) * 32);
                    const uint64_t ad = desc_sw128(sb + kb * 16384u + off);
                    const uint64_t bd = desc_sw128(bs + kb * 2048u + off);
                    const uint32_t id = (uint32_t)((j & 1) * 2);
                    const uint32_t atom = (uint32_t)(4 * (j >> 1));
                    tc_mma(dcol, ad, bd, idesc_mxf4<G::kCols>(id), j > 0 ? 1u : 0u, (sfa + atom) | (id << 30),
                           (sfb + atom) | (id << 30));
                }
                tc_commit(b_empty + 8 * st);
                g++;
                tc_commit(b_accf + 8 * buf);
            }
        }
        __syncwarp();
    } else if (warp >= 5) {
        // ---------------------------------------------------------------- epilogue
        // a warp reads the tensor-memory lanes of its own quadrant (warp % 4)
        const int q = warp & 3, m = q * 32 + lane;
        bool ok = true;
        // gate/up runs: the global index of the first down run continues from them
        int ra = 0;
        {
            int key = -1, chunk = -1;
            for (int k = 0; k < na; k++)
                if (fused_new_run(items[k], 0, key, chunk)) { ra++; key = items[k].vec; chunk = items[k].s; }
        }
        int rb = ra, key = -1, chunk = -1, gen = 0;   // down runs begun; epilogue barriers
        int built = ra;                                // down runs whose B operand is formed
        for (int k = 0; k <= n && ok; k++) {
            if (k == na) {
                // every gate/up row of this CTA is stored: publish them, one release per act
                // chunk this CTA touched (each thread's stores are made visible by its fence
                // before the epilogue barrier, and the releases come after it)
                __threadfence();
                if (!epi_barrier(s_epi, ++gen, abort, lane)) { ok = false; break; }
                for (int i = m; i < F.npos * F.nact; i += 128)
                    if (s_ctr[i]) red_release_add(F.cnt + i, s_ctr[i]);
            }
            if (k == n) break;
            const ItemEnt &it = items[k];
            const bool up = k < na;
            if (!up && fused_new_run(it, 1, key, chunk)) {
                // the B operands of the down runs are formed in their slots one run ahead: the
                // first run's here, then the next run's while the MMA works on this one (its
                // slot is free once the MMA has begun this run)
                bool fail_ = false;
                for (int r = rb, kk = k; r < rb + 2 && !fail_; r++) {
                    if (r < built) continue;
                    // the first item of run r (kk for r == rb; the next key change after it)
                    if (r > rb) {
                        int k2 = kk + 1;
                        while (k2 < n && !fused_new_run(items[k2], 1, (1 << 24) | items[kk].vec, items[kk].s)) k2++;
                        if (k2 >= n) break;
                        kk = k2;
                    }
                    const ItemEnt &ir = items[kk];
                    const int slot = r & 1;
                    if (r >= 2) {
                        int okw = 1;
                        if (lane == 0) okw = mbar_wait(b_bempty + 8 * slot, ((r >> 1) - 1) & 1, abort) ? 1 : 0;
                        if (!__shfl_sync(0xffffffffu, okw, 0)) { fail_ = true; break; }
                    }
                    // formed in global memory (the down pass's B operand at this position and
                    // chunk; every CTA with this run writes the same bytes), then one bulk copy
                    // into the slot
                    const size_t vix = (size_t)ir.vec * F.B.nch + ir.s;
                    unsigned char *gq = const_cast<unsigned char *>(F.B.bq) + vix * kTileB;
                    unsigned char *gs = const_cast<unsigned char *>(F.B.bs) + vix * kTileSF;
                    if (!fused_make_b(F, ir.vec, ir.s, gq, gs, q, lane, abort, gabort) ||
                        !epi_barrier(s_epi, ++gen, abort, lane)) {
                        fail_ = true;
                        break;
                    }
                    if (m == 0) {
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        const uint32_t bb = b_bfull + 8 * slot, dst = bslots + (uint32_t)(slot * G::kBSlot);
                        mbar_expect_tx(bb, G::kBTile + kTileSF);
                        bulk_g2s(dst, gq, G::kBTile, bb);
                        bulk_g2s(dst + G::kBTile, gs, kTileSF, bb);
                    }
                    built = r + 1;
                }
                if (fail_) { ok = false; break; }
                rb++;
                key = (1 << 24) | it.vec;
                chunk = it.s;
            }
            const Job &J = up ? F.A : F.B;
            const int row = up ? (m < 64 ? it.tile * 64 + m : (J.out_w >> 1) + it.tile * 64 + (m - 64))
                               : it.tile * 128 + m;
            float *dst = J.part + (size_t)it.s * J.slice_stride + (size_t)it.out * J.out_w + row;
            const int buf = k % kAccBufs;
            int okw = 1;
            if (!mbar_wait(b_accf + 8 * buf, (k / kAccBufs) & 1, abort)) okw = 0;
            if (!__all_sync(0xffffffffu, okw)) { ok = false; break; }
            tc_fence_after();
            float v[kN];
            tc_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * G::kCols), v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(b_acce + 8 * buf);
            float sum = v[15];
#pragma unroll
            for (int i = 14; i >= 0; i--) sum += v[i];
            *dst = sum;
            if (up && lane == 0) atomicAdd(&s_ctr[it.out * F.nact + it.tile / 8], 1);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && *abort) atomicExch(gabort, 1);   // other CTAs' waiters give up
    if (warp == 4 && lane == 0) {
        tc_commit(b_drain);
        mbar_drain(b_drain, 0);
    }
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem), "r"(G::kTmem) : "memory");
    }
}

// ------------------------------------------------------------- grouped items (T > 8)
// Groups of up to four consecutive grouped positions of one expert: g_p0, g_n, g_e per
// group (experts in grouping order), ng[0] their count; pos_of[a] = the position of
// assignment a (the grouped passes write partials by position). One CTA, 1024 threads.
__global__ void __launch_bounds__(1024) k_make_groups(const int *n_active, const int *act_expert,
                                                      const int *act_off, const int *assign, int *ng,
                                                      int *g_p0, int *g_n, int *g_e, int *pos_of)
{
    pdl_wait();
    pdl_trigger();
    __shared__ int wsum[32];
    const int nu = __ldcg(n_active), npos = __ldcg(n_active + 1);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per = (nu + 1023) / 1024;
    const int u0 = min(nu, (int)threadIdx.x * per), u1 = min(nu, u0 + per);
    int local = 0;
    for (int u = u0; u < u1; u++) local += (__ldcg(act_off + u + 1) - __ldcg(act_off + u) + 3) >> 2;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = wsum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        wsum[lane] = w;
    }
    __syncthreads();
    int g = incl - local + (warp > 0 ? wsum[warp - 1] : 0);
    for (int u = u0; u < u1; u++) {
        const int base = __ldcg(act_off + u), cnt = __ldcg(act_off + u + 1) - base, e = __ldcg(act_expert + u);
        for (int i = 0; i < cnt; i += 4, g++) {
            g_p0[g] = base + i;
            g_n[g] = min(4, cnt - i);
            g_e[g] = e;
        }
    }
    if (threadIdx.x == 1023) ng[0] = g;
    for (int p = threadIdx.x; p < npos; p += 1024) pos_of[__ldcg(assign + p)] = p;
}

// B operand of the grouped gate/up pass: slot v of group g holds the token of position
// g_p0[g] + v (assignment a = assign[p], token a / K); empty slots split 0 (zero codes and
// scales). grid (ceil(hidden / 32 / 8), groups at most), 256 threads, a warp per block.
__global__ void k_bsplit_group_x(uint8_t *bq, uint8_t *bs, const float *x, int hidden, const int *assign,
                                 int K, const int *ng, const int *g_p0, const int *g_n)
{
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = blockIdx.y, blk = blockIdx.x * 8 + warp;
    if (g >= __ldcg(ng) || blk >= hidden / 32) return;
    const int p0 = __ldcg(g_p0 + g), n = __ldcg(g_n + g);
    int tok[4];
#pragma unroll
    for (int v = 0; v < 4; v++) tok[v] = v < n ? __ldcg(assign + p0 + v) / K : 0;
    float r[4];
#pragma unroll
    for (int v = 0; v < 4; v++) r[v] = v < n ? __ldcg(x + (size_t)tok[v] * hidden + blk * 32 + lane) : 0.0f;
    const int nch = hidden / kStageK;
#pragma unroll
    for (int v = 0; v < 4; v++)
        split_block<4>(bq + (size_t)g * nch * (4 * kTileB), bs + (size_t)g * nch * kTileSF, r[v], blk, v, lane);
}

// B operand of the grouped down pass: silu(gate) * up of positions g_p0[g] + v, as
// k_bsplit_swiglu computes it; empty slots split 0.
__global__ void k_bsplit_swiglu_group(uint8_t *bq, uint8_t *bs, const float *part, int ks, size_t slice_stride,
                                      int inter, const int *ng, const int *g_p0, const int *g_n)
{
    pdl_wait();
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = blockIdx.y, blk = blockIdx.x * 8 + warp;
    if (g >= __ldcg(ng) || blk >= inter / 32) return;
    const int p0 = __ldcg(g_p0 + g), n = __ldcg(g_n + g);
    const int nch = inter / kStageK;
#pragma unroll
    for (int v = 0; v < 4; v++) {
        const float act = v < n ? act_value(part + (size_t)(p0 + v) * 2 * inter + blk * 32 + lane, ks,
                                            slice_stride, inter)
                                : 0.0f;
        split_block<4>(bq + (size_t)g * nch * (4 * kTileB), bs + (size_t)g * nch * kTileSF, act, blk, v, lane);
    }
}

// ------------------------------------------------------------- weight tiling
// Rewrites MXFP4 weights from the checkpoint layout into the stage-ordered tiled layout:
// for 128-row tile t and 512-element chunk c, a 32 KB block at codes + 32768 (c * ntiles + t)
// holding the tile's codes exactly as the kernel's shared-memory stage (SWIZZLE_128B
// K-major), and a 2 KB block at sf + 2048 (c * ntiles + t) holding its scales as the four
// tcgen05.cp atoms, with E8M0 255 replaced by 0. Blocks are chunk-major: the kernel walks
// its items (vector, chunk, tile) with the tile fastest, so the weight stream of a CTA is
// one contiguous region of memory, as a GEMV's row stream is. Gate/up tiles interleave 64
// gate rows and the same 64 up rows (c1/s1 given); down tiles are 128 rows of one matrix
// (c1 null). grid (ntiles * nch), 256 threads.
__global__ void k_pretile(uint8_t *dc, uint8_t *ds, const uint8_t *c0, const uint8_t *s0,
                          const uint8_t *c1, const uint8_t *s1, int K)
{
    const int nch = K / kStageK;
    const int ntiles = gridDim.x / nch;
    const int c = blockIdx.x / ntiles, t = blockIdx.x % ntiles;
    const int rowbytes = K >> 1, sfrow = K >> 5;
    const bool gu = c1 != nullptr;
    uint8_t *dtile = dc + (size_t)blockIdx.x * kTileA;
    for (int q = threadIdx.x; q < 2048; q += blockDim.x) {
        const int r = q >> 4, j = q & 15;
        const uint8_t *row = gu ? (r < 64 ? c0 + (size_t)(t * 64 + r) * rowbytes
                                          : c1 + (size_t)(t * 64 + r - 64) * rowbytes)
                                : c0 + (size_t)(t * 128 + r) * rowbytes;
        const uint4 v = *reinterpret_cast<const uint4 *>(row + (size_t)c * kRowBytes + 16 * j);
        *reinterpret_cast<uint4 *>(dtile + (j >> 3) * 16384 + (r >> 3) * 1024 + (r & 7) * 128 +
                                   (((j & 7) ^ (r & 7)) << 4)) = v;
    }
    if (threadIdx.x < 128) {
        const int r = threadIdx.x;
        const uint8_t *srow = gu ? (r < 64 ? s0 + (size_t)(t * 64 + r) * sfrow
                                           : s1 + (size_t)(t * 64 + r - 64) * sfrow)
                                 : s0 + (size_t)(t * 128 + r) * sfrow;
        const uint4 v = *reinterpret_cast<const uint4 *>(srow + (size_t)c * 16);
        uint32_t *atom = reinterpret_cast<uint32_t *>(ds + (size_t)blockIdx.x * kTileSF +
                                                      16 * (r & 31) + 4 * (r >> 5));
        atom[0] = clean_e8m0(v.x);
        atom[128] = clean_e8m0(v.y);
        atom[256] = clean_e8m0(v.z);
        atom[384] = clean_e8m0(v.w);
    }
}

// y[r] = sum over K slices of part[s][r] (single-expert mode)
__global__ void k_slice_sum(float *y, const float *part, int ks, size_t slice_stride, int n)
{
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    float acc = 0.0f;
    for (int s0 = 0; s0 < ks; s0 += 16) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (s0 + i < ks) v[i] = part[(size_t)(s0 + i) * slice_stride + r];
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (s0 + i < ks) acc += v[i];
    }
    y[r] = acc;
}

}  // namespace umma

using namespace umma;

bool umma_supported(int K, int rows, int mode)
{
    if (K % kStageK != 0 || K < kStageK || K > 16384) return false;
    return mode == GATEUP ? (rows % 64 == 0) : (rows % 128 == 0);
}

// K slices for `units` assignments: the divisor of the stage count that minimises the
// estimated time (rounds of items over the SMs x bytes per item, plus a fixed per-item
// cost for the accumulator hand-off and the partial-sum write and read).
int umma_slices(int units, int K, int rows, int mode)
{
    const int chunks = K / kStageK;
    const int ntiles = mode == GATEUP ? rows / 64 : rows / 128;
    const int G = sm_count();
    int best = 1;
    double best_cost = 1e30;
    for (int d = 1; d <= chunks; d++) {
        if (chunks % d) continue;
        const long long items = (long long)units * ntiles * d;
        const long long rounds = (items + G - 1) / G;
        const double item_bytes = 128.0 * (K / d) * 0.53125 + 2048.0;
        const double cost = (double)rounds * item_bytes;
        if (cost < best_cost * 0.999) { best_cost = cost; best = d; }
    }
    return best;
}

size_t umma_bq_bytes(int K) { return (size_t)(K / kStageK) * kTileB; }
size_t umma_bs_bytes(int K) { return (size_t)(K / kStageK) * kTileSF; }

int umma_bsplit(uint8_t *bq, uint8_t *bs, const float *x, int K, int nvec, size_t ld,
                cudaStream_t st)
{
    if (nvec <= 0) return K3D_OK;
    dim3 grid((K / 32 + 7) / 8, nvec);
    launch_pdl(k_bsplit, dim3(grid), dim3(256), 0, st, bq, bs, x, K, ld);
    note_launch();
    return check_launch("umma bsplit");
}

int umma_bsplit_swiglu(uint8_t *bq, uint8_t *bs, const float *part, int ks, size_t slice_stride,
                       int inter, const int *count, int npos, cudaStream_t st)
{
    if (npos <= 0) return K3D_OK;
    dim3 grid((inter / 32 + 7) / 8, npos);
    launch_pdl(k_bsplit_swiglu, dim3(grid), dim3(256), 0, st, bq, bs, part, ks, slice_stride, inter, count, npos);
    note_launch();
    return check_launch("umma bsplit swiglu");
}

int umma_slice_sum(float *y, const float *part, int ks, size_t slice_stride, int n, cudaStream_t st)
{
    launch_pdl(k_slice_sum, dim3((n + 255) / 256), dim3(256), 0, st, y, part, ks, slice_stride, n);
    note_launch();
    return check_launch("umma slice sum");
}

// The work description of one pass over `npos_max` assignment positions (the device count,
// when given, may be smaller). MoE mode: w.table/assign/idx; single mode: w.single_mode
// with positions 0..n-1.
static int make_job(Job &J, int mode, int tiled, const MoeWork &w, const int *idx, const int *count,
                    int npos_max, int K, int rows, int ks, const uint8_t *bq, const uint8_t *bs,
                    int vec_div, float *part, int out_w, size_t slice_stride, int early)
{
    if (!umma_supported(K, rows, mode)) return fail(K3D_EINVAL, "umma: unsupported K=%d rows=%d", K, rows);
    const int chunks = K / kStageK;
    if (ks < 1 || chunks % ks) return fail(K3D_EINVAL, "umma: %d slices of %d stages", ks, chunks);
    J.table = w.table;
    J.single = w.single;
    J.single_mode = w.single_mode;
    J.assign = w.assign;
    J.idx = idx;
    J.count = count;
    J.count_host = npos_max;
    J.mode = mode;
    J.K = K;
    J.ntiles = mode == GATEUP ? rows / 64 : rows / 128;
    J.ks = ks;
    J.cps = chunks / ks;
    J.nch = chunks;
    J.tiled = tiled;
    J.bq = bq;
    J.bs = bs;
    J.vec_div = vec_div;
    // gate/up partials and the act pieces built from them are indexed by grouped position
    // (no assignment lookup between the two passes); down partials by assignment, for the
    // combine
    J.out_pos = mode == GATEUP;
    J.vec_pos = mode == DOWN;
    J.early = early;
    J.n_experts = w.n_experts;
    J.part = part;
    J.out_w = out_w;
    J.slice_stride = slice_stride;
    J.g_p0 = J.g_n = J.g_e = nullptr;
    return K3D_OK;
}

template <int NV, int RES>
static int launch_job(const Job &J, long long items, cudaStream_t st)
{
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) {
        cudaError_t e = cudaFuncSetAttribute(k_mxfp4_umma<NV, RES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)Geo<NV, RES>::kSmem);
        if (e != cudaSuccess) return fail(K3D_ECUDA, "umma smem attribute: %s", cudaGetErrorString(e));
        init |= dev_bit();
    }
    if (items <= 0) return K3D_OK;
    const int grid = (int)(items < sm_count() ? items : sm_count());
    launch_pdl(k_mxfp4_umma<NV, RES>, dim3(grid), dim3(kThreads), Geo<NV, RES>::kSmem, st, J);
    note_launch();
    return check_launch("mxfp4 umma");
}

int umma_launch(int mode, int tiled, const MoeWork &w, const int *idx, const int *count,
                int npos_max, int K, int rows, int ks, const uint8_t *bq, const uint8_t *bs,
                int vec_div, float *part, int out_w, size_t slice_stride, cudaStream_t st,
                int early, int resident)
{
    Job J;
    K3_TRY(make_job(J, mode, tiled, w, idx, count, npos_max, K, rows, ks, bq, bs, vec_div, part, out_w,
                    slice_stride, early));
    if (resident) {
        // one stage per item: the (vector, chunk, tile) order needs one K chunk per slice
        if (!tiled || J.cps != 1) return fail(K3D_EINVAL, "umma: resident B needs tiled experts, ks = K / 512");
        return launch_job<1, 1>(J, (long long)npos_max * J.ntiles * ks, st);
    }
    return launch_job<1, 0>(J, (long long)npos_max * J.ntiles * ks, st);
}

// Items per CTA of the two passes of the fused launch for npos positions (the table
// bound), and whether the shapes take it: tiled experts, the resident-B geometry.
int umma_fused_items(int npos, int hidden, int inter)
{
    if (!umma_supported(hidden, inter, GATEUP) || !umma_supported(inter, hidden, DOWN)) return 1 << 30;
    const long long a = (long long)npos * (inter / 64) * (hidden / kStageK);
    const long long b = (long long)npos * (hidden / 128) * (inter / kStageK);
    const long long g = sm_count();
    return (int)((a + g - 1) / g + (b + g - 1) / g);
}

size_t umma_fused_cnt_ints(int npos, int inter) { return (size_t)2 * npos * (inter / kStageK) + 1; }

int umma_fused_ok(int npos, int hidden, int inter)
{
    return umma_fused_items(npos, hidden, inter) <= kMaxItems && npos * (inter / kStageK) <= kFusedCtr;
}

// gate/up, act split and down in one launch (k_mxfp4_fused). cnt: umma_fused_cnt_ints
// ints, zero on entry (the router's grouping zeroes them). Partials and B operands as the
// three-launch path: part_gu [hidden/512][npos][2 inter] by position, act pieces by
// position, part_d [inter/512][npos][hidden] by assignment.
int umma_launch_fused(const MoeWork &w, const int *idx, const int *count, int npos_max, int hidden, int inter,
                      const uint8_t *bq_x, const uint8_t *bs_x, int vec_div, float *part_gu, size_t sl_gu,
                      uint8_t *bq_a, uint8_t *bs_a, float *part_d, size_t sl_d, int *cnt, cudaStream_t st)
{
    if (!umma_fused_ok(npos_max, hidden, inter)) return fail(K3D_EINVAL, "umma fused: %d positions", npos_max);
    FusedJob F;
    K3_TRY(make_job(F.A, GATEUP, 1, w, idx, count, npos_max, hidden, inter, hidden / kStageK, bq_x, bs_x, vec_div,
                    part_gu, 2 * inter, sl_gu, 0));
    K3_TRY(make_job(F.B, DOWN, 1, w, idx, count, npos_max, inter, hidden, inter / kStageK, bq_a, bs_a, 1, part_d,
                    hidden, sl_d, 1));
    F.cnt = cnt;
    F.npos = npos_max;
    F.nact = inter / kStageK;
    F.arrivals = 4 * (kStageK / 64) * F.A.ks;      // 4 epilogue warps x 8 tiles x K slices
    static unsigned long long init = 0;   // one bit per device
    if (!(init & dev_bit())) {
        cudaError_t e = cudaFuncSetAttribute(k_mxfp4_fused, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)Geo<1, 1>::kSmem);
        if (e != cudaSuccess) return fail(K3D_ECUDA, "umma fused smem attribute: %s", cudaGetErrorString(e));
        init |= dev_bit();
    }
    if (npos_max <= 0) return K3D_OK;
    launch_pdl(k_mxfp4_fused, dim3(sm_count()), dim3(kThreads), Geo<1, 1>::kSmem, st, F);
    note_launch();
    return check_launch("mxfp4 umma fused");
}

// The grouped pass: items over the groups of G (ng = their device count, at most
// max_groups), four vectors per item, partials by position; tiled experts only.
int umma_launch_grouped(int mode, const MoeWork &w, const UmmaGroups &G, int max_groups, int K, int rows,
                        int ks, const uint8_t *bq, const uint8_t *bs, float *part, int out_w,
                        size_t slice_stride, cudaStream_t st)
{
    Job J;
    K3_TRY(make_job(J, mode, 1, w, nullptr, G.ng, max_groups, K, rows, ks, bq, bs, 1, part, out_w,
                    slice_stride, 0));
    J.out_pos = 1;
    J.g_p0 = G.p0;
    J.g_n = G.n;
    J.g_e = G.e;
    // one stage per item: resident B when every slice is one K chunk
    if (J.cps == 1) return launch_job<4, 1>(J, (long long)max_groups * J.ntiles * ks, st);
    return launch_job<4, 0>(J, (long long)max_groups * J.ntiles * ks, st);
}

size_t umma_bq_group_bytes(int K) { return (size_t)(K / kStageK) * 4 * kTileB; }

int umma_make_groups(const MoeWork &w, const UmmaGroups &G, cudaStream_t st)
{
    launch_pdl(k_make_groups, dim3(1), dim3(1024), 0, st, (const int *)w.n_active, (const int *)w.act_expert,
               (const int *)w.act_off, (const int *)w.assign, G.ng, G.p0, G.n, G.e, G.pos_of);
    note_launch();
    return check_launch("umma groups");
}

int umma_bsplit_group_x(uint8_t *bq, uint8_t *bs, const float *x, int hidden, const int *assign, int K,
                        const UmmaGroups &G, int max_groups, cudaStream_t st)
{
    dim3 grid((hidden / 32 + 7) / 8, max_groups);
    launch_pdl(k_bsplit_group_x, dim3(grid), dim3(256), 0, st, bq, bs, x, hidden, assign, K, (const int *)G.ng,
               (const int *)G.p0, (const int *)G.n);
    note_launch();
    return check_launch("umma bsplit group");
}

int umma_bsplit_swiglu_group(uint8_t *bq, uint8_t *bs, const float *part, int ks, size_t slice_stride, int inter,
                             const UmmaGroups &G, int max_groups, cudaStream_t st)
{
    dim3 grid((inter / 32 + 7) / 8, max_groups);
    launch_pdl(k_bsplit_swiglu_group, dim3(grid), dim3(256), 0, st, bq, bs, part, ks, slice_stride, inter,
               (const int *)G.ng, (const int *)G.p0, (const int *)G.n);
    note_launch();
    return check_launch("umma bsplit swiglu group");
}

}  // namespace k3

using namespace k3;

extern "C" {

int k3d_expert_pretile(const K3ExpertQ *dst, const K3ExpertQ *src, int hidden, int inter)
{
    K3_TRY(ensure_ctx());
    if (!dst || !src) return fail(K3D_EINVAL, "k3d_expert_pretile null pointer");
    if (!umma_supported(hidden, inter, GATEUP) || !umma_supported(inter, hidden, DOWN))
        return fail(K3D_EINVAL, "k3d_expert_pretile: hidden=%d and inter=%d must be multiples of 512",
                    hidden, inter);
    const uintptr_t al = (uintptr_t)dst->p1 | (uintptr_t)dst->s1 | (uintptr_t)dst->p2 |
                         (uintptr_t)dst->s2 | (uintptr_t)src->p1 | (uintptr_t)src->s1 |
                         (uintptr_t)src->p3 | (uintptr_t)src->s3 | (uintptr_t)src->p2 |
                         (uintptr_t)src->s2;
    if (al & 15u) return fail(K3D_EINVAL, "k3d_expert_pretile pointers must be 16-byte aligned");
    cudaStream_t st = stream();
    k_pretile<<<(inter / 64) * (hidden / kStageK), 256, 0, st>>>(
        (uint8_t *)dst->p1, (uint8_t *)dst->s1, src->p1, src->s1, src->p3, src->s3, hidden);
    k_pretile<<<(hidden / 128) * (inter / kStageK), 256, 0, st>>>(
        (uint8_t *)dst->p2, (uint8_t *)dst->s2, src->p2, src->s2, nullptr, nullptr, inter);
    note_launch(2);
    return check_launch("expert pretile");
}

}  // extern "C"
