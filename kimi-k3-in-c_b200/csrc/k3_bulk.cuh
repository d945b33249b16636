// k3_bulk.cuh -- mbarrier and bulk-copy (cp.async.bulk, no multicast) helpers for the
// streaming kernels, with bounded waits: a wait that runs past its limit stores
// K3D_ETIMEOUT in the device error flag and reports failure instead of spinning on.
#pragma once
#include "k3_common.cuh"

namespace k3 {
namespace bulk {

constexpr long long kSpinLimit = 4000000000LL;   // ~2 s at 1.9 GHz

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

__device__ __forceinline__ void mbar_expect_tx(uint32_t b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(b), "r"(bytes) : "memory");
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

// Bounded wait; false when it gave up (time limit, or another role already aborted). On
// a time-out the error records (who, where, which CTA) for the report.
__device__ __forceinline__ bool mbar_wait(uint32_t b, uint32_t parity, volatile int *abort, int site,
                                          int who = 0, int where = 0)
{
    if (mbar_try(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(b, parity)) {
        if (*abort) return false;
        if (clock64() - t0 > kSpinLimit) {
            k3_raise_at(K3D_ETIMEOUT, site, who, where, (int)blockIdx.x);
            *abort = 1;
            return false;
        }
    }
    return true;
}

// 1-D bulk copy global -> shared (no multicast), completing on an mbarrier; both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

}  // namespace bulk
}  // namespace k3
