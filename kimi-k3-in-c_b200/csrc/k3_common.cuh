// k3_common.cuh -- shared plumbing for the libk3cuda kernels: status, launch
// accounting, device error flag, bf16/E2M1 helpers and warp reductions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include <mutex>

#include "k3.h"
#include "k3_cuda.h"

// ------------------------------------------------------------------ host side ----
namespace k3 {

// Records `code` (first one wins) with a message; returns code.
int fail(int code, const char *fmt, ...);
// Ensures the context exists on the current device; returns K3D_OK or an error.
int ensure_ctx();
// Guards the context's one-time set-up (k3d_init and the per-device look-ups).
extern std::recursive_mutex g_mu;
cudaStream_t stream();
cudaStream_t side_stream();          // null if it could not be created
cudaEvent_t side_event(int i);       // fork/join events of the side stream (i = 0..3)
bool profiling();                    // section timers on (k3d_prof_enable)
int sm_count();
// Host-side launch accounting: every kernel launch of this library goes through
// note_launch() so that tests and the bench can count them.
void note_launch(int n = 1);
// Checks cudaGetLastError() after a launch; records K3D_ECUDA on failure.
int check_launch(const char *what);
// Reads the device error flag (call after a synchronisation): K3D_OK, or K3D_EDEVICE
// recorded with the kernel's site and location details.
int device_flag_status();

// Raises a kernel's dynamic shared memory limit to the device's opt-in maximum minus
// the kernel's static shared memory (cudaFuncSetAttribute rejects anything above that).
void allow_dyn_smem(const void *func);
template <typename F> inline void allow_smem_max(F *f) { allow_dyn_smem((const void *)f); }

// The current device's bit in a one-time set-up mask: a kernel attribute such as its
// dynamic shared memory limit is set per device, so launchers keep one bit per device
// (`static unsigned long long init`; device ids below 64) instead of one flag per process.
inline unsigned long long dev_bit()
{
    int d = 0;
    cudaGetDevice(&d);
    return 1ull << (d & 63);
}

// Programmatic dependent launch: kernels of the decode path are launched with
// launch_pdl, so that a kernel's launch and prologue overlap the end of the kernel before
// it in the stream. Such a kernel must execute pdl_wait() before its first access to
// memory that earlier work in the stream writes or reads (after which everything earlier
// in the stream has completed and is visible), and calls pdl_trigger() to let the next
// kernel launch. Off when the environment sets K3_PDL=0.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// launch_pdl with thread-block clusters of cluster_x CTAs along x (gridDim.x a multiple).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t st, int cluster_x, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cluster_x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Section timers (k3d_prof_*): begin/end record events on the library stream when
// profiling is on and no capture is in progress.
void prof_begin(const char *section);
void prof_end(const char *section);

// Growable device workspace owned by the context (used by the k3.h entry points,
// which have no workspace argument of their own). Slots 0-5: 0 normalised inputs, 1 and 4
// the tensor-core GEMM on the library and the side stream, 2 and 3 other callers.
void *scratch(size_t bytes, int slot = 0);

// Argument staging for the k3.h entry points (see the POINTERS note in k3.h).
struct Stage {
    struct Out { void *host; void *dev; size_t bytes; };
    Out outs[16];
    int n_out = 0;
    bool any_host = false;
    int err = 0;
    // Stages nest (an operator may stage per-call expert bytes while its caller's
    // arguments are staged): each takes arena space above the enclosing one and gives it
    // back when it goes out of scope.
    size_t base = 0;
    Stage();
    ~Stage();
    // device pointer usable by kernels for a read-only model tensor
    const void *weight(const void *p, size_t bytes);
    // input activations / state read by the call
    const void *in(const void *p, size_t bytes);
    // outputs written by the call
    void *out(void *p, size_t bytes);
    // state read and written by the call
    void *inout(void *p, size_t bytes);
    // issue host copies for staged outputs and wait if any host memory was involved
    int finish();
private:
    void *arena(size_t bytes);
};

bool is_device_ptr(const void *p);

}  // namespace k3

#define K3_TRY(x) do { int _e = (x); if (_e) return _e; } while (0)

// ---------------------------------------------------------------- device side ----
// Device error flag: first (code, site) pair wins. Read back by k3d_sync().
extern __device__ int k3_dev_err[2];
// Where the first error happened, when its kernel says (three integers and a valid flag).
extern __device__ int k3_dev_diag[4];
// Limit of the bounded waits on mbarriers and cross-CTA counters, in SM clock cycles
// (k3d_set_wait_limit; default 4e9, about 2 s at 1.9 GHz). A wait that runs out records
// K3D_ETIMEOUT and its kernel drains what it started and returns.
extern __device__ long long k3_wait_cycles;

__device__ __forceinline__ void k3_raise(int code, int site)
{
    if (atomicCAS(&k3_dev_err[0], 0, code) == 0) k3_dev_err[1] = site;
}

__device__ __forceinline__ void k3_raise_at(int code, int site, int a, int b, int c)
{
    if (atomicCAS(&k3_dev_err[0], 0, code) == 0) {
        k3_dev_err[1] = site;
        k3_dev_diag[0] = a;
        k3_dev_diag[1] = b;
        k3_dev_diag[2] = c;
        k3_dev_diag[3] = 1;
    }
}

// Waits until every earlier kernel of the stream has completed and its memory operations
// are visible (a no-op for a kernel launched without the PDL attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the stream launch (its CTAs then wait in their own pdl_wait).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float bf16_to_f32(uint16_t h)
{
    return __uint_as_float((uint32_t)h << 16);
}

// Round-to-nearest-even fp32 -> bf16 bits (NaN kept quiet).
__host__ __device__ __forceinline__ uint16_t f32_to_bf16_bits(float f)
{
#ifdef __CUDA_ARCH__
    uint32_t u = __float_as_uint(f);
#else
    union { float f; uint32_t u; } c; c.f = f; uint32_t u = c.u;
#endif
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// E8M0 byte -> its power of two as fp32; 255 (NaN by the OCP spec) -> 0.
// 2^(s-127) for s in 1..254 is the normal float with exponent field s; s == 0 is the
// denormal 2^-127.
__device__ __forceinline__ float e8m0_to_f32(uint32_t s)
{
    float v = __uint_as_float(s << 23);
    v = (s == 0u) ? __uint_as_float(0x00400000u) : v;
    return (s == 255u) ? 0.0f : v;
}

// Two E2M1 codes (one packed byte, low nibble first) -> f16x2, exact.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte_in_low8)
{
    uint32_t r;
    asm("{\n\t.reg .b8 b0;\n\tcvt.u8.u32 b0, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b0;\n\t}"
        : "=r"(r) : "r"(byte_in_low8));
    return r;
}

// Four packed bytes (8 codes) -> four f16x2 words, element order preserved.
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t out[4])
{
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(out[0]), "=r"(out[1]), "=r"(out[2]), "=r"(out[3]) : "r"(w));
}

__device__ __forceinline__ float2 f16x2_to_f32x2(uint32_t h2)
{
    __half2 h = *reinterpret_cast<__half2 *>(&h2);
    return __half22float2(h);
}

// Packed fp32 pair FMA (sm_100): d = a * b + c per lane.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c)
{
    unsigned long long A, B, C, D;
    A = *reinterpret_cast<unsigned long long *>(&a);
    B = *reinterpret_cast<unsigned long long *>(&b);
    C = *reinterpret_cast<unsigned long long *>(&c);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(D) : "l"(A), "l"(B), "l"(C));
    return *reinterpret_cast<float2 *>(&D);
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// Site ids for k3_raise, so a device error names the kernel that stored it.
enum {
    K3_SITE_MXFP4 = 1, K3_SITE_ROUTER = 2, K3_SITE_MOE = 3, K3_SITE_GEMV = 4,
    K3_SITE_KDA = 5, K3_SITE_MLA = 6, K3_SITE_SMALL = 7, K3_SITE_STACK = 8,
    K3_SITE_EP = 9
};
