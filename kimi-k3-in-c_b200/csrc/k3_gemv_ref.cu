// k3_gemv_ref.cu -- the CPU engine's GEMV arithmetic, bit for bit, for the reference-
// semantics entry points (k3_matmul, k3_matmul_bf16 and the k3.h composites built on
// k3_mmw: k3_moe, k3_mla_cached, k3_kda_layer, k3_decoder_layer_inc).
//
// k3_matmul (k3_ops.c:265-291) sums each row with sixteen double accumulators: accumulator
// l takes elements l, l + 16, l + 32, ... of the row by fused multiply-add in that order;
// the tree is ((a0 + a4) + (a8 + a12)) ... into b0..b3, then (b0 + b1) + (b2 + b3); the
// in % 16 tail is added sequentially by fma; the double is rounded to float once.
// k3_matmul_bf16 widens each bf16 weight exactly (<< 16) and is bit-identical to
// k3_matmul on the widened weights (test_ops.c:811-848).
//
// Here a half-warp owns a row and lane l of it is accumulator l: each step the 16 lanes
// read 16 consecutive weights (a coalesced 64- or 32-byte segment), every lane runs its
// own fma chain in the CPU's order, and the tree is four shuffles that pair the lanes
// exactly as the CPU pairs its accumulators. Products of two floats are exact in double,
// so the fma and the CPU's fma round identically; the results are the CPU's bits.
//
// These kernels serve the drop-in path, where the engine's own tests compare results
// with tolerances calibrated on its double arithmetic. The BASELINE decode stack (k3d_*)
// uses the streamed fp32 GEMVs of k3_gemv_stream.cu instead.
#include "k3_ops.cuh"

namespace k3 {

template <typename WT> __device__ __forceinline__ double wref(const WT *p);
template <> __device__ __forceinline__ double wref<float>(const float *p) { return (double)__ldg(p); }
template <> __device__ __forceinline__ double wref<uint16_t>(const uint16_t *p)
{
    return (double)__uint_as_float((uint32_t)__ldg(p) << 16);
}

// One row per half-warp; 256 threads = 16 rows per CTA, row pairs strided over the grid.
template <typename WT>
__global__ void __launch_bounds__(256) k_gemv_ref(float *y, const float *x, const WT *W, int in,
                                                  int out, int accumulate)
{
    pdl_wait();
    pdl_trigger();
    const int l = threadIdx.x & 15, half = (threadIdx.x >> 4) & 1;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int body = in & ~15;
    // the loop is uniform across the warp (both halves run every trip), so the full-mask
    // shuffles below always have all 32 lanes
    for (int o0 = 2 * warp; o0 < out; o0 += 2 * nwarps) {
        const int o = o0 + half;
        const bool valid = o < out;
        const WT *row = W + (size_t)(valid ? o : o0) * in;
        double a = 0.0;
        if (valid)
            for (int i = l; i < body; i += 16) a = __fma_rn(wref<WT>(row + i), (double)__ldg(x + i), a);
        // ((a_l + a_{l+4}) + (a_{l+8} + a_{l+12})) = b_l on lanes 0..3, then
        // (b0 + b1) + (b2 + b3) on lane 0: the CPU's tree
        const unsigned m = 0xffffffffu;
        double s = __dadd_rn(a, __shfl_down_sync(m, a, 4, 16));
        s = __dadd_rn(s, __shfl_down_sync(m, s, 8, 16));
        s = __dadd_rn(s, __shfl_down_sync(m, s, 1, 16));
        s = __dadd_rn(s, __shfl_down_sync(m, s, 2, 16));
        if (valid && l == 0) {
            for (int i = body; i < in; i++) s = __fma_rn(wref<WT>(row + i), (double)__ldg(x + i), s);
            const float v = (float)s;
            y[o] = accumulate ? __fadd_rn(y[o], v) : v;
        }
    }
}

template <typename WT>
static int launch_ref(float *y, const float *x, const WT *W, int in, int out, int T, int accumulate,
                      cudaStream_t s)
{
    if (out <= 0 || in <= 0 || T <= 0) return K3D_OK;
    int grid = (out + 15) / 16;          // 16 rows per CTA
    if (grid > sm_count() * 8) grid = sm_count() * 8;
    for (int t = 0; t < T; t++) {
        launch_pdl(k_gemv_ref<WT>, dim3(grid), dim3(256), 0, s, y + (size_t)t * out,
                   x + (size_t)t * in, W, in, out, accumulate);
        note_launch();
        K3_TRY(check_launch("gemv ref"));
    }
    return K3D_OK;
}

int gemv_ref_f32(float *y, const float *x, const float *W, int in, int out, int T, int accumulate,
                 cudaStream_t s)
{
    return launch_ref<float>(y, x, W, in, out, T, accumulate, s);
}

int gemv_ref_bf16(float *y, const float *x, const uint16_t *W, int in, int out, int T, int accumulate,
                  cudaStream_t s)
{
    return launch_ref<uint16_t>(y, x, W, in, out, T, accumulate, s);
}

}  // namespace k3
