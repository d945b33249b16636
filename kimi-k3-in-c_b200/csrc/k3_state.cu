// k3_state.cu -- device helpers for moving the decode caches in and out of the CPU
// engine's conversation-state layout (K3ST, src/cli/k3_run.c:158-300): widening bf16
// cache rows to fp32, rounding fp32 rows back to bf16, and a bf16 matrix transpose (kv_b^T
// for recovering a latent from expanded keys and values). All three are plain memory
// passes (HBM-bound, one read and one write per element); they run once per save or load,
// not per token.
#include "k3_common.cuh"
#include "k3_ops.cuh"

namespace k3 {

// dst[r][c] = widen(src[r * spitch + c]) for r < rows, c < cols; grid-stride over elements.
__global__ void k_bf16_rows_to_f32(float *dst, const uint16_t *src, size_t spitch, int rows, int cols)
{
    const size_t n = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        dst[i] = bf16_to_f32(src[r * spitch + c]);
    }
}

// dst[r * dpitch + c] = bf16(src[r][c]), round to nearest even (NaN stays NaN).
__global__ void k_f32_rows_to_bf16(uint16_t *dst, size_t dpitch, const float *src, int rows, int cols)
{
    const size_t n = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        dst[r * dpitch + c] = f32_to_bf16_bits(src[i]);
    }
}

// dst[c][r] = src[r][c] for a rows x cols matrix of 16-bit values: 32 x 32 tiles through
// shared memory so both the reads and the writes are coalesced. grid (ceil(cols/32),
// ceil(rows/32)), block (32, 8).
__global__ void k_transpose_u16(uint16_t *dst, const uint16_t *src, int rows, int cols)
{
    __shared__ uint16_t tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int r = r0 + k, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[k][threadIdx.x] = src[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int c = c0 + k, r = r0 + threadIdx.x;
        if (r < rows && c < cols) dst[(size_t)c * rows + r] = tile[threadIdx.x][k];
    }
}

static int grid_elems(size_t n)
{
    size_t g = (n + 255) / 256;
    const size_t cap = (size_t)(sm_count() > 0 ? sm_count() : 148) * 16;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace k3

using namespace k3;

extern "C" {

int k3d_bf16_rows_to_f32(float *dst, const uint16_t *src, size_t spitch, int rows, int cols)
{
    K3_TRY(ensure_ctx());
    if (!dst || !src || rows < 0 || cols < 0 || spitch < (size_t)cols)
        return fail(K3D_EINVAL, "k3d_bf16_rows_to_f32");
    if (!rows || !cols) return K3D_OK;
    k_bf16_rows_to_f32<<<grid_elems((size_t)rows * cols), 256, 0, stream()>>>(dst, src, spitch, rows, cols);
    note_launch();
    return check_launch("bf16 rows to f32");
}

int k3d_f32_rows_to_bf16(uint16_t *dst, size_t dpitch, const float *src, int rows, int cols)
{
    K3_TRY(ensure_ctx());
    if (!dst || !src || rows < 0 || cols < 0 || dpitch < (size_t)cols)
        return fail(K3D_EINVAL, "k3d_f32_rows_to_bf16");
    if (!rows || !cols) return K3D_OK;
    k_f32_rows_to_bf16<<<grid_elems((size_t)rows * cols), 256, 0, stream()>>>(dst, dpitch, src, rows, cols);
    note_launch();
    return check_launch("f32 rows to bf16");
}

int k3d_transpose_u16(uint16_t *dst, const uint16_t *src, int rows, int cols)
{
    K3_TRY(ensure_ctx());
    if (!dst || !src || rows < 0 || cols < 0 || dst == src) return fail(K3D_EINVAL, "k3d_transpose_u16");
    if (!rows || !cols) return K3D_OK;
    k_transpose_u16<<<dim3((cols + 31) / 32, (rows + 31) / 32), dim3(32, 8), 0, stream()>>>(dst, src, rows, cols);
    note_launch();
    return check_launch("transpose u16");
}

}  // extern "C"
