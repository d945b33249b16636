// k3_fill.cu -- seeded device-side fills for the synthetic benchmark inputs. Element i
// of a fill depends only on (seed, i) through a SplitMix64 hash, so any slice can be
// regenerated independently (and a run is reproducible from its seed).
#include "k3_common.cuh"

namespace k3 {

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z)
{
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t hash_at(uint64_t seed, uint64_t i)
{
    return mix64(mix64(seed) ^ (i * 0xd1b54a32d192ed03ull));
}

// Irwin-Hall: sum of four 16-bit uniforms, centred; standard deviation
// sqrt((2^32 - 1) / 3) = 37837.23 before scaling.
__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t i, float stddev)
{
    const uint64_t h = hash_at(seed, i);
    const int s = (int)(h & 0xffff) + (int)((h >> 16) & 0xffff) + (int)((h >> 32) & 0xffff) +
                  (int)((h >> 48) & 0xffff) - 131070;
    return (float)s * (stddev / 37837.23f);
}

__global__ void k_fill_bf16_normal(uint16_t *dst, size_t n, uint64_t seed, float sd, size_t offset)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        dst[i] = f32_to_bf16_bits(normal_at(seed, offset + i, sd));
}

__global__ void k_fill_f32_normal(float *dst, size_t n, uint64_t seed, float sd, size_t offset)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        dst[i] = normal_at(seed, offset + i, sd);
}

__global__ void k_fill_f32_uniform(float *dst, size_t n, uint64_t seed, float lo, float hi, size_t offset)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const uint64_t h = hash_at(seed, offset + i);
        const float u = (float)(h >> 40) * (1.0f / 16777216.0f);   // [0, 1)
        dst[i] = lo + (hi - lo) * u;
    }
}

__global__ void k_fill_i32_uniform(int *dst, size_t n, uint64_t seed, int lo, int hi)
{
    const uint64_t span = (uint64_t)((int64_t)hi - (int64_t)lo + 1);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        dst[i] = lo + (int)(hash_at(seed, i) % span);
}

// 8 bytes per thread-iteration for the codes (uniform bytes = two uniform nibbles)
__global__ void k_fill_bytes(unsigned char *dst, size_t n, uint64_t seed)
{
    const size_t n8 = n / 8;
    uint64_t *d8 = reinterpret_cast<uint64_t *>(dst);
    const bool al = ((uintptr_t)dst & 7u) == 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (al ? n8 : n);
         i += (size_t)gridDim.x * blockDim.x) {
        if (al) d8[i] = hash_at(seed, i);
        else dst[i] = (unsigned char)(hash_at(seed, i) >> 24);
    }
    if (al && blockIdx.x == 0 && threadIdx.x < (n & 7))
        dst[n8 * 8 + threadIdx.x] = (unsigned char)(hash_at(seed ^ 0x5555, threadIdx.x) >> 24);
}

__global__ void k_fill_scales(unsigned char *dst, size_t n, uint64_t seed, int lo, int hi)
{
    const uint64_t span = (uint64_t)(hi - lo + 1);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        dst[i] = (unsigned char)(lo + (int)((hash_at(seed, i) >> 20) % span));
}

static int grid_n(size_t n)
{
    size_t g = (n + 255) / 256;
    const size_t cap = (size_t)sm_count() * 32;
    if (g > cap) g = cap;
    return g < 1 ? 1 : (int)g;
}

}  // namespace k3

using namespace k3;

extern "C" {

int k3d_fill_bf16_normal(uint16_t *dst, size_t n, uint64_t seed, float sd)
{
    K3_TRY(ensure_ctx());
    if (!dst) return fail(K3D_EINVAL, "fill null pointer");
    if (!n) return K3D_OK;
    k_fill_bf16_normal<<<grid_n(n), 256, 0, stream()>>>(dst, n, seed, sd, 0);
    note_launch();
    return check_launch("fill bf16");
}

int k3d_fill_bf16_normal_at(uint16_t *dst, size_t n, uint64_t seed, float sd, size_t offset)
{
    K3_TRY(ensure_ctx());
    if (!dst) return fail(K3D_EINVAL, "fill null pointer");
    if (!n) return K3D_OK;
    k_fill_bf16_normal<<<grid_n(n), 256, 0, stream()>>>(dst, n, seed, sd, offset);
    note_launch();
    return check_launch("fill bf16 at");
}

int k3d_fill_f32_normal_at(float *dst, size_t n, uint64_t seed, float sd, size_t offset)
{
    K3_TRY(ensure_ctx());
    if (!dst) return fail(K3D_EINVAL, "fill null pointer");
    if (!n) return K3D_OK;
    k_fill_f32_normal<<<grid_n(n), 256, 0, stream()>>>(dst, n, seed, sd, offset);
    note_launch();
    return check_launch("fill f32");
}

int k3d_fill_f32_normal(float *dst, size_t n, uint64_t seed, float sd)
{
    return k3d_fill_f32_normal_at(dst, n, seed, sd, 0);
}

int k3d_fill_f32_uniform_at(float *dst, size_t n, uint64_t seed, float lo, float hi, size_t offset)
{
    K3_TRY(ensure_ctx());
    if (!dst) return fail(K3D_EINVAL, "fill null pointer");
    if (!n) return K3D_OK;
    k_fill_f32_uniform<<<grid_n(n), 256, 0, stream()>>>(dst, n, seed, lo, hi, offset);
    note_launch();
    return check_launch("fill uniform");
}

int k3d_fill_f32_uniform(float *dst, size_t n, uint64_t seed, float lo, float hi)
{
    return k3d_fill_f32_uniform_at(dst, n, seed, lo, hi, 0);
}

int k3d_fill_i32_uniform(int *dst, size_t n, uint64_t seed, int lo, int hi)
{
    K3_TRY(ensure_ctx());
    if (!dst || hi < lo) return fail(K3D_EINVAL, "fill i32 arguments");
    if (!n) return K3D_OK;
    k_fill_i32_uniform<<<grid_n(n), 256, 0, stream()>>>(dst, n, seed, lo, hi);
    note_launch();
    return check_launch("fill i32");
}

int k3d_fill_mxfp4(unsigned char *packed, size_t packed_bytes, unsigned char *scales,
                   size_t scale_bytes, uint64_t seed, int s_lo, int s_hi)
{
    K3_TRY(ensure_ctx());
    if (!packed || !scales || s_lo < 0 || s_hi > 255 || s_hi < s_lo)
        return fail(K3D_EINVAL, "fill mxfp4 arguments");
    if (packed_bytes) {
        k_fill_bytes<<<grid_n(packed_bytes / 8 + 1), 256, 0, stream()>>>(packed, packed_bytes, seed);
        note_launch();
    }
    if (scale_bytes) {
        k_fill_scales<<<grid_n(scale_bytes), 256, 0, stream()>>>(scales, scale_bytes,
                                                                  seed ^ 0xa5a5a5a5ull, s_lo, s_hi);
        note_launch();
    }
    return check_launch("fill mxfp4");
}

}  // extern "C"
