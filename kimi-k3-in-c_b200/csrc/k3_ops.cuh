// k3_ops.cuh -- internal launchers shared between the libk3cuda translation units.
// All take device pointers and a stream, launch asynchronously, and return K3D_OK or
// the recorded error code.
#pragma once
#include "k3_common.cuh"

namespace k3 {

// k3_mxfp4.cu
int mxfp4_gemv(float *y, const float *x, const unsigned char *packed,
               const unsigned char *scales, int in, int rows, int group, cudaStream_t s);

// k3_gemv.cu
int gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out, int T,
              int accumulate, cudaStream_t s);
int gemv_bf16_swiglu(float *act, const float *x, const uint16_t *Wg, const uint16_t *Wu,
                     int in, int inter, int T, cudaStream_t s);
int gemv_f32(float *y, const float *x, const float *W, int in, int out, cudaStream_t s);
int gemv_bf16_multi(int nseg, const uint16_t *const *W, float *const *y, const int *rows,
                    const float *x, int in, int T, cudaStream_t s);
int gemv_bf16_argmax(float *y, unsigned long long *key, int *next, const float *x,
                     const uint16_t *W, int in, int out, int T, cudaStream_t s);
// tagged weight: wdt 0 fp32, 1 bf16
int gemv_tagged(float *y, const float *x, const void *W, int wdt, int in, int out,
                cudaStream_t s);

// k3_mxfp4_mma.cu
struct MoeWork;
bool mma_supported(int in, int rows, int mode);
int xsplit(__half *xb, float *xsc, const float *x, int n, int nvec, size_t ld, cudaStream_t s);
int mxfp4_mma_launch(int mode, const MoeWork &w, int umax, int in, int rows, const __half *xb,
                     const float *xsc, int x_by_assign, float *out, cudaStream_t st);

// k3_router.cu
size_t router_ws_bytes(int T, int n_experts);
int router_f32(int *idx, float *w, const float *x, const float *W, const float *bias,
               int T, int hidden, int n_experts, int topk, int renorm, float routed_scale,
               void *ws, cudaStream_t s);
int router_bf16(int *idx, float *w, const float *x, const uint16_t *W, const float *bias,
                int T, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                void *ws, cudaStream_t s);

// k3_small.cu
int rmsnorm(float *y, const float *x, const float *w, int n, int rows, float eps,
            cudaStream_t s);
int situ_glu(float *y, const float *x, int n, int rows, float b1, float b2, cudaStream_t s);
int silu_mul(float *y, const float *gu, int n, int rows, cudaStream_t s);

}  // namespace k3
