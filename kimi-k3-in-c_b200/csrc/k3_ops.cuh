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
// RMSNorm of the input done by the consuming GEMV (x is then the raw residual stream).
struct NormIn {
    const float *w;
    float eps;
};
// k3_gemv_stream.cu: the streamed forms; each returns 1 when it launched, 0 when the shape
// needs the register-staged kernels instead
int gemv_stream_multi(int nseg, const uint16_t *const *W, float *const *y, const int *rows,
                      const float *x, int in, int T, int accumulate, cudaStream_t st,
                      const NormIn *ni = nullptr);
int gemv_stream_swiglu(float *act, const float *x, const uint16_t *Wg, const uint16_t *Wu,
                       int in, int inter, int T, cudaStream_t st);
int gemv_stream_argmax(float *y, unsigned long long *key, const float *x, const uint16_t *W,
                       int in, int out, int T, cudaStream_t st, const NormIn *ni = nullptr);
// With ni, x is the raw residual stream and is RMS-normalised first (in the streamed
// kernel's load when it runs, else by a separate rmsnorm into the library scratch).
int gemv_bf16_multi(int nseg, const uint16_t *const *W, float *const *y, const int *rows,
                    const float *x, int in, int T, cudaStream_t s, const NormIn *ni = nullptr);
int gemv_bf16_argmax(float *y, unsigned long long *key, int *next, const float *x,
                     const uint16_t *W, int in, int out, int T, cudaStream_t s,
                     const NormIn *ni = nullptr);
// x RMS-normalised into the library scratch (slot 0) for consumers that cannot normalise on
// load; returns the normalised copy, or null with the error recorded.
const float *norm_to_scratch(const float *x, const NormIn &ni, int n, int rows, cudaStream_t s);
// k3_gemv_ref.cu: k3_matmul's double-accumulator order, bit-exact with the CPU engine
// (the reference-semantics entry points); T rows of x one after another
int gemv_ref_f32(float *y, const float *x, const float *W, int in, int out, int T, int accumulate,
                 cudaStream_t s);
int gemv_ref_bf16(float *y, const float *x, const uint16_t *W, int in, int out, int T, int accumulate,
                  cudaStream_t s);
// tagged weight: wdt 0 fp32, 1 bf16 (the CPU engine's arithmetic, through gemv_ref_*)
int gemv_tagged(float *y, const float *x, const void *W, int wdt, int in, int out,
                cudaStream_t s);

// k3_mxfp4_mma.cu
struct MoeWork;
bool mma_supported(int in, int rows, int mode);
int xsplit(__half *xb, float *xsc, const float *x, int n, int nvec, size_t ld, cudaStream_t s);
int mxfp4_mma_launch(int mode, const MoeWork &w, int umax, int in, int rows, const __half *xb,
                     const float *xsc, int x_by_assign, float *out, cudaStream_t st);

// k3_mxfp4_umma.cu (tcgen05 block-scaled MXFP4; mode 0 gate/up, 1 down)
bool umma_supported(int K, int rows, int mode);
int umma_slices(int units, int K, int rows, int mode);
size_t umma_bq_bytes(int K);
size_t umma_bs_bytes(int K);
int umma_bsplit(uint8_t *bq, uint8_t *bs, const float *x, int K, int nvec, size_t ld,
                cudaStream_t st);
// the fused decode pass (gate/up, act split, down in one launch)
int umma_fused_ok(int npos, int hidden, int inter);
size_t umma_fused_cnt_ints(int npos, int inter);
int umma_launch_fused(const MoeWork &w, const int *idx, const int *count, int npos_max, int hidden, int inter,
                      const uint8_t *bq_x, const uint8_t *bs_x, int vec_div, float *part_gu, size_t sl_gu,
                      uint8_t *bq_a, uint8_t *bs_a, float *part_d, size_t sl_d, int *cnt, cudaStream_t st);
int umma_bsplit_swiglu(uint8_t *bq, uint8_t *bs, const float *part, int ks, size_t slice_stride,
                       int inter, const int *count, int npos, cudaStream_t st);
int umma_slice_sum(float *y, const float *part, int ks, size_t slice_stride, int n,
                   cudaStream_t st);
int umma_launch(int mode, int tiled, const MoeWork &w, const int *idx, const int *count,
                int npos_max, int K, int rows, int ks, const uint8_t *bq, const uint8_t *bs,
                int vec_div, float *part, int out_w, size_t slice_stride, cudaStream_t st,
                int early, int resident = 0);
// Grouped items (a batch: several tokens per expert): groups of up to four consecutive
// grouped positions of one expert share each weight stage (tiled experts).
struct UmmaGroups {
    int *ng;                 // [1] number of groups
    int *p0, *n, *e;         // per group: first position, positions (<= 4), expert
    int *pos_of;             // per assignment: its grouped position
};
size_t umma_bq_group_bytes(int K);
int umma_make_groups(const MoeWork &w, const UmmaGroups &G, cudaStream_t st);
int umma_bsplit_group_x(uint8_t *bq, uint8_t *bs, const float *x, int hidden, const int *assign, int K,
                        const UmmaGroups &G, int max_groups, cudaStream_t st);
int umma_bsplit_swiglu_group(uint8_t *bq, uint8_t *bs, const float *part, int ks, size_t slice_stride, int inter,
                             const UmmaGroups &G, int max_groups, cudaStream_t st);
int umma_launch_grouped(int mode, const MoeWork &w, const UmmaGroups &G, int max_groups, int K, int rows,
                        int ks, const uint8_t *bq, const uint8_t *bs, float *part, int out_w,
                        size_t slice_stride, cudaStream_t st);

// k3_gemm_tc.cu: Y[j][T][rows[j]] (+)= x[T][in] . W[j]^T on the tensor cores (more than four
// tokens); swiglu: two matrices (gate, up), Y[0] = silu(gate) * up
int gemm_bf16_tc(int nmat, const uint16_t *const *W, float *const *Y, const int *rows, const float *x,
                 int in, int T, int accumulate, int swiglu, cudaStream_t st);

// k3_gemv.cu: the LM head in pieces (keys of a vocabulary slice, global index shift, finish)
int lm_head_keys(float *y, unsigned long long *key, const float *x, const uint16_t *W, int in, int out, int T,
                 cudaStream_t s, const NormIn *ni);
int key_offset(unsigned long long *key, int T, int v0, cudaStream_t s);
int argmax_finish(int *next, const unsigned long long *key, int T, cudaStream_t s);
// k3_ep.cu: element-wise max of n uint64 over the ranks, in place (no-op on one rank)
int ep_allreduce_max_u64(unsigned long long *buf, size_t n, cudaStream_t s);

// k3_ep.cu: grouped byte exchange with every rank (a device copy on one rank)
int ep_exchange(const void *send, const size_t *scnt, const size_t *soff, void *recv,
                const size_t *rcnt, const size_t *roff, cudaStream_t st);

// k3_router.cu
size_t router_ws_bytes(int T, int n_experts);
int router_f32(int *idx, float *w, const float *x, const float *W, const float *bias,
               int T, int hidden, int n_experts, int topk, int renorm, float routed_scale,
               void *ws, cudaStream_t s);
// Optional grouping of the routed assignments by expert (the MoE's prep step), done by the
// router's own launch when its fused kernel runs (done = 1), else left to the caller.
struct RouterGroup {
    int *n_active, *act_expert, *act_off, *assign;
    int lo, hi;
    int done;
    int *zero = nullptr;     // zeroed by the grouping (the fused expert pass's counters)
    int nzero = 0;
};
int router_bf16(int *idx, float *w, const float *x, const uint16_t *W, const float *bias,
                int T, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                void *ws, cudaStream_t s, RouterGroup *grp = nullptr);

// k3_small.cu
int rmsnorm(float *y, const float *x, const float *w, int n, int rows, float eps,
            cudaStream_t s);
int situ_glu(float *y, const float *x, int n, int rows, float b1, float b2, cudaStream_t s);
int silu_mul(float *y, const float *gu, int n, int rows, cudaStream_t s);

}  // namespace k3
