// moe.h -- mixture-of-experts routing kernels (moe.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tptc {

constexpr int kMoeMaxExperts = 1024;  // experts per layer the select kernel holds in shared memory
constexpr int kMoeMaxUsed = 16;       // experts chosen per token
constexpr int kMoeMaxDim = 16384;     // the router kernel keeps the normed activation in shared memory

struct MoeRouteParams {
    const float* x;       // residual stream [dim]
    const float* norm_w;  // ffn_norm gain [dim]
    float eps;
    const void* router;   // [n_expert][dim] rows, f32 or (router_f16) fp16; 16-byte aligned
    int router_f16;
    int dim, n_expert, n_used;
    float* logits;  // [n_expert] scratch
    int* sel;       // [n_used] out: selected experts, ascending
    float* w;       // [n_used] out: their renormalised routing weights
    int* count;     // decode: a zeroed counter (the routing kernel leaves it zeroed)
};

// Router logits and the top-n_used selection in one launch (a CTA per expert; the last one
// selects), after the previous kernel (programmatic dependent launch when pdl).
cudaError_t launch_moe_route(const MoeRouteParams& p, cudaStream_t st, bool pdl);
// Batched prefill: the same routing for T tokens (x, sel and w hold T rows), one launch.
cudaError_t launch_moe_route_rows(const MoeRouteParams& p, int T, cudaStream_t st);
// dst[r] = src[idx[r]] for r < rows (fp16 rows of dim elements, dim a multiple of 8).
cudaError_t launch_gather_rows_f16(const __half* src, const int* idx, int rows, int dim, __half* dst, cudaStream_t st);
// x[t] = (sum over k of y[row_of[t K + k]] * w[t K + k], in k order, then + shared_y[t]) + x[t]
// for t < T (f32 rows of dim; shared_y may be null).
cudaError_t launch_moe_combine_rows(float* x, const float* y, const int* row_of, const float* w, int K,
                                    const float* shared_y, int T, int dim, cudaStream_t st);
cudaError_t moe_init_device();

}  // namespace tptc
