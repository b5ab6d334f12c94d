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
};

// Router logits and the top-n_used selection: two launches (a grid over the experts, then
// one warp), both after the previous kernel (programmatic dependent launch when pdl).
cudaError_t launch_moe_route(const MoeRouteParams& p, cudaStream_t st, bool pdl);
cudaError_t moe_init_device();

}  // namespace tptc
