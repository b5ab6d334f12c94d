// moe.cu -- mixture-of-experts routing for the decode step.
//
// Semantics: candle quantized_llama MlpOrMoe::MoE (the forward of Mixtral-style GGUFs, which
// the reference's candle engine loads through ModelWeights::from_gguf): router logits of the
// ffn-normed activation, softmax over every expert, the n_used largest routing weights (ties
// to the lower expert index: candle sorts the expert indices with a stable sort_by on
// total_cmp), those weights divided by their sum, and the experts' outputs accumulated in
// ascending expert order.  The reference's wgpu engine (wgpu_engine.rs:781-864) runs the same
// router, reads its logits back to the host and selects there; here the selection stays on
// the device, so a decode step remains one CUDA graph:
//   moe_router_kernel  RMSNorm of the residual stream with the ffn_norm gain, then one warp
//                      per expert: logit[e] = dot(router row e, xn) in f32 (F32 or F16 rows,
//                      which candle dequantises to f32 and multiplies in f32)
//   moe_select_kernel  one warp: softmax, top n_used, renormalised weights, written in
//                      ascending expert order (sel[k], w[k]) for the expert GEMVs
#include "common.cuh"
#include "moe.h"

namespace tptc {
namespace {

constexpr int kRouterWarps = 8;

__global__ void __launch_bounds__(kRouterWarps * 32) moe_router_kernel(const MoeRouteParams p) {
    extern __shared__ __align__(16) float xn[];
    __shared__ float red[kRouterWarps];
    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dim = p.dim;
    // candle_nn::ops::rms_norm: m = sqrt(sum(x^2) / dim + eps); xn = x / m * w
    float ss = 0.f;
    for (int i = tid; i < dim; i += blockDim.x) ss = __fmaf_rn(p.x[i], p.x[i], ss);
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < kRouterWarps; w++) tot += red[w];
    const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)dim), p.eps));
    for (int i = tid; i < dim; i += blockDim.x) xn[i] = __fmul_rn(__fdiv_rn(p.x[i], m), p.norm_w[i]);
    __syncthreads();
    const int e = blockIdx.x * kRouterWarps + warp;
    if (e >= p.n_expert) return;
    float acc = 0.f;
    if (p.router_f16) {
        const __half* row = static_cast<const __half*>(p.router) + (size_t)e * dim;
        for (int i = 4 * lane; i < dim; i += 128) {
            const uint2 raw = *reinterpret_cast<const uint2*>(row + i);
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
            const float4 v = *reinterpret_cast<const float4*>(xn + i);
            acc = __fmaf_rn(a.x, v.x, acc);
            acc = __fmaf_rn(a.y, v.y, acc);
            acc = __fmaf_rn(b.x, v.z, acc);
            acc = __fmaf_rn(b.y, v.w, acc);
        }
    } else {
        const float* row = static_cast<const float*>(p.router) + (size_t)e * dim;
        for (int i = 4 * lane; i < dim; i += 128) {
            const float4 w4 = *reinterpret_cast<const float4*>(row + i);
            const float4 v = *reinterpret_cast<const float4*>(xn + i);
            acc = __fmaf_rn(w4.x, v.x, acc);
            acc = __fmaf_rn(w4.y, v.y, acc);
            acc = __fmaf_rn(w4.z, v.z, acc);
            acc = __fmaf_rn(w4.w, v.w, acc);
        }
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) p.logits[e] = acc;
}

// (value, index) of the better of two routing weights: larger weight, then lower index.
__device__ __forceinline__ bool route_better(float v, int i, float bv, int bi) {
    return i >= 0 && (bi < 0 || v > bv || (v == bv && i < bi));
}

__global__ void __launch_bounds__(32) moe_select_kernel(const MoeRouteParams p) {
    __shared__ float rw[kMoeMaxExperts];
    __shared__ unsigned char taken[kMoeMaxExperts];
    __shared__ int order[kMoeMaxUsed];
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x, E = p.n_expert, K = p.n_used;
    // softmax_last_dim: max, exp(l - max), the sum in index order, then each divided by it
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, __ldcg(p.logits + e));
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int e = lane; e < E; e += 32) {
        rw[e] = expf(__fsub_rn(__ldcg(p.logits + e), mx));
        taken[e] = 0;
    }
    __syncwarp();
    float sum = 0.f;
    if (lane == 0)
        for (int e = 0; e < E; e++) sum = __fadd_rn(sum, rw[e]);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int e = lane; e < E; e += 32) rw[e] = __fdiv_rn(rw[e], sum);
    __syncwarp();
    // the K largest, one per round (stable descending order: ties to the lower index)
    for (int k = 0; k < K; k++) {
        float bv = -INFINITY;
        int bi = -1;
        for (int e = lane; e < E; e += 32)
            if (!taken[e] && route_better(rw[e], e, bv, bi)) {
                bv = rw[e];
                bi = e;
            }
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (route_better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            order[k] = bi;
            taken[bi] = 1;
        }
        __syncwarp();
    }
    if (lane == 0) {
        float s = 0.f;  // the selected weights' sum in selection order
        for (int k = 0; k < K; k++) s = __fadd_rn(s, rw[order[k]]);
        // ascending expert order (the order candle accumulates the experts in)
        int ids[kMoeMaxUsed];
        for (int k = 0; k < K; k++) {
            int v = order[k], j = k;
            while (j > 0 && ids[j - 1] > v) {
                ids[j] = ids[j - 1];
                j--;
            }
            ids[j] = v;
        }
        for (int k = 0; k < K; k++) {
            p.sel[k] = ids[k];
            p.w[k] = __fdiv_rn(rw[ids[k]], s);
        }
    }
}

cudaLaunchConfig_t route_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

}  // namespace

cudaError_t launch_moe_route(const MoeRouteParams& p, cudaStream_t st, bool pdl) {
    if (p.n_expert < 2 || p.n_expert > kMoeMaxExperts || p.n_used < 1 || p.n_used > kMoeMaxUsed ||
        p.n_used > p.n_expert || p.dim % 128 || p.dim > kMoeMaxDim)
        return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = route_cfg(dim3((p.n_expert + kRouterWarps - 1) / kRouterWarps), dim3(kRouterWarps * 32),
                                       (size_t)p.dim * 4, st, pdl, attr);
    cudaError_t e = cudaLaunchKernelEx(&cfg, moe_router_kernel, p);
    if (e != cudaSuccess) return e;
    cfg = route_cfg(dim3(1), dim3(32), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, moe_select_kernel, p);
}

cudaError_t moe_init_device() {
    return cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMoeMaxDim * 4);
}

}  // namespace tptc
