// moe.cu -- mixture-of-experts routing (decode and batched prefill) and the batched
// prefill's row gather and combine.
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
//                      the last CTA to finish (a ticket) then, with one warp: softmax,
//                      top n_used, renormalised weights, written in ascending expert order
//                      (sel[k], w[k]) for the expert GEMVs
// The batched prefill routes every token of a chunk in one launch (moe_route_rows_kernel: the
// same norm, logits and selection per token), gathers each expert's rows
// (gather_rows_f16_kernel) for the GEMMs, and adds the experts' outputs back in candle's order
// (moe_combine_rows_kernel).
#include "common.cuh"
#include "moe.h"

namespace tptc {
namespace {

constexpr int kRouterWarps = 8;

// xn[0, dim) = x / sqrt(sum(x^2) / dim + eps) * w (candle_nn::ops::rms_norm) by the whole CTA
// (kRouterWarps warps); `red` holds kRouterWarps floats.  Ends with a barrier.
__device__ __forceinline__ void norm_row(const float* x, const float* w, int dim, float eps, float* xn, float* red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float ss = 0.f;
    for (int i = tid; i < dim; i += blockDim.x) ss = __fmaf_rn(x[i], x[i], ss);
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < kRouterWarps; k++) tot += red[k];
    const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)dim), eps));
    for (int i = tid; i < dim; i += blockDim.x) xn[i] = __fmul_rn(__fdiv_rn(x[i], m), w[i]);
    __syncthreads();
}

// Router logit of expert e (one warp; the result in every lane): dot(router row e, xn).
__device__ __forceinline__ float router_logit(const MoeRouteParams& p, int e, const float* xn, int lane) {
    const int dim = p.dim;
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
    return acc;
}

// (value, index) of the better of two routing weights: larger weight, then lower index.
__device__ __forceinline__ bool route_better(float v, int i, float bv, int bi) {
    return i >= 0 && (bi < 0 || v > bv || (v == bv && i < bi));
}

struct SelectScratch {
    float rw[kMoeMaxExperts];
    unsigned char taken[kMoeMaxExperts];
    int order[kMoeMaxUsed];
};

// One warp: softmax over logits[0, E) (max, exp(l - max), the sum in index order, each divided
// by it), the K largest (stable descending order: ties to the lower index), their weights
// divided by the sum of the chosen ones in that order; sel / w written in ascending expert
// order.  `logits` is global memory written by the previous kernel (read after its wait) or
// shared memory: plain loads.
__device__ __forceinline__ void select_topk(const float* logits, int E, int K, int* sel, float* w, SelectScratch& s) {
    const int lane = threadIdx.x & 31;
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, logits[e]);
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int e = lane; e < E; e += 32) {
        s.rw[e] = expf(__fsub_rn(logits[e], mx));
        s.taken[e] = 0;
    }
    __syncwarp();
    float sum = 0.f;
    if (lane == 0)
        for (int e = 0; e < E; e++) sum = __fadd_rn(sum, s.rw[e]);
    sum = __shfl_sync(0xffffffffu, sum, 0);
    for (int e = lane; e < E; e += 32) s.rw[e] = __fdiv_rn(s.rw[e], sum);
    __syncwarp();
    for (int k = 0; k < K; k++) {
        float bv = -INFINITY;
        int bi = -1;
        for (int e = lane; e < E; e += 32)
            if (!s.taken[e] && route_better(s.rw[e], e, bv, bi)) {
                bv = s.rw[e];
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
            s.order[k] = bi;
            s.taken[bi] = 1;
        }
        __syncwarp();
    }
    if (lane == 0) {
        float tot = 0.f;  // the selected weights' sum in selection order
        for (int k = 0; k < K; k++) tot = __fadd_rn(tot, s.rw[s.order[k]]);
        int ids[kMoeMaxUsed];
        for (int k = 0; k < K; k++) {  // ascending expert order
            int v = s.order[k], j = k;
            while (j > 0 && ids[j - 1] > v) {
                ids[j] = ids[j - 1];
                j--;
            }
            ids[j] = v;
        }
        for (int k = 0; k < K; k++) {
            sel[k] = ids[k];
            w[k] = __fdiv_rn(s.rw[ids[k]], tot);
        }
    }
    __syncwarp();
}

// Four consecutive router weights of row `row` from element i, as f32.
__device__ __forceinline__ float4 router_quad(const MoeRouteParams& p, int row, int i) {
    if (p.router_f16) {
        const uint2 raw = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p.router) + (size_t)row * p.dim + i);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        return make_float4(a.x, a.y, b.x, b.y);
    }
    return *reinterpret_cast<const float4*>(static_cast<const float*>(p.router) + (size_t)row * p.dim + i);
}

// One CTA per expert: the expert's router row is loaded into registers before the wait for
// the previous kernel (weights do not depend on it), the CTA normalises x after it, and its
// threads split the dot product (a fixed-order block reduction).  The last CTA to write its
// logit (a ticket on p.count, which it resets) selects the experts with one warp.
constexpr int kRouterPre = 4;  // float4 quads of the row each thread holds (dim <= 4096 in registers)
__global__ void __launch_bounds__(kRouterWarps * 32) moe_router_kernel(const MoeRouteParams p) {
    extern __shared__ __align__(16) float xn[];
    __shared__ float red[kRouterWarps];
    __shared__ float lg[kMoeMaxExperts];
    __shared__ SelectScratch s;
    __shared__ int last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, e = blockIdx.x, nt = blockDim.x;
    float4 wq[kRouterPre];
#pragma unroll
    for (int j = 0; j < kRouterPre; j++) {
        const int i = (j * nt + tid) * 4;
        wq[j] = i < p.dim ? router_quad(p, e, i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    pdl_wait();
    pdl_launch_dependents();
    norm_row(p.x, p.norm_w, p.dim, p.eps, xn, red);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < kRouterPre; j++) {
        const int i = (j * nt + tid) * 4;
        if (i < p.dim) {
            const float4 v = *reinterpret_cast<const float4*>(xn + i);
            acc = __fmaf_rn(wq[j].x, v.x, acc);
            acc = __fmaf_rn(wq[j].y, v.y, acc);
            acc = __fmaf_rn(wq[j].z, v.z, acc);
            acc = __fmaf_rn(wq[j].w, v.w, acc);
        }
    }
    for (int i = (kRouterPre * nt + tid) * 4; i < p.dim; i += nt * 4) {  // rows beyond dim 4096
        const float4 w4 = router_quad(p, e, i), v = *reinterpret_cast<const float4*>(xn + i);
        acc = __fmaf_rn(w4.x, v.x, acc);
        acc = __fmaf_rn(w4.y, v.y, acc);
        acc = __fmaf_rn(w4.z, v.z, acc);
        acc = __fmaf_rn(w4.w, v.w, acc);
    }
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    __syncthreads();  // red is free again (norm_row's readers are past its last barrier)
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (tid == 0) {
        float tot = 0.f;
        for (int k = 0; k < kRouterWarps; k++) tot += red[k];
        p.logits[e] = tot;
        __threadfence();  // the logit before the ticket
        last = atomicAdd(p.count, 1) == p.n_expert - 1;
    }
    __syncthreads();
    if (!last || warp != 0) return;
    __threadfence();  // every other CTA's logit is visible after its ticket
    for (int i = lane; i < p.n_expert; i += 32) lg[i] = __ldcg(p.logits + i);
    __syncwarp();
    select_topk(lg, p.n_expert, p.n_used, p.sel, p.w, s);
    if (lane == 0) *p.count = 0;  // for the next launch
}

// Every token of a prefill chunk: x, sel and w are [T] rows of dim, n_used and n_used.
__global__ void __launch_bounds__(kRouterWarps * 32) moe_route_rows_kernel(const MoeRouteParams p) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[kRouterWarps];
    __shared__ SelectScratch s;
    float* xn = sm;
    float* lg = sm + p.dim;
    const size_t t = blockIdx.x;
    norm_row(p.x + t * p.dim, p.norm_w, p.dim, p.eps, xn, red);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int e = warp; e < p.n_expert; e += kRouterWarps) {
        const float v = router_logit(p, e, xn, lane);
        if (lane == 0) lg[e] = v;
    }
    __syncthreads();
    if (warp == 0) select_topk(lg, p.n_expert, p.n_used, p.sel + t * p.n_used, p.w + t * p.n_used, s);
}

// dst[r][0, dim) = src[idx[r]][0, dim) (fp16 rows, dim a multiple of 8); one CTA per row.
__global__ void __launch_bounds__(128) gather_rows_f16_kernel(const __half* src, const int* idx, int dim, __half* dst) {
    const size_t r = blockIdx.x;
    const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)idx[r] * dim);
    uint4* d = reinterpret_cast<uint4*>(dst + r * dim);
    for (int i = threadIdx.x; i < dim / 8; i += blockDim.x) d[i] = s[i];
}

// x[t] = ys + x[t] with ys = the token's chosen experts' rows y[row_of[t][k]] times w[t][k],
// added in ascending expert order from zero, then the shared expert's row (candle
// MlpOrMoe::MoE's index_add order, as the decode path's down GEMVs add them).
__global__ void __launch_bounds__(256) moe_combine_rows_kernel(float* x, const float* y, const int* row_of,
                                                              const float* w, int K, const float* shared_y, int dim) {
    const size_t t = blockIdx.x;
    for (int j = threadIdx.x; j < dim; j += blockDim.x) {
        float ys = 0.f;
        for (int k = 0; k < K; k++) {
            const float a = __fmul_rn(y[(size_t)row_of[t * K + k] * dim + j], w[t * K + k]);
            ys = k == 0 ? a : __fadd_rn(ys, a);
        }
        if (shared_y) ys = __fadd_rn(ys, shared_y[t * dim + j]);
        x[t * dim + j] = __fadd_rn(ys, x[t * dim + j]);
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

bool route_params_ok(const MoeRouteParams& p) {
    return p.n_expert >= 2 && p.n_expert <= kMoeMaxExperts && p.n_used >= 1 && p.n_used <= kMoeMaxUsed &&
           p.n_used <= p.n_expert && p.dim % 128 == 0 && p.dim <= kMoeMaxDim;
}

}  // namespace

cudaError_t launch_moe_route(const MoeRouteParams& p, cudaStream_t st, bool pdl) {
    if (!route_params_ok(p)) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    if (!p.count) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = route_cfg(dim3(p.n_expert), dim3(kRouterWarps * 32), (size_t)p.dim * 4, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, moe_router_kernel, p);
}

cudaError_t launch_moe_route_rows(const MoeRouteParams& p, int T, cudaStream_t st) {
    if (!route_params_ok(p) || T < 1) return cudaErrorInvalidValue;
    moe_route_rows_kernel<<<T, kRouterWarps * 32, (size_t)(p.dim + p.n_expert) * 4, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_gather_rows_f16(const __half* src, const int* idx, int rows, int dim, __half* dst, cudaStream_t st) {
    if (rows < 1 || dim % 8) return rows == 0 ? cudaSuccess : cudaErrorInvalidValue;
    gather_rows_f16_kernel<<<rows, 128, 0, st>>>(src, idx, dim, dst);
    return cudaGetLastError();
}

cudaError_t launch_moe_combine_rows(float* x, const float* y, const int* row_of, const float* w, int K,
                                    const float* shared_y, int T, int dim, cudaStream_t st) {
    if (T < 1) return cudaSuccess;
    moe_combine_rows_kernel<<<T, 256, 0, st>>>(x, y, row_of, w, K, shared_y, dim);
    return cudaGetLastError();
}

cudaError_t moe_init_device() {
    cudaError_t e = cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMoeMaxDim * 4);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(moe_route_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (kMoeMaxDim + kMoeMaxExperts) * 4);
}

}  // namespace tptc
