// gemm_epi.cuh -- epilogue of the tcgen05 prefill GEMMs (gemm_tc.cu, gemm_q.cu): 32 f32
// accumulator columns of one row of C written as a plain store, a residual add, or the fused
// gate|up SiLU (or GEGLU) product in fp16.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "prefill.h"

namespace tptc {

__device__ __forceinline__ float silu_mul(float g, float u) { return __fmul_rn(__fdiv_rn(g, 1.f + expf(-g)), u); }
__device__ __forceinline__ float glu_mul(int geglu, float g, float u) { return geglu ? gelu_tanh_mul(g, u) : silu_mul(g, u); }

// Epilogue of 32 accumulator columns (col .. col + 31) of one row.
template <int EPI>
__device__ __forceinline__ void store_cols(const GemmTcParams& p, int row, int col, const uint32_t (&r)[32]) {
    if (row >= p.M || col >= p.N) return;
    if (EPI == GEMM_STORE || EPI == GEMM_RESID) {
        float* c = p.c + (size_t)row * p.ldc + col;
        if (col + 32 <= p.N && (p.ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(p.c) & 15) == 0) {
            float4* c4 = reinterpret_cast<float4*>(c);
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; j++)
                v[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            if (EPI == GEMM_RESID) {
                float4 o[8];
#pragma unroll
                for (int j = 0; j < 8; j++) o[j] = c4[j];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    v[j].x += o[j].x;
                    v[j].y += o[j].y;
                    v[j].z += o[j].z;
                    v[j].w += o[j].w;
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) c4[j] = v[j];
        } else {
            const int nv = min(32, p.N - col);
#pragma unroll
            for (int j = 0; j < 32; j++) {
                if (j < nv) {
                    const float v = __uint_as_float(r[j]);
                    if (EPI == GEMM_RESID) c[j] += v;
                    else c[j] = v;
                }
            }
        }
    } else {  // GEMM_GLU: columns 8t..8t+3 gate, 8t+4..8t+7 up of outputs 4t..4t+3
        __half* h = p.h + (size_t)row * p.ldh + col / 2;
        if (col + 32 <= p.N && (p.ldh & 7) == 0 && (reinterpret_cast<uintptr_t>(p.h) & 15) == 0) {
            __align__(16) __half o[16];
#pragma unroll
            for (int t = 0; t < 4; t++)
#pragma unroll
                for (int i = 0; i < 4; i++)
                    o[4 * t + i] = __float2half_rn(glu_mul(p.geglu, __uint_as_float(r[8 * t + i]), __uint_as_float(r[8 * t + 4 + i])));
            reinterpret_cast<uint4*>(h)[0] = reinterpret_cast<const uint4*>(o)[0];
            reinterpret_cast<uint4*>(h)[1] = reinterpret_cast<const uint4*>(o)[1];
        } else {
#pragma unroll
            for (int t = 0; t < 4; t++)
#pragma unroll
                for (int i = 0; i < 4; i++)
                    if (col + 8 * t + 4 + i < p.N)
                        h[4 * t + i] =
                            __float2half_rn(glu_mul(p.geglu, __uint_as_float(r[8 * t + i]), __uint_as_float(r[8 * t + 4 + i])));
        }
    }
}

}  // namespace tptc
