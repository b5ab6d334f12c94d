// act.cuh -- writing a prepared GEMV activation (ActLayout, gemv.cuh) one 256-element block
// at a time; shared by the activation kernel and kernels that produce a GEMV input in their
// epilogue (the attention kernel for the o projection).
#pragma once

#include "gemv.cuh"
#include "quant.cuh"

namespace tptc {

// Block b (elements 256b .. +255, lane holding 8b' = 8*lane .. +7 in v) of an activation of
// nb blocks into `out` with layout L: f32 copy, Q8_K (transposed = lane-transposed quants)
// and/or Q8_0, whichever parts L has.  All 32 lanes of the warp call it.
__device__ __forceinline__ void act_store_block(const ActLayout& L, int transposed, int nb, uint8_t* out, int b,
                                                const float (&v)[8], int lane) {
    if (L.f32 >= 0) {
        float4* dst = reinterpret_cast<float4*>(out + L.f32 + (size_t)(b * QK_K + 8 * lane) * 4);
        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (L.q8k >= 0) {
        const float(&vv)[1][8] = *reinterpret_cast<const float(*)[1][8]>(&v);
        uint32_t q[1][2];
        int s16[1], s32[1];
        float d[1];
        q8k_quant_regs<1>(vv, q, s16, s32, d, lane);
        const int oq = transposed ? xt_offset(b, lane, nb, L.cbs) : b * QK_K + 8 * lane;
        *reinterpret_cast<uint2*>(out + L.q8k + oq) = make_uint2(q[0][0], q[0][1]);
        if ((lane & 1) == 0) reinterpret_cast<int16_t*>(out + L.q8k_bs)[b * 16 + (lane >> 1)] = (int16_t)s16[0];
        if ((lane & 3) == 0) reinterpret_cast<int16_t*>(out + L.q8k_ps)[b * 8 + (lane >> 2)] = (int16_t)s32[0];
        if (lane == 0) reinterpret_cast<float*>(out + L.q8k_d)[b] = d[0];
    }
    if (L.q80 >= 0) {
        uint32_t q[2];
        float d;
        q80_quant_lane8(v, q, d);
        *reinterpret_cast<uint2*>(out + L.q80 + b * QK_K + 8 * lane) = make_uint2(q[0], q[1]);
        if ((lane & 3) == 0) reinterpret_cast<float*>(out + L.q80_d)[b * 8 + (lane >> 2)] = h2f(f2h(d));
    }
}

// NB blocks at once (their quantisation reductions interleaved): block b[k] from v[k]; blocks
// with b[k] >= nb are skipped (their registers may hold anything finite).
template <int NB>
__device__ __forceinline__ void act_store_blocks(const ActLayout& L, int transposed, int nb, uint8_t* out,
                                                 const int (&b)[NB], const float (&v)[NB][8], int lane) {
    if (L.f32 >= 0) {
#pragma unroll
        for (int k = 0; k < NB; k++) {
            if (b[k] >= nb) continue;
            float4* dst = reinterpret_cast<float4*>(out + L.f32 + (size_t)(b[k] * QK_K + 8 * lane) * 4);
            dst[0] = make_float4(v[k][0], v[k][1], v[k][2], v[k][3]);
            dst[1] = make_float4(v[k][4], v[k][5], v[k][6], v[k][7]);
        }
    }
    if (L.q8k >= 0) {
        uint32_t q[NB][2];
        int s16[NB], s32[NB];
        float d[NB];
        q8k_quant_regs<NB>(v, q, s16, s32, d, lane);
#pragma unroll
        for (int k = 0; k < NB; k++) {
            if (b[k] >= nb) continue;
            const int oq = transposed ? xt_offset(b[k], lane, nb, L.cbs) : b[k] * QK_K + 8 * lane;
            *reinterpret_cast<uint2*>(out + L.q8k + oq) = make_uint2(q[k][0], q[k][1]);
            if ((lane & 1) == 0) reinterpret_cast<int16_t*>(out + L.q8k_bs)[b[k] * 16 + (lane >> 1)] = (int16_t)s16[k];
            if ((lane & 3) == 0) reinterpret_cast<int16_t*>(out + L.q8k_ps)[b[k] * 8 + (lane >> 2)] = (int16_t)s32[k];
            if (lane == 0) reinterpret_cast<float*>(out + L.q8k_d)[b[k]] = d[k];
        }
    }
    if (L.q80 >= 0) {
#pragma unroll
        for (int k = 0; k < NB; k++) {
            if (b[k] >= nb) continue;
            uint32_t q[2];
            float d;
            q80_quant_lane8(v[k], q, d);
            *reinterpret_cast<uint2*>(out + L.q80 + b[k] * QK_K + 8 * lane) = make_uint2(q[0], q[1]);
            if ((lane & 3) == 0) reinterpret_cast<float*>(out + L.q80_d)[b[k] * 8 + (lane >> 2)] = h2f(f2h(d));
        }
    }
}

// Sum of squares of a lane's 8 elements as an explicit multiply-add chain (the same
// instructions wherever it is inlined, so every kernel that normalises a vector this way gets
// the same m).
__device__ __forceinline__ float sumsq8(const float (&v)[8]) {
    float s = __fmul_rn(v[0], v[0]);
#pragma unroll
    for (int i = 1; i < 8; i++) s = __fmaf_rn(v[i], v[i], s);
    return s;
}

// RMSNorm partition shared by the activation kernel and the GEMV chains: 8 warps, warp w
// holding 256-blocks w, w + 8, ... (lane l: elements 8l .. 8l+7 of each), a thread's blocks
// summed in order, the warp by xor butterfly, then the 8 warp sums in warp order.
constexpr int kNormWarps = 8;

}  // namespace tptc
