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

}  // namespace tptc
