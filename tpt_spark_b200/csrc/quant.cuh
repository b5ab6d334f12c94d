// quant.cuh -- device functions for GGUF block formats and activation quantisation.
//
// Dequantisation rounds exactly as gguf-py's numpy code and candle's Rust code do (one
// rounding per operation, no FMA contraction), so f32 results are bit-identical.
// Activation quantisation restates candle 0.8.4 k_quants:
//   BlockQ8K::from_float  -- signed value of the first element of largest magnitude `max`,
//                            iscale = -128/max, q = min(127, round(iscale*x)),
//                            d = 1/iscale, bsums over 16 elements;
//   BlockQ8_0::from_float -- d = amax/127, q = round(x * (1/d)), d stored as f16.
// round() is half away from zero (roundf), matching f32::round.
#pragma once

#include "common.cuh"

namespace tptc {

// Quantise one 256-element block held in registers across a warp: lane holds x[8*lane ..
// 8*lane+7].  Writes the lane's 8 int8 quants to qs_lane (4-byte aligned; the caller picks
// the layout), d via *d_dst (lane 0) and the 16 bsums (lanes with lane%2==0 own bsum
// lane/2).  Integer results are bit-exact with candle.
__device__ __forceinline__ void q8k_quant_warp(const float (&x)[8], int8_t* qs_lane, int16_t* bsums_dst,
                                               float* d_dst, int lane) {
    // first index of the largest |x| and its signed value
    float amax = 0.f, vmax = 0.f;
    int imax = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float a = fabsf(x[i]);
        if (a > amax) {
            amax = a;
            vmax = x[i];
            imax = lane * 8 + i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float a2 = __shfl_xor_sync(0xffffffffu, amax, o);
        float v2 = __shfl_xor_sync(0xffffffffu, vmax, o);
        int i2 = __shfl_xor_sync(0xffffffffu, imax, o);
        if (a2 > amax || (a2 == amax && i2 < imax)) {
            amax = a2;
            vmax = v2;
            imax = i2;
        }
    }
    int8_t q[8];
    int s = 0;
    float d = 0.f;
    if (amax == 0.f) {
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = 0;
    } else {
        float iscale = __fdiv_rn(-128.f, vmax);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float v = roundf(__fmul_rn(iscale, x[i]));
            q[i] = static_cast<int8_t>(fminf(v, 127.f));
            s += q[i];
        }
        d = __fdiv_rn(1.f, iscale);
    }
    uint32_t w0 = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) | ((uint32_t)(uint8_t)q[2] << 16) |
                  ((uint32_t)(uint8_t)q[3] << 24);
    uint32_t w1 = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) | ((uint32_t)(uint8_t)q[6] << 16) |
                  ((uint32_t)(uint8_t)q[7] << 24);
    // 4-byte stores: in a block_q8_K array, qs starts at 4 + 292*b (4-byte aligned only)
    reinterpret_cast<uint32_t*>(qs_lane)[0] = w0;
    reinterpret_cast<uint32_t*>(qs_lane)[1] = w1;
    int s2 = s + __shfl_xor_sync(0xffffffffu, s, 1);
    if ((lane & 1) == 0) bsums_dst[lane >> 1] = static_cast<int16_t>(s2);
    if (lane == 0) *d_dst = d;
}

// Quantise one 32-element block to Q8_0 across a warp (lane = element).  Returns the
// int8 value; every lane receives the f32 scale `d` (stored as f16 by the caller).
__device__ __forceinline__ int8_t q80_quant_warp(float x, float& d) {
    float amax = warp_max(fabsf(x));
    d = __fdiv_rn(amax, 127.f);
    float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
    return static_cast<int8_t>(roundf(__fmul_rn(x, id)));
}

// Q8_0 of eight 32-element blocks held across a warp as in q8k_quant_warp (lane holds
// elements 8*lane .. +7, so block lane/4): writes the lane's 8 int8 quants to qs_lane and
// returns the block's f32 scale d (before f16 storage) in every lane of the block.
__device__ __forceinline__ void q80_quant_lane8(const float (&x)[8], int8_t* qs_lane, float& d) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(x[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    d = __fdiv_rn(amax, 127.f);
    const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
    uint32_t w[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; i++)
        w[i >> 2] |= (uint32_t)(uint8_t)static_cast<int8_t>(roundf(__fmul_rn(x[i], id))) << (8 * (i & 3));
    reinterpret_cast<uint32_t*>(qs_lane)[0] = w[0];
    reinterpret_cast<uint32_t*>(qs_lane)[1] = w[1];
}

// ---- dequantisation of GGUF blocks (raw layout) ------------------------------------------

// Element e (0..255) of a Q4_K block: (d*sc)*q - (dmin*m).
__device__ __forceinline__ float q4k_elem(const uint8_t* blk, int e) {
    int g = e >> 6, r = e & 63, j = 2 * g + (r >> 5), l = r & 31;
    int sc, m;
    q4k_scale_min(blk + 4, j, sc, m);
    float d = h2f(blk[0] | (blk[1] << 8)), dmin = h2f(blk[2] | (blk[3] << 8));
    uint8_t b = blk[16 + 32 * g + l];
    int q = (r >> 5) ? (b >> 4) : (b & 0x0f);
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
}

// q-32 of element e of a Q6_K block whose ql / qh / scales start at `main`.
__device__ __forceinline__ int q6k_q(const uint8_t* main, int e) {
    int h = e >> 7, r = e & 127, i = r >> 5, l = r & 31;
    const uint8_t* ql = main + 64 * h;
    const uint8_t* qh = main + 128 + 32 * h;
    int lo = (i & 1) ? ql[l + 32] : ql[l];
    lo = (i & 2) ? (lo >> 4) : (lo & 0x0f);
    int hi = (qh[l] >> (2 * i)) & 3;
    return (lo | (hi << 4)) - 32;
}

__device__ __forceinline__ float q6k_elem(const uint8_t* main, float d, int e) {
    const int8_t* sc = reinterpret_cast<const int8_t*>(main + 192);
    return __fmul_rn(__fmul_rn(d, (float)sc[e >> 4]), (float)q6k_q(main, e));
}

}  // namespace tptc
