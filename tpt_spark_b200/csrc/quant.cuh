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
#include "gemv.cuh"

namespace tptc {

// Q8_K quantisation of NB 256-element blocks held in registers across a warp: for block k,
// lane holds x[k][0..7] = elements 8*lane .. 8*lane+7.  Per block the lane receives its 8
// int8 quants packed in q[k][0..1], the sum of 16 elements s16[k] (bsum lane/2, equal in
// both lanes of a pair), the sum of 32 elements s32[k] (sub-block lane/4, equal in its 4
// lanes) and the block scale d[k] (every lane).  The blocks are independent, so their
// reduction chains overlap.  The largest |x| and its first index come from the hardware
// warp reductions (non-negative floats order like their bit patterns).  Integer results are
// bit-exact with candle.
template <int NB>
__device__ __forceinline__ void q8k_quant_regs(const float (&x)[NB][8], uint32_t (&q)[NB][2], int (&s16)[NB],
                                               int (&s32)[NB], float (&d)[NB], int lane) {
    uint32_t amax_bits[NB];
#pragma unroll
    for (int k = 0; k < NB; k++) {
        uint32_t a = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) a = max(a, __float_as_uint(fabsf(x[k][i])));
        amax_bits[k] = __reduce_max_sync(0xffffffffu, a);
    }
    float vmax[NB];
#pragma unroll
    for (int k = 0; k < NB; k++) {
        uint32_t first = 0xffffffffu;
        float v = 0.f;
#pragma unroll
        for (int i = 7; i >= 0; i--)
            if (__float_as_uint(fabsf(x[k][i])) == amax_bits[k]) {
                first = (uint32_t)(lane * 8 + i);
                v = x[k][i];
            }
        const uint32_t imin = __reduce_min_sync(0xffffffffu, first);
        vmax[k] = __shfl_sync(0xffffffffu, v, (int)(imin >> 3) & 31);
    }
#pragma unroll
    for (int k = 0; k < NB; k++) {
        int s = 0;
        q[k][0] = q[k][1] = 0;
        d[k] = 0.f;
        if (amax_bits[k] != 0) {
            const float iscale = __fdiv_rn(-128.f, vmax[k]);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int qi = (int)static_cast<int8_t>(fminf(roundf(__fmul_rn(iscale, x[k][i])), 127.f));
                q[k][i >> 2] |= (uint32_t)(qi & 0xff) << (8 * (i & 3));
                s += qi;
            }
            d[k] = __fdiv_rn(1.f, iscale);
        }
        s16[k] = s + __shfl_xor_sync(0xffffffffu, s, 1);
        s32[k] = s16[k] + __shfl_xor_sync(0xffffffffu, s16[k], 2);
    }
}

// One block into a block_q8_K-style destination: qs_lane = this lane's 8 quants (4-byte
// aligned), 16 bsums, d.
__device__ __forceinline__ void q8k_quant_warp(const float (&x)[8], int8_t* qs_lane, int16_t* bsums_dst,
                                               float* d_dst, int lane) {
    const float(&xx)[1][8] = *reinterpret_cast<const float(*)[1][8]>(&x);
    uint32_t q[1][2];
    int s16[1], s32[1];
    float d[1];
    q8k_quant_regs<1>(xx, q, s16, s32, d, lane);
    reinterpret_cast<uint32_t*>(qs_lane)[0] = q[0][0];
    reinterpret_cast<uint32_t*>(qs_lane)[1] = q[0][1];
    if ((lane & 1) == 0) bsums_dst[lane >> 1] = static_cast<int16_t>(s16[0]);
    if (lane == 0) *d_dst = d[0];
}

// Quantise one 32-element block to Q8_0 across a warp (lane = element).  Returns the
// int8 value; every lane receives the f32 scale `d` (stored as f16 by the caller).
__device__ __forceinline__ int8_t q80_quant_warp(float x, float& d) {
    float amax = warp_max(fabsf(x));
    d = __fdiv_rn(amax, 127.f);
    float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
    return static_cast<int8_t>(roundf(__fmul_rn(x, id)));
}

// Q8_0 of eight 32-element blocks held across a warp as in q8k_quant_regs (lane holds
// elements 8*lane .. +7, so block lane/4): the lane's 8 int8 quants packed in q[0..1] and the
// block's f32 scale d (before f16 storage) in every lane of the block.
__device__ __forceinline__ void q80_quant_lane8(const float (&x)[8], uint32_t (&q)[2], float& d) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(x[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    d = __fdiv_rn(amax, 127.f);
    const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
    q[0] = q[1] = 0;
#pragma unroll
    for (int i = 0; i < 8; i++)
        q[i >> 2] |= (uint32_t)(uint8_t)static_cast<int8_t>(roundf(__fmul_rn(x[i], id))) << (8 * (i & 3));
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

// Element e (0..31) of the 32-element formats (gguf-py Q4_0 / Q4_1 / Q5_0 / Q5_1): the
// 4-bit value is the low nibble of qs[e] for e < 16, the high nibble of qs[e - 16] above;
// Q5_* add bit e of the little-endian qh word as the 5th bit.  Q4_0: d*(q-8), Q5_0: d*(q-16),
// Q4_1 / Q5_1: (d*q) + m.
__device__ __forceinline__ int q4_nibble(const uint8_t* qs, int e) {
    return e < 16 ? (qs[e] & 0x0f) : (qs[e - 16] >> 4);
}
__device__ __forceinline__ int q5_hbit(const uint8_t* qh, int e) { return (qh[e >> 3] >> (e & 7)) & 1; }
__device__ __forceinline__ float q40_elem(const uint8_t* blk, int e) {
    return __fmul_rn(h2f(blk[0] | (blk[1] << 8)), (float)(q4_nibble(blk + 2, e) - 8));
}
__device__ __forceinline__ float q41_elem(const uint8_t* blk, int e) {
    return __fadd_rn(__fmul_rn(h2f(blk[0] | (blk[1] << 8)), (float)q4_nibble(blk + 4, e)), h2f(blk[2] | (blk[3] << 8)));
}
__device__ __forceinline__ float q50_elem(const uint8_t* blk, int e) {
    const int q = q4_nibble(blk + 6, e) | (q5_hbit(blk + 2, e) << 4);
    return __fmul_rn(h2f(blk[0] | (blk[1] << 8)), (float)(q - 16));
}
__device__ __forceinline__ float q51_elem(const uint8_t* blk, int e) {
    const int q = q4_nibble(blk + 8, e) | (q5_hbit(blk + 4, e) << 4);
    return __fadd_rn(__fmul_rn(h2f(blk[0] | (blk[1] << 8)), (float)q), h2f(blk[2] | (blk[3] << 8)));
}

// Element e (0..255) of a Q2_K block (gguf-py Q2_K): e = 128h + 32s + l takes bits 2s of
// qs[32h + l]; the 16-element group e / 16 has scale byte sc | m << 4:
// (d*sc)*q - (dmin*m).
__device__ __forceinline__ float q2k_elem(const uint8_t* blk, int e) {
    const int h = e >> 7, sh = (e >> 5) & 3, l = e & 31, g = e >> 4;
    const int q = (blk[16 + 32 * h + l] >> (2 * sh)) & 3;
    const float d = h2f(blk[80] | (blk[81] << 8)), dmin = h2f(blk[82] | (blk[83] << 8));
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)(blk[g] & 0x0f)), (float)q), __fmul_rn(dmin, (float)(blk[g] >> 4)));
}

// Element e of a Q3_K block (gguf-py Q3_K): 2 low bits as Q2_K, minus 4 where bit e / 32 of
// hmask[e % 32] is clear; 16-element group scales of 6 bits (low 4 from scales[k % 8], nibble
// k / 8; high 2 from scales[8 + k % 4], bits 2 (k / 4)) minus 32: (d*scale)*q.
__device__ __forceinline__ float q3k_elem(const uint8_t* blk, int e) {
    const int h = e >> 7, sh = (e >> 5) & 3, l = e & 31, k = e >> 4;
    const int ql = (blk[32 + 32 * h + l] >> (2 * sh)) & 3;
    const int hb = (blk[l] >> (e >> 5)) & 1;
    const uint8_t* sc = blk + 96;
    const int scale = (((sc[k & 7] >> (4 * (k >> 3))) & 0x0f) | (((sc[8 + (k & 3)] >> (2 * (k >> 2))) & 3) << 4)) - 32;
    return __fmul_rn(__fmul_rn(h2f(blk[108] | (blk[109] << 8)), (float)scale), (float)(ql - ((hb ^ 1) << 2)));
}

// Element e of a Q5_K block (gguf-py Q5_K): Q4_K's scales and nibbles, plus bit e / 32 of
// qh[e % 32] as the 5th bit: (d*sc)*q - (dmin*m).
__device__ __forceinline__ float q5k_elem(const uint8_t* blk, int e) {
    const int g = e >> 6, j = e >> 5, l = e & 31;
    int sc, m;
    q4k_scale_min(blk + 4, j, sc, m);
    const uint8_t b = blk[48 + 32 * g + l];
    const int q = ((j & 1) ? (b >> 4) : (b & 0x0f)) | (((blk[16 + l] >> j) & 1) << 4);
    const float d = h2f(blk[0] | (blk[1] << 8)), dmin = h2f(blk[2] | (blk[3] << 8));
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

// Element i (0 .. K-1) of physical row `prow` of a matrix in the device layout, with the
// value (and rounding) of the raw-block dequantisation above.
__device__ __forceinline__ float dm_elem(const DevMatrix& m, int prow, int i) {
    const int sb = i / QK_K, e = i % QK_K;
    const uint8_t* blk = dm_block(m, prow, sb);
    switch (m.type) {
    case TPTC_TYPE_Q4_K: return q4k_elem(blk, e);
    case TPTC_TYPE_Q5_K: return q5k_elem(blk, e);
    case TPTC_TYPE_Q6_K: return q6k_elem(blk, h2f(dm_scales(m, prow, sb)[0]), e);
    case TPTC_TYPE_Q8_0:
        return __fmul_rn((float)(int8_t)blk[e], h2f(dm_scales(m, prow, sb)[e / QK8_0]));
    case TPTC_TYPE_Q2_K: {  // device: qs[64] | scales[16]; d, dmin in the scale section
        const uint16_t* dd = dm_scales(m, prow, sb);
        const int q = (blk[32 * (e >> 7) + (e & 31)] >> (2 * ((e >> 5) & 3))) & 3, g = blk[64 + (e >> 4)];
        return __fsub_rn(__fmul_rn(__fmul_rn(h2f(dd[0]), (float)(g & 0x0f)), (float)q),
                         __fmul_rn(h2f(dd[1]), (float)(g >> 4)));
    }
    case TPTC_TYPE_Q3_K: {  // device: hmask[32] | qs[64]; scales[12] and d in the scale section
        const uint8_t* sc = reinterpret_cast<const uint8_t*>(dm_scales(m, prow, sb));
        const int h = e >> 7, sh = (e >> 5) & 3, l = e & 31, k = e >> 4;
        const int ql = (blk[32 + 32 * h + l] >> (2 * sh)) & 3;
        const int hb = (blk[l] >> (e >> 5)) & 1;
        const int scale =
            (((sc[k & 7] >> (4 * (k >> 3))) & 0x0f) | (((sc[8 + (k & 3)] >> (2 * (k >> 2))) & 3) << 4)) - 32;
        return __fmul_rn(__fmul_rn(h2f(sc[12] | (sc[13] << 8)), (float)scale), (float)(ql - ((hb ^ 1) << 2)));
    }
    case TPTC_TYPE_Q4_0: {
        const int j = e / QK8_0;
        return __fmul_rn(h2f(dm_scales(m, prow, sb)[j]), (float)(q4_nibble(blk + 16 * j, e % QK8_0) - 8));
    }
    case TPTC_TYPE_Q5_0: {
        const int j = e / QK8_0, l = e % QK8_0;
        const int q = q4_nibble(blk + 16 * j, l) | (q5_hbit(blk + 128 + 4 * j, l) << 4);
        return __fmul_rn(h2f(dm_scales(m, prow, sb)[j]), (float)(q - 16));
    }
    case TPTC_TYPE_Q4_1:
    case TPTC_TYPE_Q5_1: {
        const int j = e / QK8_0, l = e % QK8_0;
        int q = q4_nibble(blk + 16 * j, l);
        if (m.type == TPTC_TYPE_Q5_1) q |= q5_hbit(blk + 128 + 4 * j, l) << 4;
        const uint16_t* dm = dm_scales(m, prow, sb) + 2 * j;
        return __fadd_rn(__fmul_rn(h2f(dm[0]), (float)q), h2f(dm[1]));
    }
    }
    return h2f(reinterpret_cast<const uint16_t*>(blk)[e]);
}

}  // namespace tptc
