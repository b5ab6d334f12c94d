// quant.cu -- standalone block kernels: dequantisation of raw GGUF blocks (the reference's
// dequant_q4k/q6k/q8/f16.wgsl entry points and its Q4_0 / Q5_0 / Q5_1 / Q2_K / Q3_K / Q5_K
// shaders, with the GGUF layouts of gguf-py rather than the reference's wrong nibble splits), activation quantisation to Q8_K / Q8_0, the load-time
// repack into the device layout, and the dense f16 expansion used by the prefill GEMM.
#include "kernels.h"
#include "quant.cuh"

namespace tptc {

namespace {

// One thread per element; raw GGUF blocks.
__global__ void dequant_raw_kernel(int type, const uint8_t* __restrict__ blocks, int64_t n, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v;
    if (type == TPTC_TYPE_Q4_K) {
        v = q4k_elem(blocks + (i / QK_K) * Q4K_BYTES, (int)(i % QK_K));
    } else if (type == TPTC_TYPE_Q6_K) {
        const uint8_t* blk = blocks + (i / QK_K) * Q6K_BYTES;
        v = q6k_elem(blk, h2f(blk[208] | (blk[209] << 8)), (int)(i % QK_K));
    } else if (type == TPTC_TYPE_Q8_0) {
        const uint8_t* blk = blocks + (i / QK8_0) * Q80_BYTES;
        v = __fmul_rn((float)(int8_t)blk[2 + i % QK8_0], h2f(blk[0] | (blk[1] << 8)));
    } else if (type == TPTC_TYPE_F16) {
        v = h2f(reinterpret_cast<const uint16_t*>(blocks)[i]);
    } else if (type == TPTC_TYPE_Q4_0) {
        v = q40_elem(blocks + (i / 32) * Q40_BYTES, (int)(i % 32));
    } else if (type == TPTC_TYPE_Q4_1) {
        v = q41_elem(blocks + (i / 32) * Q41_BYTES, (int)(i % 32));
    } else if (type == TPTC_TYPE_Q5_0) {
        v = q50_elem(blocks + (i / 32) * Q50_BYTES, (int)(i % 32));
    } else if (type == TPTC_TYPE_Q5_1) {
        v = q51_elem(blocks + (i / 32) * Q51_BYTES, (int)(i % 32));
    } else if (type == TPTC_TYPE_Q2_K) {
        v = q2k_elem(blocks + (i / QK_K) * Q2K_BYTES, (int)(i % QK_K));
    } else if (type == TPTC_TYPE_Q3_K) {
        v = q3k_elem(blocks + (i / QK_K) * Q3K_BYTES, (int)(i % QK_K));
    } else if (type == TPTC_TYPE_Q5_K) {
        v = q5k_elem(blocks + (i / QK_K) * Q5K_BYTES, (int)(i % QK_K));
    } else {
        v = reinterpret_cast<const float*>(blocks)[i];
    }
    out[i] = v;
}

// One warp per 256-element block.
__global__ void quant_q8k_kernel(const float* __restrict__ x, int64_t nb, BlockQ8K* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (b >= nb) return;
    float v[8];
    const float4* src = reinterpret_cast<const float4*>(x + b * QK_K + lane * 8);
    const float4 a = src[0], c = src[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    q8k_quant_warp(v, out[b].qs + 8 * lane, out[b].bsums, &out[b].d, lane);
}

// One warp per 32-element block; output 34-byte blocks (f16 d, int8 qs[32]).
__global__ void quant_q80_kernel(const float* __restrict__ x, int64_t nb, uint8_t* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (b >= nb) return;
    float d;
    const int8_t q = q80_quant_warp(x[b * QK8_0 + lane], d);
    uint8_t* blk = out + b * Q80_BYTES;  // 34-byte blocks: 2-byte aligned
    blk[2 + lane] = (uint8_t)q;
    if (lane == 0) *reinterpret_cast<uint16_t*>(blk) = f2h(d);
}

// Raw GGUF rows -> tiled device layout, one thread per 256-element super-block.  `nr` raw
// rows (raw_row bytes apart) become logical rows first_row .. first_row + nr - 1 of `m`.
__global__ void repack_kernel(const uint8_t* __restrict__ raw, int64_t raw_row, int nr, int first_row, DevMatrix m) {
    const int nsb = m.K / QK_K;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)nr * nsb) return;
    const int r = (int)(i / nsb), sb = (int)(i % nsb);
    const int prow = dm_phys_row(m, first_row + r);
    uint8_t* dst = const_cast<uint8_t*>(dm_block(m, prow, sb));
    const uint8_t* row = raw + (int64_t)r * raw_row;
    if (m.type == TPTC_TYPE_Q4_K) {
        const uint8_t* src = row + (int64_t)sb * Q4K_BYTES;
        for (int k = 0; k < Q4K_BYTES; k++) dst[k] = src[k];
    } else if (m.type == TPTC_TYPE_Q6_K) {
        const uint8_t* src = row + (int64_t)sb * Q6K_BYTES;
        for (int k = 0; k < Q6K_MAIN; k++) dst[k] = src[k];
        const_cast<uint16_t*>(dm_scales(m, prow, sb))[0] = (uint16_t)(src[208] | (src[209] << 8));
    } else if (m.type == TPTC_TYPE_Q8_0) {
        uint16_t* dsc = const_cast<uint16_t*>(dm_scales(m, prow, sb));
        for (int j = 0; j < 8; j++) {
            const uint8_t* src = row + ((int64_t)sb * 8 + j) * Q80_BYTES;
            for (int k = 0; k < 32; k++) dst[32 * j + k] = src[2 + k];
            dsc[j] = (uint16_t)(src[0] | (src[1] << 8));
        }
    } else if (m.type == TPTC_TYPE_Q5_K) {
        const uint8_t* src = row + (int64_t)sb * Q5K_BYTES;
        for (int k = 0; k < Q5K_BYTES; k++) dst[k] = src[k];
    } else if (m.type == TPTC_TYPE_Q2_K) {  // scales[16] qs[64] d dmin -> qs | scales, (d, dmin)
        const uint8_t* src = row + (int64_t)sb * Q2K_BYTES;
        for (int k = 0; k < 64; k++) dst[k] = src[16 + k];
        for (int k = 0; k < 16; k++) dst[64 + k] = src[k];
        uint8_t* dsc = reinterpret_cast<uint8_t*>(const_cast<uint16_t*>(dm_scales(m, prow, sb)));
        for (int k = 0; k < 4; k++) dsc[k] = src[80 + k];
    } else if (m.type == TPTC_TYPE_Q3_K) {  // hmask[32] qs[64] | scales[12] d
        const uint8_t* src = row + (int64_t)sb * Q3K_BYTES;
        for (int k = 0; k < 96; k++) dst[k] = src[k];
        uint8_t* dsc = reinterpret_cast<uint8_t*>(const_cast<uint16_t*>(dm_scales(m, prow, sb)));
        for (int k = 0; k < 14; k++) dsc[k] = src[96 + k];
    } else if (m.type == TPTC_TYPE_Q4_0) {
        uint16_t* dsc = const_cast<uint16_t*>(dm_scales(m, prow, sb));
        for (int j = 0; j < 8; j++) {
            const uint8_t* src = row + ((int64_t)sb * 8 + j) * Q40_BYTES;
            for (int k = 0; k < 16; k++) dst[16 * j + k] = src[2 + k];
            dsc[j] = (uint16_t)(src[0] | (src[1] << 8));
        }
    } else if (m.type == TPTC_TYPE_Q5_0) {
        uint16_t* dsc = const_cast<uint16_t*>(dm_scales(m, prow, sb));
        for (int j = 0; j < 8; j++) {
            const uint8_t* src = row + ((int64_t)sb * 8 + j) * Q50_BYTES;
            for (int k = 0; k < 16; k++) dst[16 * j + k] = src[6 + k];
            for (int k = 0; k < 4; k++) dst[128 + 4 * j + k] = src[2 + k];
            dsc[j] = (uint16_t)(src[0] | (src[1] << 8));
        }
    } else if (m.type == TPTC_TYPE_Q4_1 || m.type == TPTC_TYPE_Q5_1) {  // d m [qh] qs -> qs | [qh], (d, m)
        const bool five = m.type == TPTC_TYPE_Q5_1;
        uint16_t* dsc = const_cast<uint16_t*>(dm_scales(m, prow, sb));
        for (int j = 0; j < 8; j++) {
            const uint8_t* src = row + ((int64_t)sb * 8 + j) * (five ? Q51_BYTES : Q41_BYTES);
            for (int k = 0; k < 16; k++) dst[16 * j + k] = src[(five ? 8 : 4) + k];
            if (five)
                for (int k = 0; k < 4; k++) dst[128 + 4 * j + k] = src[4 + k];
            dsc[2 * j] = (uint16_t)(src[0] | (src[1] << 8));
            dsc[2 * j + 1] = (uint16_t)(src[2] | (src[3] << 8));
        }
    } else {
        const uint8_t* src = row + (int64_t)sb * 512;
        for (int k = 0; k < 512; k++) dst[k] = src[k];
    }
}

// Device layout -> dense f16 rows [row0, row0 + rows), one thread per 32-element group (a
// Q4_K sub-block, half a Q6_K 16-pair, a Q8_0 block): the group's scales are decoded once,
// its quant bytes read as 16-byte vectors and the 64 output bytes written as four 16-byte
// stores.  Values are those of q4k_elem / q6k_elem / the Q8_0 product, rounded to fp16.
__global__ void dequant_rows_f16_kernel(DevMatrix m, int row0, int rows, int physical, __half* __restrict__ out) {
    const int64_t per_row = m.K / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= per_row * rows) return;
    const int r = (int)(i / per_row), k0 = (int)(i % per_row) * 32;
    const int prow = physical ? row0 + r : dm_phys_row(m, row0 + r);
    const int sb = k0 / QK_K, e0 = k0 % QK_K, j = e0 / 32;
    const uint8_t* blk = dm_block(m, prow, sb);
    __align__(16) __half v[32];
    if (m.type == TPTC_TYPE_F16) {
#pragma unroll
        for (int k = 0; k < 4; k++)
            reinterpret_cast<uint4*>(v)[k] = reinterpret_cast<const uint4*>(blk + e0 * 2)[k];
    } else if (m.type == TPTC_TYPE_Q4_K) {
        // sub-block j: low (j even) or high (j odd) nibbles of qs[32 (j/2) .. +32)
        int sc, mn;
        q4k_scale_min(blk + 4, j, sc, mn);
        const float d = h2f(blk[0] | (blk[1] << 8)), dmin = h2f(blk[2] | (blk[3] << 8));
        const float ds = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)mn);
        const uint4* qv = reinterpret_cast<const uint4*>(blk + 16 + 32 * (j >> 1));
        const int sh = (j & 1) * 4;
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const uint4 w = qv[k];
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int b = 0; b < 16; b++) {
                const int q = (ww[b >> 2] >> (8 * (b & 3) + sh)) & 0x0f;
                v[16 * k + b] = __float2half_rn(__fsub_rn(__fmul_rn(ds, (float)q), dm));
            }
        }
    } else if (m.type == TPTC_TYPE_Q6_K) {
        // elements 128h + 32i + l: ql[64h + 32 (i & 1) + l] nibble (i & 2), qh[32h + l] bits 2i
        const int h = j >> 2, ii = j & 3;
        const float d = h2f(dm_scales(m, prow, sb)[0]);
        const int8_t* scs = reinterpret_cast<const int8_t*>(blk + 192);
        const float ds0 = __fmul_rn(d, (float)scs[(e0 >> 4)]), ds1 = __fmul_rn(d, (float)scs[(e0 >> 4) + 1]);
        const uint4* qlv = reinterpret_cast<const uint4*>(blk + 64 * h + 32 * (ii & 1));
        const uint4* qhv = reinterpret_cast<const uint4*>(blk + 128 + 32 * h);
        const int lsh = (ii & 2) ? 4 : 0, hsh = 2 * ii;
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const uint4 a = qlv[k], hb = qhv[k];
            const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, hh[4] = {hb.x, hb.y, hb.z, hb.w};
#pragma unroll
            for (int b = 0; b < 16; b++) {
                const int lo = (aa[b >> 2] >> (8 * (b & 3) + lsh)) & 0x0f;
                const int hi = (hh[b >> 2] >> (8 * (b & 3) + hsh)) & 0x03;
                const int q = (lo | (hi << 4)) - 32;
                v[16 * k + b] = __float2half_rn(__fmul_rn(k == 0 ? ds0 : ds1, (float)q));
            }
        }
    } else if (m.type == TPTC_TYPE_Q8_0) {
        const int8_t* q = reinterpret_cast<const int8_t*>(blk + e0);
        const float d = h2f(dm_scales(m, prow, sb)[e0 / QK8_0]);
#pragma unroll
        for (int b = 0; b < 32; b++) v[b] = __float2half_rn(__fmul_rn((float)q[b], d));
    } else {
        // Q2_K, Q3_K, Q5_K, Q4_0, Q5_0, Q4_1, Q5_1: the element values of dm_elem (one group of
        // 32, rounded to fp16)
#pragma unroll 8
        for (int b = 0; b < 32; b++) v[b] = __float2half_rn(dm_elem(m, prow, k0 + b));
    }
    uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)r * m.K + k0);
#pragma unroll
    for (int k = 0; k < 4; k++) dst[k] = reinterpret_cast<const uint4*>(v)[k];
}

}  // namespace

cudaError_t launch_dequant_raw(int type, const void* blocks, int64_t n, float* out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int t = 256;
    dequant_raw_kernel<<<(unsigned)ceil_div64(n, t), t, 0, st>>>(type, static_cast<const uint8_t*>(blocks), n, out);
    return cudaGetLastError();
}

cudaError_t launch_quant_q8k(const float* x, int64_t k, void* out, cudaStream_t st) {
    const int64_t nb = k / QK_K;
    if (nb <= 0) return cudaSuccess;
    quant_q8k_kernel<<<(unsigned)ceil_div64(nb, 8), 256, 0, st>>>(x, nb, static_cast<BlockQ8K*>(out));
    return cudaGetLastError();
}

cudaError_t launch_quant_q80(const float* x, int64_t k, void* out, cudaStream_t st) {
    const int64_t nb = k / QK8_0;
    if (nb <= 0) return cudaSuccess;
    quant_q80_kernel<<<(unsigned)ceil_div64(nb, 8), 256, 0, st>>>(x, nb, static_cast<uint8_t*>(out));
    return cudaGetLastError();
}

cudaError_t launch_repack(const uint8_t* raw, int64_t raw_row, int nr, int first_row, const DevMatrix& m,
                          cudaStream_t st) {
    const int64_t n = (int64_t)nr * (m.K / QK_K);
    if (n <= 0) return cudaSuccess;
    repack_kernel<<<(unsigned)ceil_div64(n, 128), 128, 0, st>>>(raw, raw_row, nr, first_row, m);
    return cudaGetLastError();
}

cudaError_t launch_dequant_rows_f16(const DevMatrix& m, int row0, int rows, __half* out, cudaStream_t st,
                                    bool physical) {
    const int64_t n = (int64_t)rows * (m.K / 32);
    if (n <= 0) return cudaSuccess;
    dequant_rows_f16_kernel<<<(unsigned)ceil_div64(n, 128), 128, 0, st>>>(m, row0, rows, physical ? 1 : 0, out);
    return cudaGetLastError();
}

}  // namespace tptc
