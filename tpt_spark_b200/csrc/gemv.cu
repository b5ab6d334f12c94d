// gemv.cu -- batch-1 dequant-fused GEMV for decode.
//
// Replaces the reference's per-matmul pair "dequantise the whole weight to f32, then a
// 16x16-tiled f32 GEMM with M=1" (shaders/dequant_q4k.wgsl:74-115, dequant_q6k.wgsl:58-92,
// dequant_q8.wgsl:51-73, dequant_f16.wgsl:30-37, gemm.wgsl:28-70, driven by
// engine/wgpu_engine.rs:581-605), with candle QMatMul semantics (candle_engine.rs:221,273):
// the activation is quantised to Q8_K (Q4_K/Q6_K weights) or Q8_0 (Q8_0 weights) and every
// super-block contributes (d_w*d_x)*isum - (dmin_w*d_x)*msum from exact integer sums.
//
// Kernel structure (one CTA = 8 warps = 8 weight rows):
//   1. thread 0 starts 1-D TMA bulk copies of the CTA's weight rows, chunk by chunk, into
//      a shared-memory ring (mbarrier completion, L2 evict-first) -- weights do not depend
//      on the previous kernel, so this runs before griddepcontrol.wait;
//   2. griddepcontrol.wait, then the CTA RMS-normalises (optional) and quantises the
//      activation into shared memory (every CTA computes the same bytes);
//   3. each warp reduces its row from the ring: dp4a integer dots per sub-block, exact
//      integer sums across the lanes of a super-block, one f32 FMA per super-block;
//   4. fused epilogue: store / residual add / RoPE + fp16 KV-cache write / SiLU(gate)*up.
#include <algorithm>

#include "gemv.cuh"
#include "quant.cuh"

namespace tptc {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxStages = 4;

struct WarpRow {
    int seg;    // -1: no row for this warp
    int row;
    int type;
    const uint8_t* main;
    const uint16_t* dplane;
    int64_t row_bytes;
    int64_t d_per_row;
};

__device__ __forceinline__ WarpRow warp_row(const GemvParams& p, int warp) {
    WarpRow r;
    int s = 0, row = 0;
    if (p.paired) {
        s = warp >> 2;
        row = blockIdx.x * 4 + (warp & 3);
    } else {
        s = 0;
        while (s + 1 < p.nseg && (int)blockIdx.x >= p.seg[s + 1].cta_begin) s++;
        row = (blockIdx.x - p.seg[s].cta_begin) * kWarps + warp;
    }
    const GemvSeg& g = p.seg[s];
    r.seg = row < g.N ? s : -1;
    r.row = row;
    r.type = g.type;
    r.main = g.main;
    r.dplane = g.dplane;
    r.row_bytes = g.row_bytes;
    r.d_per_row = g.d_per_row;
    return r;
}

// Activation pieces in shared memory.
struct Act {
    const float* f32;
    const int8_t* q8k;
    const float* q8k_d;
    const int16_t* q8k_bs;
    const int8_t* q80;
    const float* q80_d;
};

template <bool DOTS>
__device__ __forceinline__ float chunk_q4k(const uint8_t* slot, const Act& a, int c0, int cb, int lane, int32_t* isum_row,
                                           int32_t* msum_row) {
    float acc = 0.f;
    const int items = cb * 4;
    for (int base = 0; base < items; base += 32) {
        const int it = base + lane;
        const bool valid = it < items;
        const int sb = it >> 2, g = it & 3;
        int isum = 0, msum = 0;
        float dd = 0.f, dm = 0.f;
        if (valid) {
            const uint8_t* blk = slot + sb * Q4K_BYTES;
            const uint4 w0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
            const uint4 w1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * g);
            const int4* xq = reinterpret_cast<const int4*>(a.q8k + (c0 + sb) * QK_K + 64 * g);
            const int4 x0 = xq[0], x1 = xq[1], x2 = xq[2], x3 = xq[3];
            const uint32_t m4 = 0x0f0f0f0fu;
            int lo = 0, hi = 0;
            lo = __dp4a((int)(w0.x & m4), x0.x, lo);
            lo = __dp4a((int)(w0.y & m4), x0.y, lo);
            lo = __dp4a((int)(w0.z & m4), x0.z, lo);
            lo = __dp4a((int)(w0.w & m4), x0.w, lo);
            lo = __dp4a((int)(w1.x & m4), x1.x, lo);
            lo = __dp4a((int)(w1.y & m4), x1.y, lo);
            lo = __dp4a((int)(w1.z & m4), x1.z, lo);
            lo = __dp4a((int)(w1.w & m4), x1.w, lo);
            hi = __dp4a((int)((w0.x >> 4) & m4), x2.x, hi);
            hi = __dp4a((int)((w0.y >> 4) & m4), x2.y, hi);
            hi = __dp4a((int)((w0.z >> 4) & m4), x2.z, hi);
            hi = __dp4a((int)((w0.w >> 4) & m4), x2.w, hi);
            hi = __dp4a((int)((w1.x >> 4) & m4), x3.x, hi);
            hi = __dp4a((int)((w1.y >> 4) & m4), x3.y, hi);
            hi = __dp4a((int)((w1.z >> 4) & m4), x3.z, hi);
            hi = __dp4a((int)((w1.w >> 4) & m4), x3.w, hi);
            int sc0, m0, sc1, m1;
            q4k_scale_min(blk + 4, 2 * g, sc0, m0);
            q4k_scale_min(blk + 4, 2 * g + 1, sc1, m1);
            const int16_t* bs = a.q8k_bs + (c0 + sb) * 16 + 4 * g;
            isum = sc0 * lo + sc1 * hi;
            msum = m0 * ((int)bs[0] + (int)bs[1]) + m1 * ((int)bs[2] + (int)bs[3]);
            if (g == 0) {
                const float dx = a.q8k_d[c0 + sb];
                dd = __fmul_rn(h2f(blk[0] | (blk[1] << 8)), dx);
                dm = __fmul_rn(h2f(blk[2] | (blk[3] << 8)), dx);
            }
        }
        isum += __shfl_xor_sync(0xffffffffu, isum, 1);
        isum += __shfl_xor_sync(0xffffffffu, isum, 2);
        msum += __shfl_xor_sync(0xffffffffu, msum, 1);
        msum += __shfl_xor_sync(0xffffffffu, msum, 2);
        if (valid && g == 0) {
            if (DOTS) {
                isum_row[c0 + sb] = isum;
                msum_row[c0 + sb] = msum;
            } else {
                acc += dd * (float)isum - dm * (float)msum;
            }
        }
    }
    return acc;
}

template <bool DOTS>
__device__ __forceinline__ float chunk_q6k(const uint8_t* slot, const uint16_t* drow, const Act& a, int c0, int cb,
                                           int lane, int32_t* isum_row) {
    float acc = 0.f;
    const int items = cb * 4;
    for (int base = 0; base < items; base += 32) {
        const int it = base + lane;
        const bool valid = it < items;
        const int sb = it >> 2, t = it & 3, h = t >> 1, l0 = (t & 1) * 16;
        int isum = 0;
        float dd = 0.f;
        if (valid) {
            const uint8_t* m = slot + sb * Q6K_MAIN;
            const uint4 A = *reinterpret_cast<const uint4*>(m + 64 * h + l0);
            const uint4 B = *reinterpret_cast<const uint4*>(m + 64 * h + 32 + l0);
            const uint4 H = *reinterpret_cast<const uint4*>(m + 128 + 32 * h + l0);
            const int8_t* sc = reinterpret_cast<const int8_t*>(m + 192 + 8 * h + (l0 >> 4));
            const int8_t* xb = a.q8k + (c0 + sb) * QK_K + 128 * h + l0;
            const int4 x1 = *reinterpret_cast<const int4*>(xb);
            const int4 x2 = *reinterpret_cast<const int4*>(xb + 32);
            const int4 x3 = *reinterpret_cast<const int4*>(xb + 64);
            const int4 x4 = *reinterpret_cast<const int4*>(xb + 96);
            const uint32_t m4 = 0x0f0f0f0fu, m2 = 0x30303030u;
            int d1 = 0, d2 = 0, d3 = 0, d4 = 0;
#define Q6K_WORD(Aw, Bw, Hw, X1, X2, X3, X4)                                  \
    d1 = __dp4a((int)(((Aw) & m4) | (((Hw) << 4) & m2)), X1, d1);             \
    d2 = __dp4a((int)(((Bw) & m4) | (((Hw) << 2) & m2)), X2, d2);             \
    d3 = __dp4a((int)((((Aw) >> 4) & m4) | ((Hw) & m2)), X3, d3);             \
    d4 = __dp4a((int)((((Bw) >> 4) & m4) | (((Hw) >> 2) & m2)), X4, d4);
            Q6K_WORD(A.x, B.x, H.x, x1.x, x2.x, x3.x, x4.x)
            Q6K_WORD(A.y, B.y, H.y, x1.y, x2.y, x3.y, x4.y)
            Q6K_WORD(A.z, B.z, H.z, x1.z, x2.z, x3.z, x4.z)
            Q6K_WORD(A.w, B.w, H.w, x1.w, x2.w, x3.w, x4.w)
#undef Q6K_WORD
            // q stored +32: sum (q-32)*x = sum q*x - 32 * bsum over the 16 elements
            const int16_t* bs = a.q8k_bs + (c0 + sb) * 16 + 8 * h + (l0 >> 4);
            d1 -= 32 * (int)bs[0];
            d2 -= 32 * (int)bs[2];
            d3 -= 32 * (int)bs[4];
            d4 -= 32 * (int)bs[6];
            isum = (int)sc[0] * d1 + (int)sc[2] * d2 + (int)sc[4] * d3 + (int)sc[6] * d4;
            if (t == 0 && !DOTS) dd = __fmul_rn(h2f(drow[c0 + sb]), a.q8k_d[c0 + sb]);
        }
        isum += __shfl_xor_sync(0xffffffffu, isum, 1);
        isum += __shfl_xor_sync(0xffffffffu, isum, 2);
        if (valid && t == 0) {
            if (DOTS) isum_row[c0 + sb] = isum;
            else acc += dd * (float)isum;
        }
    }
    return acc;
}

template <bool DOTS>
__device__ __forceinline__ float chunk_q80(const uint8_t* slot, const uint16_t* drow, const Act& a, int c0, int cb,
                                           int lane, int32_t* isum_row) {
    float acc = 0.f;
    const int nblk = cb * 8;  // 32-element blocks in the chunk
    const int b0 = c0 * 8;
    for (int b = lane; b < nblk; b += 32) {
        const uint4 w0 = *reinterpret_cast<const uint4*>(slot + b * 32);
        const uint4 w1 = *reinterpret_cast<const uint4*>(slot + b * 32 + 16);
        const int4* xq = reinterpret_cast<const int4*>(a.q80 + (b0 + b) * 32);
        const int4 x0 = xq[0], x1 = xq[1];
        int s = 0;
        s = __dp4a((int)w0.x, x0.x, s);
        s = __dp4a((int)w0.y, x0.y, s);
        s = __dp4a((int)w0.z, x0.z, s);
        s = __dp4a((int)w0.w, x0.w, s);
        s = __dp4a((int)w1.x, x1.x, s);
        s = __dp4a((int)w1.y, x1.y, s);
        s = __dp4a((int)w1.z, x1.z, s);
        s = __dp4a((int)w1.w, x1.w, s);
        if (DOTS) {
            isum_row[b0 + b] = s;
        } else {
            // candle BlockQ8_0::vec_dot: sumi as f32 * d_w * d_x, left to right
            acc += __fmul_rn(__fmul_rn((float)s, h2f(drow[b0 + b])), a.q80_d[b0 + b]);
        }
    }
    return acc;
}

__device__ __forceinline__ float chunk_f16(const uint8_t* slot, const Act& a, int c0, int cb, int lane) {
    float acc = 0.f;
    const int units = cb * 32;  // 16-byte units (8 halfs)
    const float* x = a.f32 + c0 * QK_K;
    for (int u = lane; u < units; u += 32) {
        const uint4 w = *reinterpret_cast<const uint4*>(slot + u * 16);
        const float4 xa = *reinterpret_cast<const float4*>(x + u * 8);
        const float4 xb = *reinterpret_cast<const float4*>(x + u * 8 + 4);
        const __half2* h = reinterpret_cast<const __half2*>(&w);
        float2 f0 = __half22float2(h[0]), f1 = __half22float2(h[1]), f2 = __half22float2(h[2]),
               f3 = __half22float2(h[3]);
        acc = fmaf(f0.x, xa.x, acc);
        acc = fmaf(f0.y, xa.y, acc);
        acc = fmaf(f1.x, xa.z, acc);
        acc = fmaf(f1.y, xa.w, acc);
        acc = fmaf(f2.x, xb.x, acc);
        acc = fmaf(f2.y, xb.y, acc);
        acc = fmaf(f3.x, xb.z, acc);
        acc = fmaf(f3.y, xb.w, acc);
    }
    return acc;
}

// Prologue: optional RMSNorm (candle_nn::ops::rms_norm: m = sqrt(sum(x^2)/K + eps),
// y = x / m * w) and quantisation of the activation into shared memory.
__device__ void build_activation(const GemvParams& p, uint8_t* smem, float* red) {
    const int K = p.K, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float m = 1.f;
    const bool norm = p.norm_w != nullptr;
    if (norm) {
        float ss = 0.f;
        for (int i = tid * 4; i < K; i += kThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(p.x + i);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (warp == 0) {
            float v = lane < kWarps ? red[lane] : 0.f;
            v = warp_sum(v);
            if (lane == 0) red[kWarps] = v;
        }
        __syncthreads();
        m = sqrtf(__fdiv_rn(red[kWarps], (float)K) + p.eps);
    }
    auto xval = [&](int i) -> float {
        float v = p.x[i];
        if (norm) v = __fmul_rn(__fdiv_rn(v, m), p.norm_w[i]);
        return v;
    };
    if (p.act_f32 >= 0) {
        float* dst = reinterpret_cast<float*>(smem + p.act_f32);
        for (int i = tid; i < K; i += kThreads) dst[i] = xval(i);
    }
    if (p.act_q8k >= 0) {
        int8_t* qs = reinterpret_cast<int8_t*>(smem + p.act_q8k);
        float* dd = reinterpret_cast<float*>(smem + p.act_q8k_d);
        int16_t* bs = reinterpret_cast<int16_t*>(smem + p.act_q8k_bs);
        for (int b = warp; b < K / QK_K; b += kWarps) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = xval(b * QK_K + lane * 8 + i);
            q8k_quant_warp(v, qs + b * QK_K, bs + b * 16, dd + b, lane);
        }
    }
    if (p.act_q80 >= 0) {
        int8_t* qs = reinterpret_cast<int8_t*>(smem + p.act_q80);
        float* dd = reinterpret_cast<float*>(smem + p.act_q80_d);
        for (int b = warp; b < K / QK8_0; b += kWarps) {
            float d;
            qs[b * QK8_0 + lane] = q80_quant_warp(xval(b * QK8_0 + lane), d);
            if (lane == 0) dd[b] = h2f(f2h(d));
        }
    }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMaxStages];
    __shared__ float red[2 * kWarps + 2];
    __shared__ float res[kWarps];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = p.stages;
    const int nsb = p.K / QK_K;
    uint8_t* ring = smem + p.act_bytes;

    // Rows and chunking of every warp of this CTA (uniform per warp).
    const WarpRow wr = warp_row(p, warp);

    // The chunk count is the same for every warp of a CTA: chunk_sb depends on the type,
    // and a CTA's segments share a chunking class (all quantised or all F16).
    const int cbs = chunk_sb(p.seg[0].type);
    const int nchunks = (nsb + cbs - 1) / cbs;

    if (tid == 0) {
        for (int s = 0; s < S; s++) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();

    uint64_t policy = 0;
    auto issue = [&](int c) {
        const int s = c % S;
        const int c0 = c * cbs, cb = min(cbs, nsb - c0);
        uint32_t total = 0;
        WarpRow rows[kWarps];
#pragma unroll
        for (int w = 0; w < kWarps; w++) {
            rows[w] = warp_row(p, w);
            if (rows[w].seg >= 0) total += cb * sb_bytes(rows[w].type);
        }
        mbar_expect_tx(&full[s], total);
#pragma unroll
        for (int w = 0; w < kWarps; w++) {
            if (rows[w].seg < 0) continue;
            const int sbb = sb_bytes(rows[w].type);
            const uint8_t* src = rows[w].main + rows[w].row * rows[w].row_bytes + (int64_t)c0 * sbb;
            bulk_g2s(ring + (s * kWarps + w) * p.slot_bytes, src, cb * sbb, &full[s], policy);
        }
    };
    if (tid == 0) {
        policy = l2_evict_first_policy();
        for (int c = 0; c < S && c < nchunks; c++) issue(c);
    }

    // Everything above reads only weights; activations come from the previous kernel.
    pdl_wait();
    pdl_launch_dependents();

    build_activation(p, smem, red);
    __syncthreads();

    Act a;
    a.f32 = p.act_f32 >= 0 ? reinterpret_cast<const float*>(smem + p.act_f32) : nullptr;
    a.q8k = p.act_q8k >= 0 ? reinterpret_cast<const int8_t*>(smem + p.act_q8k) : nullptr;
    a.q8k_d = p.act_q8k >= 0 ? reinterpret_cast<const float*>(smem + p.act_q8k_d) : nullptr;
    a.q8k_bs = p.act_q8k >= 0 ? reinterpret_cast<const int16_t*>(smem + p.act_q8k_bs) : nullptr;
    a.q80 = p.act_q80 >= 0 ? reinterpret_cast<const int8_t*>(smem + p.act_q80) : nullptr;
    a.q80_d = p.act_q80 >= 0 ? reinterpret_cast<const float*>(smem + p.act_q80_d) : nullptr;

    const uint16_t* drow = wr.dplane ? wr.dplane + (int64_t)wr.row * wr.d_per_row : nullptr;
    int32_t* isum_row = nullptr;
    int32_t* msum_row = nullptr;
    if (EPI == EPI_DOTS && wr.seg >= 0) {
        const int per_row = wr.type == TPTC_TYPE_Q8_0 ? p.K / QK8_0 : nsb;
        isum_row = p.isum + (int64_t)wr.row * per_row;
        msum_row = p.msum ? p.msum + (int64_t)wr.row * per_row : nullptr;
    }

    float acc = 0.f;
    bool timed_out = false;
    for (int c = 0; c < nchunks; c++) {
        const int s = c % S;
        if (!mbar_wait_bounded(&full[s], (c / S) & 1, p.err)) timed_out = true;
        if (!timed_out && wr.seg >= 0) {
            const uint8_t* slot = ring + (s * kWarps + warp) * p.slot_bytes;
            const int c0 = c * cbs, cb = min(cbs, nsb - c0);
            switch (wr.type) {
            case TPTC_TYPE_Q4_K: acc += chunk_q4k<EPI == EPI_DOTS>(slot, a, c0, cb, lane, isum_row, msum_row); break;
            case TPTC_TYPE_Q6_K: acc += chunk_q6k<EPI == EPI_DOTS>(slot, drow, a, c0, cb, lane, isum_row); break;
            case TPTC_TYPE_Q8_0: acc += chunk_q80<EPI == EPI_DOTS>(slot, drow, a, c0, cb, lane, isum_row); break;
            default: acc += chunk_f16(slot, a, c0, cb, lane); break;
            }
        }
        if (__syncthreads_or(timed_out)) return;  // every thread leaves together
        if (tid == 0 && c + S < nchunks) {
            fence_proxy_async_smem();
            issue(c + S);
        }
    }
    if (EPI == EPI_DOTS) return;

    const float y = warp_sum(acc);
    if (EPI == EPI_STORE) {
        if (lane == 0 && wr.seg >= 0) p.out[wr.row] = y;
    } else if (EPI == EPI_RESID) {
        if (lane == 0 && wr.seg >= 0) p.out[wr.row] += y;
    } else if (EPI == EPI_QKV) {
        if (lane == 0) res[warp] = y;
        __syncthreads();
        if (tid < kWarps) {
            const WarpRow r = warp_row(p, tid);
            if (r.seg >= 0) {
                const int pos = *p.pos;
                const int d = r.row % p.hd, head = r.row / p.hd;
                float v = res[tid];
                if (r.seg <= 1) {  // q or k: interleaved-pair rotation (rope_i)
                    const int i = d >> 1;
                    const float c = p.rope_cos[(int64_t)pos * (p.hd / 2) + i];
                    const float sn = p.rope_sin[(int64_t)pos * (p.hd / 2) + i];
                    if ((d & 1) == 0) v = __fsub_rn(__fmul_rn(res[tid], c), __fmul_rn(res[tid + 1], sn));
                    else v = __fadd_rn(__fmul_rn(res[tid - 1], sn), __fmul_rn(res[tid], c));
                }
                if (r.seg == 0) {
                    p.out[r.row] = v;
                } else {
                    void* cache = r.seg == 1 ? p.kcache : p.vcache;
                    const int64_t at = ((int64_t)head * p.max_seq + pos) * p.hd + d;
                    if (p.kv_f32) static_cast<float*>(cache)[at] = v;
                    else static_cast<__half*>(cache)[at] = __float2half_rn(v);
                }
            }
        }
    } else if (EPI == EPI_GLU) {
        if (lane == 0) res[warp] = y;
        __syncthreads();
        if (tid < 4) {
            const WarpRow r = warp_row(p, tid);
            if (r.seg >= 0) {
                const float g = res[tid], u = res[tid + 4];
                p.out[r.row] = __fmul_rn(__fdiv_rn(g, 1.f + expf(-g)), u);
            }
        }
    }
}

}  // namespace

void gemv_prepare(GemvParams& p) {
    bool need_f32 = false, need_q8k = false, need_q80 = false;
    int slot = 0;
    for (int s = 0; s < p.nseg; s++) {
        const int t = p.seg[s].type;
        if (t == TPTC_TYPE_F16) need_f32 = true;
        else if (t == TPTC_TYPE_Q8_0) need_q80 = true;
        else need_q8k = true;
        slot = std::max(slot, chunk_sb(t) * sb_bytes(t));
    }
    const int K = p.K;
    int off = 0;
    auto take = [&](int bytes) {
        int o = off;
        off += (bytes + 15) / 16 * 16;
        return o;
    };
    p.act_f32 = need_f32 ? take(K * 4) : -1;
    p.act_q8k = need_q8k ? take(K) : -1;
    p.act_q8k_d = need_q8k ? take(K / QK_K * 4) : -1;
    p.act_q8k_bs = need_q8k ? take(K / 16 * 2) : -1;
    p.act_q80 = need_q80 ? take(K) : -1;
    p.act_q80_d = need_q80 ? take(K / QK8_0 * 4) : -1;
    p.act_bytes = (off + 127) / 128 * 128;
    p.slot_bytes = slot;
    const int nsb = K / QK_K;
    const int cbs = chunk_sb(p.seg[0].type);
    const int nchunks = (nsb + cbs - 1) / cbs;
    p.stages = std::min(nchunks, 2);
}

int gemv_grid(const GemvParams& p) {
    if (p.paired) return ceil_div(p.seg[0].N, 4);
    int n = 0;
    for (int s = 0; s < p.nseg; s++) n += ceil_div(p.seg[s].N, kWarps);
    return n;
}

size_t gemv_smem(const GemvParams& p) { return (size_t)p.act_bytes + (size_t)p.stages * kWarps * p.slot_bytes; }

template <int EPI>
static cudaError_t launch_epi(const GemvParams& p, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(gemv_grid(p));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = gemv_smem(p);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_kernel<EPI>, p);
}

cudaError_t gemv_init_device() {
    const int max_smem = 200 * 1024;
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<EPI_GLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    return cudaFuncSetAttribute(gemv_kernel<EPI_DOTS>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

cudaError_t gemv_launch(const GemvParams& p, int epi, cudaStream_t st, bool pdl) {
    switch (epi) {
    case EPI_STORE: return launch_epi<EPI_STORE>(p, st, pdl);
    case EPI_RESID: return launch_epi<EPI_RESID>(p, st, pdl);
    case EPI_QKV: return launch_epi<EPI_QKV>(p, st, pdl);
    case EPI_GLU: return launch_epi<EPI_GLU>(p, st, pdl);
    case EPI_DOTS: return launch_epi<EPI_DOTS>(p, st, pdl);
    }
    return cudaErrorInvalidValue;
}

}  // namespace tptc
