// gemv.cu -- batch-1 dequant-fused GEMV for decode.
//
// Replaces the reference's per-matmul pair "dequantise the whole weight to f32, then a
// 16x16-tiled f32 GEMM with M=1" (shaders/dequant_q4k.wgsl:74-115, dequant_q6k.wgsl:58-92,
// dequant_q8.wgsl:51-73, dequant_f16.wgsl:30-37, gemm.wgsl:28-70, driven by
// engine/wgpu_engine.rs:581-605), with candle QMatMul semantics (candle_engine.rs:221,273):
// the activation is quantised to Q8_K (Q4_K/Q5_K/Q6_K weights) or Q8_0 (Q4_0/Q5_0/Q8_0 weights)
// and every super-block (32-block) contributes (d_w*d_x)*isum - (dmin_w*d_x)*msum
// ((isum*d_w)*d_x) from exact integer sums.
//
// Kernel structure: a persistent grid (one CTA per SM), 9 warps per CTA.
//   - warp 8 (producer) streams the CTA's weight tiles (8 rows x a chunk of super-blocks,
//     contiguous in the tiled device layout of gemv.cuh) through a ring of shared-memory
//     stages, one 1-D TMA bulk copy of 13-32 KB per stage (L2 evict-first), gated by
//     per-stage "empty" mbarriers.  Weights do not depend on the previous kernel, so the
//     producer starts before griddepcontrol.wait: under programmatic dependent launch the
//     weight stream of this kernel overlaps the tail of the previous one.
//   - warps 0-7 (consumers) wait for the previous kernel, RMS-normalise (optional) and
//     quantise the activation into shared memory once, then each reduces one row of every
//     tile: dp4a integer dots per sub-block, one f32 FMA per lane item, a warp sum per row.
//     Each warp releases a stage by arriving on its "empty" barrier.
//   - every warp writes its own row, no barrier between warps: store / residual add / the
//     q|k|v projection (q and k unrotated -- the attention kernel applies RoPE -- and v into
//     the KV cache) / the fused gate|up rows (the down projection forms silu(gate)*up while
//     quantising its input).
#include <algorithm>

#include "act.cuh"

namespace tptc {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + producer warp
constexpr int kRingBudget = 100 * 1024;    // shared memory per CTA (two kernels fit per SM)


__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }
// Named barrier 2 + i joins consumer warps i and i + 4 only.
__device__ __forceinline__ void pair_sync(int i) { asm volatile("bar.sync %0, 64;" ::"r"(2 + i) : "memory"); }

// Logical row held in tile row r (0..7) of work unit u, and the segment it belongs to.
struct UnitRow {
    int seg;   // -1: padding row (N not a multiple of 8)
    int row;   // logical row within the segment (for glu: gate row if r < 4, up row otherwise)
    int out;   // output index (glu: the gate/up pair index)
};

__device__ __forceinline__ int unit_seg(const GemvParams& p, int u) {
    int s = 0;
    while (s + 1 < p.nseg && u >= p.seg[s + 1].unit_begin) s++;
    return s;
}

// Byte offsets of the segments' weights from m.main: 0, or for an expert segment the
// selected expert's place in the stack.  The index is written by the previous kernel (the
// routing kernel), so a launch with experts waits for it first; the producer lane calls this
// once and keeps the offsets in registers (seg_off picks one by selects, no local array).
static_assert(kGemvMaxSeg == 3, "seg_off selects among three segments");
struct SegOff {
    int64_t o0 = 0, o1 = 0, o2 = 0;
};
__device__ __forceinline__ SegOff expert_offsets(const GemvParams& p) {
    SegOff r;
    if (!p.moe_sel) return r;
    pdl_wait();
    auto off = [&](int s) -> int64_t {
        if (s >= p.nseg || p.seg[s].sel < 0) return 0;
        const int e = min(max(__ldcg(p.moe_sel + p.seg[s].sel), 0), p.moe_nexp - 1);
        return (int64_t)e * p.moe_stride;
    };
    r.o0 = off(0);
    r.o1 = off(1);
    r.o2 = off(2);
    return r;
}
__device__ __forceinline__ int64_t seg_off(const SegOff& r, int s) { return s == 0 ? r.o0 : s == 1 ? r.o1 : r.o2; }

// Whether units u and u + grid are reduced together (sharing the activation slice): both
// exist, same Q4_K / Q6_K weights, and the ring holds the pair plus at least one stage to
// refill meanwhile.  Producer and consumers take the same decision.
// Super-block byte sizes inside the kernels.  The narrow build (WIDE = false) knows four
// formats and picks among them by selects; the wide build takes the switch over every format.
// The paired path (unit_pair: Q4_K or Q6_K only) uses the narrow form in both builds.
template <bool WIDE>
__device__ __forceinline__ int k_sb_main(int t) {
    if constexpr (WIDE) return sb_main_bytes(t);
    constexpr int q4k = sb_main_bytes(TPTC_TYPE_Q4_K), q6k = sb_main_bytes(TPTC_TYPE_Q6_K),
                  q80 = sb_main_bytes(TPTC_TYPE_Q8_0), f16 = sb_main_bytes(TPTC_TYPE_F16);
    return t == TPTC_TYPE_Q4_K ? q4k : t == TPTC_TYPE_Q6_K ? q6k : t == TPTC_TYPE_Q8_0 ? q80 : f16;
}
template <bool WIDE>
__device__ __forceinline__ int k_sb_d(int t) {
    if constexpr (WIDE) return sb_d_bytes(t);
    constexpr int q6k = sb_d_bytes(TPTC_TYPE_Q6_K), q80 = sb_d_bytes(TPTC_TYPE_Q8_0);
    return t == TPTC_TYPE_Q6_K ? q6k : t == TPTC_TYPE_Q8_0 ? q80 : 0;
}
template <bool WIDE>
__device__ __forceinline__ int k_sb_bytes(int t) {
    return k_sb_main<WIDE>(t) + k_sb_d<WIDE>(t);
}

__device__ __forceinline__ bool unit_pair(const GemvParams& p, int u, int epi) {
    const int u2 = u + gridDim.x;
    if (epi == EPI_DOTS || u2 >= p.units || p.stages < 3) return false;
    const int t = p.seg[unit_seg(p, u)].m.type;
    return t == p.seg[unit_seg(p, u2)].m.type && (t == TPTC_TYPE_Q4_K || t == TPTC_TYPE_Q6_K);
}

__device__ __forceinline__ UnitRow unit_row(const GemvParams& p, int u, int r) {
    UnitRow ur;
    const int s = unit_seg(p, u);
    const DevMatrix& m = p.seg[s].m;
    const int t = u - p.seg[s].unit_begin;
    ur.seg = s;
    if (m.glu) {
        const int half = m.N / 2, pr = 4 * t + (r & 3);
        ur.out = pr + p.seg[s].out_off;
        ur.row = r < 4 ? pr : half + pr;
        if (pr >= half) ur.seg = -1;
    } else {
        ur.row = t * kTileRows + r;
        ur.out = ur.row + p.seg[s].out_off;
        if (ur.row >= m.N) ur.seg = -1;
    }
    return ur;
}

struct Act {
    const float* f32;
    const int8_t* q8k;
    const float* q8k_d;
    const int16_t* q8k_bs;  // 16 sums of 16 elements per block
    const int16_t* q8k_ps;  // 8 sums of 32 elements per block (Q4_K sub-blocks)
    const int8_t* q80;
    const float* q80_d;
};

// dp4a of unsigned bytes (a) with signed bytes (b).
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(int8_t)((w >> (8 * i)) & 0xff); }
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xff); }

// Forward path (EPI != DOTS).  For Q4_K and Q6_K lane l of a row's warp reduces half
// super-block l of the chunk (super-block l/2, elements 128*(l%2) .. +128): its quants,
// scales and activations are read once per 128 elements.  The chunk's Q8_K quants are
// stored lane-transposed in shared memory (xt_offset): 16-byte vector v of half super-block
// l sits at (v * nh + l) * 16, nh = 2 * cb, so the 32 lanes read 512 contiguous bytes per
// load.  Each lane scales its own partial integer sums by the super-block factors,
// (d_w*d_x)*isum_half - (dmin_w*d_x)*msum_half; the f32 result differs from scaling the
// whole block's integer sum only by float rounding.  The DOTS test hook keeps the exact
// per-block integers (chunk_q4k / chunk_q6k below, natural activation layout).

// The lane's slice of a chunk's Q8_K activation (half super-block `lane`): 8 transposed
// 16-byte vectors of quants, the super-block scale, and 32- (Q4_K) or 16-element (Q6_K) sums.
struct XHalf {
    int4 x[8];
    float dx;
    uint2 ps;   // pair sums of sub-blocks 4h .. 4h+3 (Q4_K)
    uint4 bs;   // bsums of the 8 16-element groups (Q6_K)
};

template <bool Q6>
__device__ __forceinline__ void load_xhalf(XHalf& xh, const Act& a, int c0, int nh, int lane) {
    const int sb = lane >> 1, h = lane & 1;
    const int4* xv = reinterpret_cast<const int4*>(a.q8k + c0 * QK_K) + lane;
#pragma unroll
    for (int v = 0; v < 8; v++) xh.x[v] = xv[v * nh];
    xh.dx = a.q8k_d[c0 + sb];
    if (Q6) xh.bs = *reinterpret_cast<const uint4*>(a.q8k_bs + (c0 + sb) * 16 + 8 * h);
    else xh.ps = *reinterpret_cast<const uint2*>(a.q8k_ps + (c0 + sb) * 8 + 4 * h);
}

__device__ __forceinline__ float q4k_half(const uint8_t* slot, const XHalf& xh, int lane) {
    const int sb = lane >> 1, h = lane & 1;
    const uint8_t* blk = slot + sb * Q4K_BYTES;
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);  // d, dmin | scales[0..3] | [4..7] | [8..11]
    const uint4* wq = reinterpret_cast<const uint4*>(blk + 16 + 64 * h);
    const uint4 w0 = wq[0], w1 = wq[1], w2 = wq[2], w3 = wq[3];
    // sub-blocks 4h, 4h+1 are the low / high nibbles of qs[64h .. +32), 4h+2, 4h+3 of
    // qs[64h+32 .. +32); high nibbles are dotted in place (16x) and shifted back
    const uint32_t lo = 0x0f0f0f0fu, hi = 0xf0f0f0f0u;
    int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    // 16 quant bytes W: low nibbles pair with activations XL, high nibbles with XH
#define Q4_VEC(W, XL, XH, SL, SH)                                      \
    SL = dp4a_us(W.x & lo, XL.x, SL); SH = dp4a_us(W.x & hi, XH.x, SH);  \
    SL = dp4a_us(W.y & lo, XL.y, SL); SH = dp4a_us(W.y & hi, XH.y, SH);  \
    SL = dp4a_us(W.z & lo, XL.z, SL); SH = dp4a_us(W.z & hi, XH.z, SH);  \
    SL = dp4a_us(W.w & lo, XL.w, SL); SH = dp4a_us(W.w & hi, XH.w, SH);
    Q4_VEC(w0, xh.x[0], xh.x[2], s0, s1)
    Q4_VEC(w1, xh.x[1], xh.x[3], s0, s1)
    Q4_VEC(w2, xh.x[4], xh.x[6], s2, s3)
    Q4_VEC(w3, xh.x[5], xh.x[7], s2, s3)
#undef Q4_VEC
    s1 >>= 4;
    s3 >>= 4;
    const uint32_t k6 = 0x3f3f3f3fu, k4 = 0x0f0f0f0fu, k2 = 0x03030303u;
    const uint32_t sc = h == 0 ? hd.y & k6 : (hd.w & k4) | (((hd.y >> 6) & k2) << 4);
    const uint32_t mn = h == 0 ? hd.z & k6 : ((hd.w >> 4) & k4) | (((hd.z >> 6) & k2) << 4);
    const int isum = ubyte(sc, 0) * s0 + ubyte(sc, 1) * s1 + ubyte(sc, 2) * s2 + ubyte(sc, 3) * s3;
    const int msum = ubyte(mn, 0) * (int)(int16_t)(xh.ps.x & 0xffff) + ubyte(mn, 1) * (int)(int16_t)(xh.ps.x >> 16) +
                     ubyte(mn, 2) * (int)(int16_t)(xh.ps.y & 0xffff) + ubyte(mn, 3) * (int)(int16_t)(xh.ps.y >> 16);
    const float dd = __fmul_rn(__half2float(__ushort_as_half((unsigned short)(hd.x & 0xffff))), xh.dx);
    const float dm = __fmul_rn(__half2float(__ushort_as_half((unsigned short)(hd.x >> 16))), xh.dx);
    return dd * (float)isum - dm * (float)msum;
}

// Q5_K (the GGUF block unchanged: d | dmin | scales[12] | qh[32] | qs[128]): q4k_half's work
// split and scales, with the 5th bit of element l of sub-block j (bit j of qh[l]) placed
// above each nibble before the dot; high nibbles are shifted down first.
__device__ __forceinline__ float q5k_half(const uint8_t* slot, const XHalf& xh, int lane) {
    const int sb = lane >> 1, h = lane & 1;
    const uint8_t* blk = slot + sb * Q5K_BYTES;
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16);  // qh[0..16)
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32);  // qh[16..32)
    const uint4* wq = reinterpret_cast<const uint4*>(blk + 48 + 64 * h);
    const uint4 w0 = wq[0], w1 = wq[1], w2 = wq[2], w3 = wq[3];
    const uint32_t lo = 0x0f0f0f0fu, one = 0x01010101u;
    const int j0 = 4 * h;
    int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#define Q5_WORD(W, H, XL, XH, SL, SH, JL)                                             \
    SL = dp4a_us((W & lo) | (((H >> (JL)) & one) << 4), XL, SL);                      \
    SH = dp4a_us(((W >> 4) & lo) | (((H >> ((JL) + 1)) & one) << 4), XH, SH);
#define Q5_VEC(W, H, XL, XH, SL, SH, JL)             \
    Q5_WORD(W.x, H.x, XL.x, XH.x, SL, SH, JL)        \
    Q5_WORD(W.y, H.y, XL.y, XH.y, SL, SH, JL)        \
    Q5_WORD(W.z, H.z, XL.z, XH.z, SL, SH, JL)        \
    Q5_WORD(W.w, H.w, XL.w, XH.w, SL, SH, JL)
    Q5_VEC(w0, qa, xh.x[0], xh.x[2], s0, s1, j0)
    Q5_VEC(w1, qb, xh.x[1], xh.x[3], s0, s1, j0)
    Q5_VEC(w2, qa, xh.x[4], xh.x[6], s2, s3, j0 + 2)
    Q5_VEC(w3, qb, xh.x[5], xh.x[7], s2, s3, j0 + 2)
#undef Q5_VEC
#undef Q5_WORD
    const uint32_t k6 = 0x3f3f3f3fu, k4 = 0x0f0f0f0fu, k2 = 0x03030303u;
    const uint32_t sc = h == 0 ? hd.y & k6 : (hd.w & k4) | (((hd.y >> 6) & k2) << 4);
    const uint32_t mn = h == 0 ? hd.z & k6 : ((hd.w >> 4) & k4) | (((hd.z >> 6) & k2) << 4);
    const int isum = ubyte(sc, 0) * s0 + ubyte(sc, 1) * s1 + ubyte(sc, 2) * s2 + ubyte(sc, 3) * s3;
    const int msum = ubyte(mn, 0) * (int)(int16_t)(xh.ps.x & 0xffff) + ubyte(mn, 1) * (int)(int16_t)(xh.ps.x >> 16) +
                     ubyte(mn, 2) * (int)(int16_t)(xh.ps.y & 0xffff) + ubyte(mn, 3) * (int)(int16_t)(xh.ps.y >> 16);
    const float dd = __fmul_rn(__half2float(__ushort_as_half((unsigned short)(hd.x & 0xffff))), xh.dx);
    const float dm = __fmul_rn(__half2float(__ushort_as_half((unsigned short)(hd.x >> 16))), xh.dx);
    return dd * (float)isum - dm * (float)msum;
}

__device__ __forceinline__ float q6k_half(const uint8_t* slot, const uint16_t* dsec, const XHalf& xh, int lane) {
    const int sb = lane >> 1, h = lane & 1;
    const uint8_t* m = slot + sb * Q6K_MAIN;
    const uint4* qa = reinterpret_cast<const uint4*>(m + 64 * h);        // ql[64h .. +32)
    const uint4* qb = reinterpret_cast<const uint4*>(m + 64 * h + 32);   // ql[64h+32 .. +32)
    const uint4* qh = reinterpret_cast<const uint4*>(m + 128 + 32 * h);  // qh[32h .. +32)
    const uint4 A0 = qa[0], A1 = qa[1], B0 = qb[0], B1 = qb[1], H0 = qh[0], H1 = qh[1];
    const uint2 scw = *reinterpret_cast<const uint2*>(m + 192 + 8 * h);  // int8 scales sc[8h .. +8)
    const float dw = h2f(dsec[sb]);
    // word k of ql/qh holds positions l = 4k..4k+3 of the four 32-element groups
    // (elements 128h + l, +32, +64, +96; sub-blocks 2*group + k/4)
    const uint32_t m4 = 0x0f0f0f0fu, m2 = 0x30303030u;
    int t[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#define Q6_WORD(Aw, Bw, Hw, X1, X2, X3, X4, T0)                                        \
    t[T0 + 0] = dp4a_us(((Aw) & m4) | (((Hw) << 4) & m2), X1, t[T0 + 0]);              \
    t[T0 + 2] = dp4a_us(((Bw) & m4) | (((Hw) << 2) & m2), X2, t[T0 + 2]);              \
    t[T0 + 4] = dp4a_us((((Aw) >> 4) & m4) | ((Hw) & m2), X3, t[T0 + 4]);              \
    t[T0 + 6] = dp4a_us((((Bw) >> 4) & m4) | (((Hw) >> 2) & m2), X4, t[T0 + 6]);
    Q6_WORD(A0.x, B0.x, H0.x, xh.x[0].x, xh.x[2].x, xh.x[4].x, xh.x[6].x, 0)
    Q6_WORD(A0.y, B0.y, H0.y, xh.x[0].y, xh.x[2].y, xh.x[4].y, xh.x[6].y, 0)
    Q6_WORD(A0.z, B0.z, H0.z, xh.x[0].z, xh.x[2].z, xh.x[4].z, xh.x[6].z, 0)
    Q6_WORD(A0.w, B0.w, H0.w, xh.x[0].w, xh.x[2].w, xh.x[4].w, xh.x[6].w, 0)
    Q6_WORD(A1.x, B1.x, H1.x, xh.x[1].x, xh.x[3].x, xh.x[5].x, xh.x[7].x, 1)
    Q6_WORD(A1.y, B1.y, H1.y, xh.x[1].y, xh.x[3].y, xh.x[5].y, xh.x[7].y, 1)
    Q6_WORD(A1.z, B1.z, H1.z, xh.x[1].z, xh.x[3].z, xh.x[5].z, xh.x[7].z, 1)
    Q6_WORD(A1.w, B1.w, H1.w, xh.x[1].w, xh.x[3].w, xh.x[5].w, xh.x[7].w, 1)
#undef Q6_WORD
    // q is stored +32: sum (q-32)*x = sum q*x - 32 * bsum over each 16 elements
    const uint32_t bw[4] = {xh.bs.x, xh.bs.y, xh.bs.z, xh.bs.w};
    int isum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int bs = (int)(int16_t)((bw[i >> 1] >> (16 * (i & 1))) & 0xffff);
        isum += sbyte(i < 4 ? scw.x : scw.y, i & 3) * (t[i] - 32 * bs);
    }
    return __fmul_rn(dw, xh.dx) * (float)isum;
}

// The lane's half super-block of Q8_K activations in the natural layout (the DOTS test hook):
// elements 128h .. 128h + 127 of block c0 + lane / 2 are contiguous there.
__device__ __forceinline__ void load_xhalf_nat(XHalf& xh, const Act& a, int c0, int lane) {
    const int sb = lane >> 1, h = lane & 1;
    const int4* xv = reinterpret_cast<const int4*>(a.q8k + (c0 + sb) * QK_K + 128 * h);
#pragma unroll
    for (int v = 0; v < 8; v++) xh.x[v] = xv[v];
    xh.dx = a.q8k_d[c0 + sb];
    xh.bs = *reinterpret_cast<const uint4*>(a.q8k_bs + (c0 + sb) * 16 + 8 * h);
}

// 16-element sum i (0..7) of the lane's half from the Q8_K bsums.
__device__ __forceinline__ int xh_bsum(const XHalf& xh, int i) {
    const uint32_t w = i < 2 ? xh.bs.x : i < 4 ? xh.bs.y : i < 6 ? xh.bs.z : xh.bs.w;
    return (int)(int16_t)((w >> (16 * (i & 1))) & 0xffff);
}

// Q2_K half super-block (device: qs[64] | scales[16]; d, dmin in the scale section).
// Element 128h + 32s + l is bits 2s of qs[32h + l]; it pairs with activation vector 2s + (l >= 16)
// and belongs to 16-element group i = 2s + (l >= 16) of the half, scale byte scales[8h + i]
// (low nibble: scale, high nibble: min).  isum = sum_i sc_i * dot_i, msum = sum_i m_i * bsum_i.
__device__ __forceinline__ void q2k_half_ints(const uint8_t* slot, const XHalf& xh, int lane, int& isum, int& msum) {
    const int sb = lane >> 1, h = lane & 1;
    const uint8_t* m = slot + sb * 80;
    const uint4 Q0 = *reinterpret_cast<const uint4*>(m + 32 * h), Q1 = *reinterpret_cast<const uint4*>(m + 32 * h + 16);
    const uint2 scw = *reinterpret_cast<const uint2*>(m + 64 + 8 * h);
    const uint32_t m3 = 0x03030303u;
    int t[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#define Q2_WORD(W, K, T0)                                                    \
    t[T0 + 0] = dp4a_us((W) & m3, xh.x[T0 + 0].K, t[T0 + 0]);                \
    t[T0 + 2] = dp4a_us(((W) >> 2) & m3, xh.x[T0 + 2].K, t[T0 + 2]);         \
    t[T0 + 4] = dp4a_us(((W) >> 4) & m3, xh.x[T0 + 4].K, t[T0 + 4]);         \
    t[T0 + 6] = dp4a_us(((W) >> 6) & m3, xh.x[T0 + 6].K, t[T0 + 6]);
    Q2_WORD(Q0.x, x, 0) Q2_WORD(Q0.y, y, 0) Q2_WORD(Q0.z, z, 0) Q2_WORD(Q0.w, w, 0)
    Q2_WORD(Q1.x, x, 1) Q2_WORD(Q1.y, y, 1) Q2_WORD(Q1.z, z, 1) Q2_WORD(Q1.w, w, 1)
#undef Q2_WORD
    isum = 0;
    msum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int g = ubyte(i < 4 ? scw.x : scw.y, i & 3);
        isum += (g & 0x0f) * t[i];
        msum += (g >> 4) * xh_bsum(xh, i);
    }
}

__device__ __forceinline__ float q2k_half(const uint8_t* slot, const uint16_t* dsec, const XHalf& xh, int lane) {
    int isum, msum;
    q2k_half_ints(slot, xh, lane, isum, msum);
    const int sb = lane >> 1;
    // candle BlockQ2K: dall = d_x * d_w, dmin = d_x * dmin_w; dall * isum - dmin * msum
    const float dall = __fmul_rn(xh.dx, h2f(dsec[2 * sb])), dmin = __fmul_rn(xh.dx, h2f(dsec[2 * sb + 1]));
    return dall * (float)isum - dmin * (float)msum;
}

// Q3_K half super-block (device: hmask[32] | qs[64]; scales[12] and d in a 14-byte scale
// entry).  Element 128h + 32s + l: q = ((qs[32h + l] >> 2s) & 3) - 4 * (1 - bit (4h + s) of
// hmask[l]); sum(q * x) over a 16-element group is dot(ql, x) - 4 * (bsum - dot(hbit, x)).
// Its 6-bit scale k = 8h + i (minus 32) as the raw-block dequantisation decodes it.
__device__ __forceinline__ int q3k_half_ints(const uint8_t* slot, const uint16_t* dsec, const XHalf& xh, int lane) {
    const int sb = lane >> 1, h = lane & 1;
    const uint8_t* m = slot + sb * 96;
    const uint4 H0 = *reinterpret_cast<const uint4*>(m), H1 = *reinterpret_cast<const uint4*>(m + 16);
    const uint4 Q0 = *reinterpret_cast<const uint4*>(m + 32 + 32 * h), Q1 = *reinterpret_cast<const uint4*>(m + 48 + 32 * h);
    const uint8_t* sc = reinterpret_cast<const uint8_t*>(dsec) + sb * 14;
    const uint32_t m3 = 0x03030303u, one = 0x01010101u;
    const int hs = 4 * h;
    int tq[8] = {0, 0, 0, 0, 0, 0, 0, 0}, th[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#define Q3_ONE(W, H, K, T, S)                                                        \
    tq[T] = dp4a_us(((W) >> (2 * (S))) & m3, xh.x[T].K, tq[T]);                      \
    th[T] = dp4a_us(((H) >> (hs + (S))) & one, xh.x[T].K, th[T]);
#define Q3_WORD(W, H, K, T0) \
    Q3_ONE(W, H, K, T0 + 0, 0) Q3_ONE(W, H, K, T0 + 2, 1) Q3_ONE(W, H, K, T0 + 4, 2) Q3_ONE(W, H, K, T0 + 6, 3)
    Q3_WORD(Q0.x, H0.x, x, 0) Q3_WORD(Q0.y, H0.y, y, 0) Q3_WORD(Q0.z, H0.z, z, 0) Q3_WORD(Q0.w, H0.w, w, 0)
    Q3_WORD(Q1.x, H1.x, x, 1) Q3_WORD(Q1.y, H1.y, y, 1) Q3_WORD(Q1.z, H1.z, z, 1) Q3_WORD(Q1.w, H1.w, w, 1)
#undef Q3_WORD
#undef Q3_ONE
    int isum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int k = 8 * h + i;
        const int scale = (((sc[k & 7] >> (4 * (k >> 3))) & 0x0f) | (((sc[8 + (k & 3)] >> (2 * (k >> 2))) & 3) << 4)) - 32;
        isum += scale * (tq[i] - 4 * (xh_bsum(xh, i) - th[i]));
    }
    return isum;
}

__device__ __forceinline__ float q3k_half(const uint8_t* slot, const uint16_t* dsec, const XHalf& xh, int lane) {
    const int isum = q3k_half_ints(slot, dsec, xh, lane);
    const uint8_t* sc = reinterpret_cast<const uint8_t*>(dsec) + (lane >> 1) * 14;
    // candle BlockQ3K: d = d_w * d_x, then d * isum
    return __fmul_rn(h2f(sc[12] | (sc[13] << 8)), xh.dx) * (float)isum;
}

// DOTS for Q2_K / Q3_K: the two halves' integers of each super-block added, written by its
// even lane.
template <int TYPE>
__device__ __forceinline__ void dots_q23k(const uint8_t* slot, const uint16_t* dsec, const Act& a, int c0, int cb,
                                          int lane, int32_t* isum_row, int32_t* msum_row) {
    int isum = 0, msum = 0;
    if (lane < 2 * cb) {
        XHalf xh;
        load_xhalf_nat(xh, a, c0, lane);
        if (TYPE == TPTC_TYPE_Q2_K) q2k_half_ints(slot, xh, lane, isum, msum);
        else isum = q3k_half_ints(slot, dsec, xh, lane);
    }
    isum += __shfl_xor_sync(0xffffffffu, isum, 1);
    msum += __shfl_xor_sync(0xffffffffu, msum, 1);
    if (lane < 2 * cb && (lane & 1) == 0) {
        isum_row[c0 + (lane >> 1)] = isum;
        if (msum_row && TYPE == TPTC_TYPE_Q2_K) msum_row[c0 + (lane >> 1)] = msum;
    }
}

template <bool DOTS>
__device__ __forceinline__ float chunk_q4k(const uint8_t* slot, const Act& a, int c0, int cb, int lane, int first,
                                           int stride, int32_t* isum_row, int32_t* msum_row) {
    float acc = 0.f;
    const int items = cb * 4;
    for (int base = first; base < items; base += stride) {
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
                if (msum_row) msum_row[c0 + sb] = msum;
            } else {
                acc += dd * (float)isum - dm * (float)msum;
            }
        }
    }
    return acc;
}

// Q5_K in chunk_q4k's item split (natural activation layout; the DOTS test hook).
template <bool DOTS>
__device__ __forceinline__ float chunk_q5k(const uint8_t* slot, const Act& a, int c0, int cb, int lane, int first,
                                           int stride, int32_t* isum_row, int32_t* msum_row) {
    float acc = 0.f;
    const int items = cb * 4;
    for (int base = first; base < items; base += stride) {
        const int it = base + lane;
        const bool valid = it < items;
        const int sb = it >> 2, g = it & 3;
        int isum = 0, msum = 0;
        float dd = 0.f, dm = 0.f;
        if (valid) {
            const uint8_t* blk = slot + sb * Q5K_BYTES;
            const uint4 w0 = *reinterpret_cast<const uint4*>(blk + 48 + 32 * g);
            const uint4 w1 = *reinterpret_cast<const uint4*>(blk + 64 + 32 * g);
            const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16);
            const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32);
            const int4* xq = reinterpret_cast<const int4*>(a.q8k + (c0 + sb) * QK_K + 64 * g);
            const int4 x0 = xq[0], x1 = xq[1], x2 = xq[2], x3 = xq[3];
            const uint32_t m4 = 0x0f0f0f0fu, one = 0x01010101u;
            const int jl = 2 * g, jh = 2 * g + 1;
            int lo = 0, hi = 0;
#define Q5_LO(W, H, X) lo = __dp4a((int)((W & m4) | (((H >> jl) & one) << 4)), X, lo);
#define Q5_HI(W, H, X) hi = __dp4a((int)(((W >> 4) & m4) | (((H >> jh) & one) << 4)), X, hi);
            Q5_LO(w0.x, qa.x, x0.x) Q5_LO(w0.y, qa.y, x0.y) Q5_LO(w0.z, qa.z, x0.z) Q5_LO(w0.w, qa.w, x0.w)
            Q5_LO(w1.x, qb.x, x1.x) Q5_LO(w1.y, qb.y, x1.y) Q5_LO(w1.z, qb.z, x1.z) Q5_LO(w1.w, qb.w, x1.w)
            Q5_HI(w0.x, qa.x, x2.x) Q5_HI(w0.y, qa.y, x2.y) Q5_HI(w0.z, qa.z, x2.z) Q5_HI(w0.w, qa.w, x2.w)
            Q5_HI(w1.x, qb.x, x3.x) Q5_HI(w1.y, qb.y, x3.y) Q5_HI(w1.z, qb.z, x3.z) Q5_HI(w1.w, qb.w, x3.w)
#undef Q5_LO
#undef Q5_HI
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
                if (msum_row) msum_row[c0 + sb] = msum;
            } else {
                acc += dd * (float)isum - dm * (float)msum;
            }
        }
    }
    return acc;
}

template <bool DOTS>
__device__ __forceinline__ float chunk_q6k(const uint8_t* slot, const uint16_t* dsec, const Act& a, int c0, int cb,
                                           int lane, int first, int stride, int32_t* isum_row) {
    float acc = 0.f;
    const int items = cb * 4;
    for (int base = first; base < items; base += stride) {
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
#define Q6K_WORD(Aw, Bw, Hw, X1, X2, X3, X4)                              \
    d1 = __dp4a((int)(((Aw) & m4) | (((Hw) << 4) & m2)), X1, d1);         \
    d2 = __dp4a((int)(((Bw) & m4) | (((Hw) << 2) & m2)), X2, d2);         \
    d3 = __dp4a((int)((((Aw) >> 4) & m4) | ((Hw) & m2)), X3, d3);         \
    d4 = __dp4a((int)((((Bw) >> 4) & m4) | (((Hw) >> 2) & m2)), X4, d4);
            Q6K_WORD(A.x, B.x, H.x, x1.x, x2.x, x3.x, x4.x)
            Q6K_WORD(A.y, B.y, H.y, x1.y, x2.y, x3.y, x4.y)
            Q6K_WORD(A.z, B.z, H.z, x1.z, x2.z, x3.z, x4.z)
            Q6K_WORD(A.w, B.w, H.w, x1.w, x2.w, x3.w, x4.w)
#undef Q6K_WORD
            // q is stored +32: sum (q-32)*x = sum q*x - 32 * bsum over the 16 elements
            const int16_t* bs = a.q8k_bs + (c0 + sb) * 16 + 8 * h + (l0 >> 4);
            d1 -= 32 * (int)bs[0];
            d2 -= 32 * (int)bs[2];
            d3 -= 32 * (int)bs[4];
            d4 -= 32 * (int)bs[6];
            isum = (int)sc[0] * d1 + (int)sc[2] * d2 + (int)sc[4] * d3 + (int)sc[6] * d4;
            if (t == 0 && !DOTS) dd = __fmul_rn(h2f(dsec[sb]), a.q8k_d[c0 + sb]);
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

// Q8_0: the warp reads the row chunk as consecutive 512-byte runs, lane l taking 16-byte
// vector l of each (half of 32-block l/2 of the run); the two lanes of a block add their
// integer sums.  Activations use the natural layout, which gives the same contiguous reads.
template <bool DOTS>
__device__ __forceinline__ float chunk_q80(const uint8_t* slot, const uint16_t* dsec, const Act& a, int c0, int cb,
                                           int lane, int32_t* isum_row) {
    float acc = 0.f;
    const int nvec = cb * 16;  // 16-byte vectors in the row chunk
    const int b0 = c0 * 8;     // first 32-block of the chunk
    const uint4* w = reinterpret_cast<const uint4*>(slot);
    const int4* x = reinterpret_cast<const int4*>(a.q80 + c0 * QK_K);
    for (int i0 = 0; i0 < nvec; i0 += 32) {
        const int i = i0 + lane;
        int sum = 0;
        if (i < nvec) {
            const uint4 wv = w[i];
            const int4 xv = x[i];
            sum = __dp4a((int)wv.x, xv.x, 0);
            sum = __dp4a((int)wv.y, xv.y, sum);
            sum = __dp4a((int)wv.z, xv.z, sum);
            sum = __dp4a((int)wv.w, xv.w, sum);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        if (i < nvec && (lane & 1) == 0) {
            const int b = i >> 1;
            if (DOTS) {
                isum_row[b0 + b] = sum;
            } else {
                // candle BlockQ8_0::vec_dot: sumi as f32 * d_w * d_x, left to right
                acc += __fmul_rn(__fmul_rn((float)sum, h2f(dsec[b])), a.q80_d[b0 + b]);
            }
        }
    }
    return acc;
}

// Four 1-bit values (bits 0..3 of v) spread to bit 0 of four bytes: bit k lands at 8k
// through the multiply (shifts 0, 7, 14, 21 give it position k + 7k).
__device__ __forceinline__ uint32_t spread4(uint32_t v) { return ((v & 0xfu) * 0x00204081u) & 0x01010101u; }

// Q4_0 / Q5_0 (device layout per super-block: the eight blocks' 16-byte qs, for Q5_0 then
// their 4-byte qh words; f16 d in the scale section): lane l takes 32-block l of each run of
// 32 blocks.  Element
// j < 16 of a block is the low nibble of qs[j] and pairs with activation j, element j + 16
// its high nibble with activation j + 16; Q5_0 adds bit j (j + 16) of qh as the 5th bit.
// The block's integer sum is sum(q * x) - off * sum(x) (off = 8 or 16), candle's
// sum((q - off) * x) exactly; its f32 contribution is candle's (sumi * d_w) * d_x.
// MIN (Q4_1 / Q5_1, (d, m) per block in the scale section): codes are unsigned, no offset, and
// candle adds m_w * s_x, where its Q8_1 activation's s = f16(f16(sum(x)) * d_x) (its quants
// and d equal Q8_0's, so the Q8_0 activation serves).
template <bool DOTS, bool Q5, bool MIN = false>
__device__ __forceinline__ float chunk_q40(const uint8_t* slot, const uint16_t* dsec, const Act& a, int c0, int cb,
                                           int lane, int32_t* isum_row) {
    float acc = 0.f;
    const int nblk = cb * 8;  // 32-blocks in the row chunk
    const int b0 = c0 * 8;
    const int4* x = reinterpret_cast<const int4*>(a.q80 + c0 * QK_K);
    const uint32_t lo = 0x0f0f0f0fu;
    for (int i0 = 0; i0 < nblk; i0 += 32) {
        const int b = i0 + lane;
        if (b >= nblk) continue;
        const uint8_t* sbp = slot + (b >> 3) * (Q5 ? 160 : 128);  // the block's super-block
        const uint4 wv = *reinterpret_cast<const uint4*>(sbp + 16 * (b & 7));
        const int4 xl = x[2 * b], xh = x[2 * b + 1];
        uint32_t l0 = wv.x & lo, l1 = wv.y & lo, l2 = wv.z & lo, l3 = wv.w & lo;
        uint32_t h0 = (wv.x >> 4) & lo, h1 = (wv.y >> 4) & lo, h2 = (wv.z >> 4) & lo, h3 = (wv.w >> 4) & lo;
        if (Q5) {
            const uint32_t hb = *reinterpret_cast<const uint32_t*>(sbp + 128 + 4 * (b & 7));
            l0 |= spread4(hb) << 4;
            l1 |= spread4(hb >> 4) << 4;
            l2 |= spread4(hb >> 8) << 4;
            l3 |= spread4(hb >> 12) << 4;
            h0 |= spread4(hb >> 16) << 4;
            h1 |= spread4(hb >> 20) << 4;
            h2 |= spread4(hb >> 24) << 4;
            h3 |= spread4(hb >> 28) << 4;
        }
        int s = dp4a_us(l0, xl.x, 0);
        s = dp4a_us(l1, xl.y, s);
        s = dp4a_us(l2, xl.z, s);
        s = dp4a_us(l3, xl.w, s);
        s = dp4a_us(h0, xh.x, s);
        s = dp4a_us(h1, xh.y, s);
        s = dp4a_us(h2, xh.z, s);
        s = dp4a_us(h3, xh.w, s);
        const int ones = 0x01010101;
        int sx = __dp4a(ones, xl.x, 0);
        sx = __dp4a(ones, xl.y, sx);
        sx = __dp4a(ones, xl.z, sx);
        sx = __dp4a(ones, xl.w, sx);
        sx = __dp4a(ones, xh.x, sx);
        sx = __dp4a(ones, xh.y, sx);
        sx = __dp4a(ones, xh.z, sx);
        sx = __dp4a(ones, xh.w, sx);
        if (MIN) {
            if (DOTS) {
                isum_row[b0 + b] = s;
            } else {
                const float dx = a.q80_d[b0 + b];
                const float s81 = __half2float(__float2half_rn(__fmul_rn(__half2float(__float2half_rn((float)sx)), dx)));
                acc += __fadd_rn(__fmul_rn(__fmul_rn((float)s, h2f(dsec[2 * b])), dx), __fmul_rn(h2f(dsec[2 * b + 1]), s81));
            }
            continue;
        }
        const int sum = s - (Q5 ? 16 : 8) * sx;
        if (DOTS) isum_row[b0 + b] = sum;
        else acc += __fmul_rn(__fmul_rn((float)sum, h2f(dsec[b])), a.q80_d[b0 + b]);
    }
    return acc;
}

__device__ __forceinline__ float chunk_f16(const uint8_t* slot, const Act& a, int c0, int cb, int lane, int first,
                                           int stride) {
    float acc = 0.f;
    const int units = cb * 32;  // 16-byte units (8 halfs)
    const float* x = a.f32 + c0 * QK_K;
    for (int base = first; base < units; base += stride) {
        const int u = base + lane;
        if (u >= units) continue;
        const uint4 w = *reinterpret_cast<const uint4*>(slot + u * 16);
        const float4 xa = *reinterpret_cast<const float4*>(x + u * 8);
        const float4 xb = *reinterpret_cast<const float4*>(x + u * 8 + 4);
        const __half2* h = reinterpret_cast<const __half2*>(&w);
        const float2 f0 = __half22float2(h[0]), f1 = __half22float2(h[1]), f2 = __half22float2(h[2]),
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

// Activation kernel, launched before every GEMV: optional RMSNorm (candle_nn::ops::rms_norm:
// m = sqrt(sum(x^2)/K + eps), y = x / m * w) and quantisation of the input into
// p.act_global, laid out exactly as the GEMV's shared-memory activation region, so that
// each GEMV CTA takes it with one bulk copy instead of quantising the vector itself.  One
// warp per 256-element block (lane l holds elements 8l .. 8l+7); with a norm every CTA also
// sums x^2 over the whole vector (each thread a strided set of float4, all in flight).
constexpr int kActWarps = 8;


__device__ __forceinline__ void load8(const float* src, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(src);
    const float4 b = *reinterpret_cast<const float4*>(src + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// candle Mlp: silu(w1 x) * (w3 x), silu(a) = a / (1 + exp(-a))
__device__ __forceinline__ float glu_val(float g, float u) { return __fmul_rn(__fdiv_rn(g, 1.f + expf(-g)), u); }

// Epoch of this use of the tensor-parallel slot (TpLink): read after the kernel's
// griddepcontrol.wait, so the current step's counter is visible.
__device__ __forceinline__ unsigned int tp_epoch(const GemvParams& p) {
    const TpLink& t = *p.tp;
    return (unsigned int)(*reinterpret_cast<volatile const int*>(t.step)) * (unsigned int)t.uses_per_step +
           (unsigned int)p.tp_use + 1u;
}

// 8 consecutive input elements at `off`: x, or with tp_gather x plus every rank's partial
// in rank order.  The partials are 64-bit (value | epoch) words that peers store into this
// rank's inbox; a word whose epoch is not yet the current one is read again (bounded; a
// word that never arrives sets TPTC_ERR_TIMEOUT and counts as 0).
template <bool GATHER>
__device__ __forceinline__ void act_in8(const GemvParams& p, int off, float (&v)[8]) {
    if (!GATHER) {
        load8(p.x + off, v);
        return;
    }
    const float4 a = __ldcg(reinterpret_cast<const float4*>(p.x + off));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(p.x + off + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    const TpLink& t = *p.tp;
    const unsigned int e = tp_epoch(p);
    const unsigned long long* in = t.inbox[t.rank] + (size_t)p.tp_slot * t.size * t.dim + off;
    for (int r = 0; r < t.size; r++) {
        const unsigned long long* src = in + (size_t)r * t.dim;
        unsigned long long w[8];
#pragma unroll
        for (int i = 0; i < 8; i += 2) ld_volatile_u64x2(src + i, w[i], w[i + 1]);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t n = 0;
            while ((unsigned int)(w[i] >> 32) != e) {
                // give up after wait_polls reads, or within 256 once any wait of the step has
                // (the error word is set: the peer is not coming)
                if (++n > t.wait_polls || ((n & 255) == 0 && p.err && *reinterpret_cast<volatile int*>(p.err))) {
                    if (p.err) atomicExch(p.err, TPTC_ERR_TIMEOUT);
                    w[i] = (unsigned long long)e << 32;  // value 0
                    break;
                }
                if (n > 64) __nanosleep(32);
                w[i] = ld_volatile_u64(src + i);
            }
            v[i] = __fadd_rn(v[i], __uint_as_float((unsigned int)(w[i] & 0xffffffffu)));
        }
    }
}

template <bool GATHER>
__device__ __forceinline__ void act_quant_body(const GemvParams& p, int transposed, float* red) {
    const int K = p.K, nb = K / QK_K, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = blockIdx.x * kActWarps + warp;
    const bool norm = p.norm_w != nullptr, mine = b < nb;
    // the norm weights do not depend on the previous kernel: load them before waiting for it
    float v[8], w8[8];
    if (mine && norm) load8(p.norm_w + b * QK_K + 8 * lane, w8);
    pdl_wait();
    pdl_launch_dependents();
    // then every load of x goes out before the first use: this warp's block and, with a
    // norm, this thread's share of the sum of squares
    if (mine) act_in8<GATHER>(p, b * QK_K + 8 * lane, v);
    if (mine && GATHER) {  // the reduced residual stream, for the next projection's residual
        float4* xo = reinterpret_cast<float4*>(p.x_out + b * QK_K + 8 * lane);
        xo[0] = make_float4(v[0], v[1], v[2], v[3]);
        xo[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (norm) {
        static_assert(kActWarps == kNormWarps, "the activation kernel uses the chains' norm partition");
        // every CTA sums the whole vector in the shared partition (blocks warp, warp + 8, ...),
        // the first kHold blocks of the warp loaded together before any is summed
        constexpr int kHold = 4;
        float ss = 0.f;
        if (!p.glu_in) {
            float xv[kHold][8];
#pragma unroll
            for (int j = 0; j < kHold; j++)
                if (warp + j * kActWarps < nb) act_in8<GATHER>(p, (warp + j * kActWarps) * QK_K + 8 * lane, xv[j]);
#pragma unroll
            for (int j = 0; j < kHold; j++)
                if (warp + j * kActWarps < nb) ss = __fadd_rn(ss, sumsq8(xv[j]));
        }
        for (int bb = p.glu_in ? warp : warp + kHold * kActWarps; bb < nb; bb += kActWarps) {
            float xv[8];
            act_in8<GATHER>(p, bb * QK_K + 8 * lane, xv);
            if (p.glu_in) {
                float u[8];
                load8(p.x + K + bb * QK_K + 8 * lane, u);
#pragma unroll
                for (int i = 0; i < 8; i++) xv[i] = glu_val(xv[i], u[i]);
            }
            ss = __fadd_rn(ss, sumsq8(xv));
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kActWarps; w++) tot = __fadd_rn(tot, red[w]);
        const float m = sqrtf(__fdiv_rn(tot, (float)K) + p.eps);
        if (mine) {
            if (p.glu_in) {
                float u[8];
                load8(p.x + K + b * QK_K + 8 * lane, u);
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = glu_val(v[i], u[i]);
            }
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fdiv_rn(v[i], m), w8[i]);
        }
    } else if (mine && p.glu_in) {
        float u[8];
        load8(p.x + K + b * QK_K + 8 * lane, u);
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = glu_val(v[i], u[i]);
    }
    if (b >= nb) return;
    act_store_block(p.act, transposed, nb, p.act_global, b, v, lane);
}

// The activation kernel; with tp_gather (tensor parallelism) its input is x plus every rank's
// partial rows (act_in8), written back as the reduced residual stream.  Two kernels so that
// each gets its own register allocation.
template <bool GATHER>
__global__ void __launch_bounds__(kActWarps * 32) act_quant_kernel(const __grid_constant__ GemvParams p, int transposed) {
    __shared__ float red[kActWarps];
    act_quant_body<GATHER>(p, transposed, red);
}

// A CTA's weight ring: S stages of stage_bytes after the activation region, with their
// "full" (copy landed) and "empty" (every consumer warp done) mbarriers.  Producer and
// consumers walk it with the same position (stage s, wrap count lap: parity source).
struct Ring {
    uint8_t* base;
    int stage_bytes, S;
    uint64_t* full;
    uint64_t* empty;
};

// Bounded wait that yields between polls and gives up early once the CTA has aborted.
__device__ __forceinline__ bool wait_backoff_abort(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 15 && *abort_flag) return false;
        __nanosleep(64);
    }
    if (err) atomicExch(err, TPTC_ERR_TIMEOUT);
    *abort_flag = 1;
    return false;
}

__device__ __forceinline__ bool wait_abort(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 15 && *abort_flag) return false;
    }
    if (err) atomicExch(err, TPTC_ERR_TIMEOUT);
    *abort_flag = 1;
    return false;
}

// Producer lane: the weight tiles of this CTA's units of GEMV p, one bulk copy per stage,
// in the order the consumers take them -- units in pairs (u, u + grid) chunk by chunk
// alternating when unit_pair holds, a single unit alone otherwise.  Weights do not depend on
// any earlier kernel or phase, so this runs ahead of every wait the consumers do (expert
// weights excepted: which expert is read depends on the routing kernel).  Returns
// false once a wait for a free stage gave up (or the CTA aborted).
template <bool WIDE>
__device__ bool produce_units(const GemvParams& p, int epi, const Ring& r, int& s, int& lap, uint64_t policy,
                              volatile int* abort_flag) {
    const int nsb = p.K / QK_K;
    const SegOff eo = expert_offsets(p);
    for (int u = blockIdx.x; u < p.units;) {
        const bool two = unit_pair(p, u, epi);
        for (int i = 0; i < (two ? 2 : 1) * p.nchunks; i++) {
            const int c = two ? i >> 1 : i, k = two ? i & 1 : 0;
            const int uk = u + k * gridDim.x, s_ = unit_seg(p, uk);
            const DevMatrix& m = p.seg[s_].m;
            const int sbb = k_sb_bytes<WIDE>(m.type);
            const int64_t tile0 = (int64_t)(uk - p.seg[s_].unit_begin) * kTileRows * m.main_row_bytes;
            if (lap > 0 && !wait_backoff_abort(&r.empty[s], (lap - 1) & 1, p.err, abort_flag)) return false;
            const int cb = min(p.cbs, nsb - c * p.cbs);
            const uint32_t bytes = (uint32_t)(kTileRows * cb * sbb);
            mbar_expect_tx(&r.full[s], bytes);
            bulk_g2s(r.base + s * r.stage_bytes, m.main + seg_off(eo, s_) + tile0 + (int64_t)c * kTileRows * p.cbs * sbb, bytes,
                     &r.full[s], policy);
            if (++s == r.S) {
                s = 0;
                lap++;
            }
        }
        u += (two ? 2 : 1) * gridDim.x;
    }
    return true;
}

// Producer lane after an abort, before the CTA may exit: every copy it issued has landed
// (bounded).  Without an abort the consumers wait for every stage, so the producer returns
// at once and takes no issue slots from them.
__device__ void drain_ring(const Ring& r, int s, int lap, volatile int* abort_flag) {
    if (!*abort_flag) return;
    const int n = lap * r.S + s;  // stages issued
    for (int j = n > r.S ? n - r.S : 0; j < n; j++) mbar_wait_backoff(&r.full[j % r.S], (j / r.S) & 1, nullptr);
}

__device__ __forceinline__ Act act_view(const ActLayout& L, const uint8_t* smem) {
    Act a;
    a.f32 = L.f32 >= 0 ? reinterpret_cast<const float*>(smem + L.f32) : nullptr;
    a.q8k = L.q8k >= 0 ? reinterpret_cast<const int8_t*>(smem + L.q8k) : nullptr;
    a.q8k_d = L.q8k >= 0 ? reinterpret_cast<const float*>(smem + L.q8k_d) : nullptr;
    a.q8k_bs = L.q8k >= 0 ? reinterpret_cast<const int16_t*>(smem + L.q8k_bs) : nullptr;
    a.q8k_ps = L.q8k >= 0 ? reinterpret_cast<const int16_t*>(smem + L.q8k_ps) : nullptr;
    a.q80 = L.q80 >= 0 ? reinterpret_cast<const int8_t*>(smem + L.q80) : nullptr;
    a.q80_d = L.q80 >= 0 ? reinterpret_cast<const float*>(smem + L.q80_d) : nullptr;
    return a;
}

// EPI_RESID of a mixture-of-experts down projection, candle's MlpOrMoe::MoE order: ys starts
// at zero, each selected expert in ascending expert order adds its output times its routing
// weight (index_add of broadcast_mul), a shared expert adds its output, then x = ys + x.
__device__ __forceinline__ void moe_resid(const GemvParams& p, int row, float y) {
    const float a = __fmul_rn(y, p.moe_slot >= 0 ? __ldcg(p.moe_w + p.moe_slot) : 1.f);
    const float acc = p.moe_first ? a : __fadd_rn(__ldcg(p.moe_acc + row), a);
    if (p.moe_last) p.out[row] = __fadd_rn(acc, __ldcg(p.out + row));
    else p.moe_acc[row] = acc;
}

// Running greedy pick of the rows a warp wrote (lane 0): candle sample_argmax keeps the last
// of equal maxima, so ties go to the higher row.
struct ArgBest {
    float v;
    int i;
};
__device__ __forceinline__ void argbest_take(ArgBest& b, float v, int i) {
    if (b.i < 0 || v > b.v || (v == b.v && i > b.i)) {
        b.v = v;
        b.i = i;
    }
}

// One row chunk of one unit on its own (DOTS test hook, mixed types, Q8_0, F16, and every
// format beyond Q4_K / Q6_K).  Kernels built with WIDE = false carry only Q4_K, Q6_K, Q8_0
// and F16: the other formats' code would raise the register pressure of the whole kernel
// (more spills in the Q4_K / Q6_K loop), so a launch takes the WIDE build only when one of
// its matrices needs it.
template <int EPI, bool WIDE>
__device__ __forceinline__ float single_chunk(const GemvParams& p, const Act& a, const DevMatrix& m,
                                              const UnitRow& ur, const uint8_t* stage, int c0, int cb,
                                              int lane, int warp) {
    const int nsb = p.K / QK_K;
    if (ur.seg < 0) return 0.f;
    const int sbm = k_sb_main<WIDE>(m.type), sbd = k_sb_d<WIDE>(m.type);
    const uint8_t* slot = stage + warp * cb * sbm;
    const uint16_t* dsec = reinterpret_cast<const uint16_t*>(stage + kTileRows * cb * sbm + warp * cb * sbd);
    int32_t* isum_row = nullptr;
    int32_t* msum_row = nullptr;
    if (EPI == EPI_DOTS) {
        const int per_row = type_q80_family(m.type) ? p.K / QK8_0 : nsb;
        isum_row = p.isum + (int64_t)ur.row * per_row;
        msum_row = p.msum ? p.msum + (int64_t)ur.row * per_row : nullptr;
    }
    if constexpr (WIDE) {
        switch (m.type) {
        case TPTC_TYPE_Q5_K:
            if (EPI == EPI_DOTS) {
                chunk_q5k<true>(slot, a, c0, cb, lane, 0, 32, isum_row, msum_row);
            } else if (lane < 2 * cb) {
                XHalf xh;
                load_xhalf<false>(xh, a, c0, 2 * cb, lane);
                return q5k_half(slot, xh, lane);
            }
            return 0.f;
        case TPTC_TYPE_Q2_K:
        case TPTC_TYPE_Q3_K:
            if (EPI == EPI_DOTS) {
                if (m.type == TPTC_TYPE_Q2_K) dots_q23k<TPTC_TYPE_Q2_K>(slot, dsec, a, c0, cb, lane, isum_row, msum_row);
                else dots_q23k<TPTC_TYPE_Q3_K>(slot, dsec, a, c0, cb, lane, isum_row, msum_row);
            } else if (lane < 2 * cb) {
                XHalf xh;
                load_xhalf<true>(xh, a, c0, 2 * cb, lane);
                return m.type == TPTC_TYPE_Q2_K ? q2k_half(slot, dsec, xh, lane) : q3k_half(slot, dsec, xh, lane);
            }
            return 0.f;
        case TPTC_TYPE_Q4_0: return chunk_q40<EPI == EPI_DOTS, false>(slot, dsec, a, c0, cb, lane, isum_row);
        case TPTC_TYPE_Q5_0: return chunk_q40<EPI == EPI_DOTS, true>(slot, dsec, a, c0, cb, lane, isum_row);
        case TPTC_TYPE_Q4_1: return chunk_q40<EPI == EPI_DOTS, false, true>(slot, dsec, a, c0, cb, lane, isum_row);
        case TPTC_TYPE_Q5_1: return chunk_q40<EPI == EPI_DOTS, true, true>(slot, dsec, a, c0, cb, lane, isum_row);
        default: break;
        }
    }
    switch (m.type) {
    case TPTC_TYPE_Q4_K:
        if (EPI == EPI_DOTS) {
            chunk_q4k<true>(slot, a, c0, cb, lane, 0, 32, isum_row, msum_row);
        } else if (lane < 2 * cb) {
            XHalf xh;
            load_xhalf<false>(xh, a, c0, 2 * cb, lane);
            return q4k_half(slot, xh, lane);
        }
        return 0.f;
    case TPTC_TYPE_Q6_K:
        if (EPI == EPI_DOTS) {
            chunk_q6k<true>(slot, dsec, a, c0, cb, lane, 0, 32, isum_row);
        } else if (lane < 2 * cb) {
            XHalf xh;
            load_xhalf<true>(xh, a, c0, 2 * cb, lane);
            return q6k_half(slot, dsec, xh, lane);
        }
        return 0.f;
    case TPTC_TYPE_Q8_0: return chunk_q80<EPI == EPI_DOTS>(slot, dsec, a, c0, cb, lane, isum_row);
    default: return chunk_f16(slot, a, c0, cb, lane, 0, 32);
    }
}

// Consumer warps: this CTA's units of GEMV p from the ring, one warp per tile row.  Units in
// pairs (u, u + grid): for every chunk the producer filled the pair's two stages back to back
// and a warp reduces its row of both in one pass; with the same weight type the two dot
// products share the lane's activation slice (same columns).  Once a wait gives up the warps
// skip the arithmetic but keep the loop's barriers (the gate|up pair barrier) and stage
// releases, so every warp leaves together.  `best` (EPI_STORE): argmax of the rows written.
template <int EPI, bool WIDE>
__device__ __forceinline__ void consume_units(const GemvParams& p, const Act& a, const Ring& r, int& s, int& lap,
                                              int& unit_no, float (&glu_up)[2][4], ArgBest* best,
                                              volatile int* abort_flag, bool& timed_out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nsb = p.K / QK_K;
    auto epilogue = [&](const UnitRow& ur, float acc) {
        if (EPI == EPI_DOTS) return;
        const float y = warp_sum(acc);
        if (EPI == EPI_GLU) {
            // tile rows 0-3 are gate rows, 4-7 the matching up rows: the up warp hands its
            // value to the gate warp through shared memory (double-buffered by unit parity,
            // one two-warp named barrier per unit), which writes silu(gate) * up
            const int buf = unit_no & 1;
            if (warp >= 4 && lane == 0) glu_up[buf][warp - 4] = y;
            pair_sync(warp & 3);
            if (warp < 4 && lane == 0 && ur.seg >= 0 && !timed_out)
                p.out[ur.out] = p.glu_act ? gelu_tanh_mul(y, glu_up[buf][warp])
                                          : __fmul_rn(__fdiv_rn(y, 1.f + expf(-y)), glu_up[buf][warp]);
            unit_no++;
            return;
        }
        if (lane != 0 || ur.seg < 0 || timed_out) return;
        if (EPI == EPI_STORE) {
            p.out[ur.row] = y;
            if (best) argbest_take(*best, y, ur.row);
        } else if (EPI == EPI_RESID) {
            if (p.tp) {  // this rank's partial row, tagged, into every rank's inbox (peer stores)
                const TpLink& t = *p.tp;
                const size_t at = ((size_t)p.tp_slot * t.size + t.rank) * t.dim + ur.out;
                const unsigned long long w = ((unsigned long long)tp_epoch(p) << 32) | __float_as_uint(y);
                for (int r = 0; r < t.size; r++) st_volatile_u64(t.inbox[r] + at, w);
            } else if (p.moe_acc) {
                moe_resid(p, ur.out, y);
            } else {
                p.out[ur.out] = __ldcg(p.out + ur.out) + y;
            }
        } else if (EPI == EPI_QKV) {
            const float* bias = p.bias[ur.seg];
            const float yb = bias ? __fadd_rn(y, bias[ur.row]) : y;  // candle QLinear: matmul, then + bias
            if (ur.seg == 0) {
                p.out[ur.row] = yb;  // q before RoPE
            } else if (ur.seg == 1) {
                p.kraw[ur.row] = yb;  // k before RoPE
            } else {
                const int pos = *p.pos, d = ur.row % p.hd, head = ur.row / p.hd;
                const int64_t at = ((int64_t)head * p.max_seq + pos) * p.hd + d;
                if (p.kv_f32) static_cast<float*>(p.vcache)[at] = yb;
                else static_cast<__half*>(p.vcache)[at] = __float2half_rn(yb);
            }
        }
    };
    // one row chunk of one unit on its own (DOTS test hook, mixed types, Q8_0, F16)
    auto single = [&](const DevMatrix& m, const UnitRow& ur, const uint8_t* stage, int c0, int cb) -> float {
        return single_chunk<EPI, WIDE>(p, a, m, ur, stage, c0, cb, lane, warp);
    };
    for (int u = blockIdx.x; u < p.units;) {
        const int u2 = u + gridDim.x;
        const bool two = unit_pair(p, u, EPI);
        const UnitRow ra = unit_row(p, u, warp);
        const UnitRow rb = unit_row(p, two ? u2 : u, warp);
        const DevMatrix& ma = p.seg[unit_seg(p, u)].m;
        const DevMatrix& mb = p.seg[unit_seg(p, two ? u2 : u)].m;
        const int ty = ma.type;
        float acca = 0.f, accb = 0.f;
        for (int c = 0; c < p.nchunks; c++) {
            const int sa = s;
            if (!timed_out && !wait_abort(&r.full[sa], lap & 1, p.err, abort_flag)) timed_out = true;
            if (++s == r.S) {
                s = 0;
                lap++;
            }
            int sb2 = sa;
            if (two) {
                sb2 = s;
                if (!timed_out && !wait_abort(&r.full[sb2], lap & 1, p.err, abort_flag)) timed_out = true;
                if (++s == r.S) {
                    s = 0;
                    lap++;
                }
            }
            if (!timed_out) {
                const int c0 = c * p.cbs, cb = min(p.cbs, nsb - c0);
                const uint8_t* stA = r.base + sa * r.stage_bytes;
                const uint8_t* stB = r.base + sb2 * r.stage_bytes;
                if (two) {
                    if (lane < 2 * cb) {
                        const int sbm = k_sb_main<false>(ty), sbd = k_sb_d<false>(ty);
                        XHalf xh;
                        if (ty == TPTC_TYPE_Q4_K) {
                            load_xhalf<false>(xh, a, c0, 2 * cb, lane);
                            acca += q4k_half(stA + warp * cb * sbm, xh, lane);
                            accb += q4k_half(stB + warp * cb * sbm, xh, lane);
                        } else {
                            load_xhalf<true>(xh, a, c0, 2 * cb, lane);
                            const int doff = kTileRows * cb * sbm + warp * cb * sbd;
                            acca += q6k_half(stA + warp * cb * sbm, reinterpret_cast<const uint16_t*>(stA + doff), xh, lane);
                            accb += q6k_half(stB + warp * cb * sbm, reinterpret_cast<const uint16_t*>(stB + doff), xh, lane);
                        }
                    }
                } else {
                    acca += single(ma, ra, stA, c0, cb);
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&r.empty[sa]);
                if (two) mbar_arrive(&r.empty[sb2]);
            }
        }
        epilogue(ra, acca);
        if (two) epilogue(rb, accb);
        u += (two ? 2 : 1) * gridDim.x;
    }
}

// The standalone GEMV (one launch per projection), written out in one body: the ring
// bookkeeping and the unit loop inline here measured faster than the shared
// produce_units / consume_units the chain kernel uses.
template <int EPI, bool WIDE>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kGemvMaxStages], empty[kGemvMaxStages], actbar;
    __shared__ float glu_up[2][4];
    int unit_no = 0;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = p.stages;
    const int nsb = p.K / QK_K;
    uint8_t* ring = smem + p.act.bytes;

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(&actbar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer: one bulk copy per stage (a whole 8-row tile), weights
        // only, so it runs ahead of griddepcontrol.wait
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            int s = 0, lap = 0;  // ring stage and how many times the ring has wrapped
            const SegOff eo = expert_offsets(p);
            // units in pairs (u, u + grid), chunk by chunk: the order the consumers take them
            for (int u = blockIdx.x; u < p.units;) {
                const bool two = unit_pair(p, u, EPI);
                // a pair goes chunk by chunk alternating its two units; a single unit alone
                for (int i = 0; i < (two ? 2 : 1) * p.nchunks; i++) {
                    const int c = two ? i >> 1 : i, k = two ? i & 1 : 0;
                    {
                        const int uk = u + k * gridDim.x, s_ = unit_seg(p, uk);
                        const DevMatrix& m = p.seg[s_].m;
                        const int sbb = k_sb_bytes<WIDE>(m.type);
                        const int64_t tile0 = (int64_t)(uk - p.seg[s_].unit_begin) * kTileRows * m.main_row_bytes;
                        if (lap > 0 && !mbar_wait_backoff(&empty[s], (lap - 1) & 1, p.err)) return;
                        const int cb = min(p.cbs, nsb - c * p.cbs);
                        const uint32_t bytes = (uint32_t)(kTileRows * cb * sbb);
                        mbar_expect_tx(&full[s], bytes);
                        bulk_g2s(ring + s * p.stage_bytes, m.main + seg_off(eo, s_) + tile0 + (int64_t)c * kTileRows * p.cbs * sbb, bytes,
                                 &full[s], policy);
                        if (++s == S) {
                            s = 0;
                            lap++;
                        }
                    }
                }
                u += (two ? 2 : 1) * gridDim.x;
            }
        }
        return;
    }

    // ---------------- consumers: one warp per tile row
    pdl_wait();
    // The next kernel may start (and prefetch its weights) only once this one is past its
    // own wait, so at most two kernels of a chain overlap.
    pdl_launch_dependents();
    // the activation, prepared by act_quant_kernel in this region's layout: one bulk copy
    if (tid == 0) {
        mbar_expect_tx(&actbar, (uint32_t)p.act.bytes);
        bulk_g2s(smem, p.act_global, (uint32_t)p.act.bytes, &actbar, 0);
    }
    bool timed_out = !mbar_wait_bounded(&actbar, 0, p.err);

    Act a;
    a.f32 = p.act.f32 >= 0 ? reinterpret_cast<const float*>(smem + p.act.f32) : nullptr;
    a.q8k = p.act.q8k >= 0 ? reinterpret_cast<const int8_t*>(smem + p.act.q8k) : nullptr;
    a.q8k_d = p.act.q8k >= 0 ? reinterpret_cast<const float*>(smem + p.act.q8k_d) : nullptr;
    a.q8k_bs = p.act.q8k >= 0 ? reinterpret_cast<const int16_t*>(smem + p.act.q8k_bs) : nullptr;
    a.q8k_ps = p.act.q8k >= 0 ? reinterpret_cast<const int16_t*>(smem + p.act.q8k_ps) : nullptr;
    a.q80 = p.act.q80 >= 0 ? reinterpret_cast<const int8_t*>(smem + p.act.q80) : nullptr;
    a.q80_d = p.act.q80 >= 0 ? reinterpret_cast<const float*>(smem + p.act.q80_d) : nullptr;

    // Units in pairs (u, u + grid): for every chunk the producer fills the pair's two stages
    // back to back, and a warp reduces its row of both in one pass; with the same weight type
    // the two dot products share the lane's activation slice (same columns).
    int s = 0, lap = 0;  // ring stage and its phase parity source
    auto epilogue = [&](const UnitRow& ur, float acc) {
        if (EPI == EPI_DOTS) return;
        const float y = warp_sum(acc);
        if (EPI == EPI_GLU) {
            // tile rows 0-3 are gate rows, 4-7 the matching up rows: the up warp hands its
            // value to the gate warp through shared memory (double-buffered by unit parity,
            // one two-warp named barrier per unit), which writes silu(gate) * up
            const int buf = unit_no & 1;
            if (warp >= 4 && lane == 0) glu_up[buf][warp - 4] = y;
            pair_sync(warp & 3);
            if (warp < 4 && lane == 0 && ur.seg >= 0)
                p.out[ur.out] = p.glu_act ? gelu_tanh_mul(y, glu_up[buf][warp])
                                          : __fmul_rn(__fdiv_rn(y, 1.f + expf(-y)), glu_up[buf][warp]);
            unit_no++;
            return;
        }
        if (lane != 0 || ur.seg < 0) return;
        if (EPI == EPI_STORE) {
            p.out[ur.row] = y;
        } else if (EPI == EPI_RESID) {
            if (p.tp) {  // this rank's partial row, tagged, into every rank's inbox (peer stores)
                const TpLink& t = *p.tp;
                const size_t at = ((size_t)p.tp_slot * t.size + t.rank) * t.dim + ur.out;
                const unsigned long long w = ((unsigned long long)tp_epoch(p) << 32) | __float_as_uint(y);
                for (int r = 0; r < t.size; r++) st_volatile_u64(t.inbox[r] + at, w);
            } else if (p.moe_acc) {
                moe_resid(p, ur.out, y);
            } else {
                p.out[ur.out] += y;
            }
        } else if (EPI == EPI_QKV) {
            const float* bias = p.bias[ur.seg];
            const float yb = bias ? __fadd_rn(y, bias[ur.row]) : y;  // candle QLinear: matmul, then + bias
            if (ur.seg == 0) {
                p.out[ur.row] = yb;  // q before RoPE
            } else if (ur.seg == 1) {
                p.kraw[ur.row] = yb;  // k before RoPE
            } else {
                const int pos = *p.pos, d = ur.row % p.hd, head = ur.row / p.hd;
                const int64_t at = ((int64_t)head * p.max_seq + pos) * p.hd + d;
                if (p.kv_f32) static_cast<float*>(p.vcache)[at] = yb;
                else static_cast<__half*>(p.vcache)[at] = __float2half_rn(yb);
            }
        }
    };
    // one row chunk of one unit on its own (DOTS test hook, mixed types, Q8_0, F16)
    auto single = [&](const DevMatrix& m, const UnitRow& ur, const uint8_t* stage, int c0, int cb) -> float {
        return single_chunk<EPI, WIDE>(p, a, m, ur, stage, c0, cb, lane, warp);
    };
    for (int u = blockIdx.x; u < p.units;) {
        const int u2 = u + gridDim.x;
        const bool two = unit_pair(p, u, EPI);
        const UnitRow ra = unit_row(p, u, warp);
        const UnitRow rb = unit_row(p, two ? u2 : u, warp);
        const DevMatrix& ma = p.seg[unit_seg(p, u)].m;
        const DevMatrix& mb = p.seg[unit_seg(p, two ? u2 : u)].m;
        const int ty = ma.type;
        const bool paired = two;
        float acca = 0.f, accb = 0.f;
        for (int c = 0; c < p.nchunks; c++) {
            const int sa = s;
            if (!timed_out && !mbar_wait_bounded(&full[sa], lap & 1, p.err)) timed_out = true;
            if (++s == S) {
                s = 0;
                lap++;
            }
            int sb2 = sa;
            if (two) {
                sb2 = s;
                if (!timed_out && !mbar_wait_bounded(&full[sb2], lap & 1, p.err)) timed_out = true;
                if (++s == S) {
                    s = 0;
                    lap++;
                }
            }
            if (!timed_out) {
                const int c0 = c * p.cbs, cb = min(p.cbs, nsb - c0);
                const uint8_t* stA = ring + sa * p.stage_bytes;
                const uint8_t* stB = ring + sb2 * p.stage_bytes;
                if (paired) {
                    if (lane < 2 * cb) {
                        const int sbm = k_sb_main<false>(ty), sbd = k_sb_d<false>(ty);
                        XHalf xh;
                        if (ty == TPTC_TYPE_Q4_K) {
                            load_xhalf<false>(xh, a, c0, 2 * cb, lane);
                            acca += q4k_half(stA + warp * cb * sbm, xh, lane);
                            accb += q4k_half(stB + warp * cb * sbm, xh, lane);
                        } else {
                            load_xhalf<true>(xh, a, c0, 2 * cb, lane);
                            const int doff = kTileRows * cb * sbm + warp * cb * sbd;
                            acca += q6k_half(stA + warp * cb * sbm, reinterpret_cast<const uint16_t*>(stA + doff), xh, lane);
                            accb += q6k_half(stB + warp * cb * sbm, reinterpret_cast<const uint16_t*>(stB + doff), xh, lane);
                        }
                    }
                } else {
                    acca += single(ma, ra, stA, c0, cb);
                    if (two) accb += single(mb, rb, stB, c0, cb);
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty[sa]);
                if (two) mbar_arrive(&empty[sb2]);
            }
        }
        epilogue(ra, acca);
        if (two) epilogue(rb, accb);
        u += (two ? 2 : 1) * gridDim.x;
    }
}

// ---------------------------------------------------------------- GEMV chains
//
// A chain runs several GEMVs of a decode step in one persistent launch (o_proj, gate|up,
// down, the next layer's q|k|v or the lm_head): between phases every CTA arrives on a global
// counter and waits (bounded) until all have, then builds the next phase's activation
// itself from the vector the previous phase completed (RMSNorm + quantisation, the
// arithmetic of act_quant_kernel).  The producer warp streams weights across the phase
// boundaries without waiting for them, so the HBM stream does not drain between GEMVs.

__device__ __forceinline__ bool consumer_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kConsumers)
        : "memory");
    return r != 0;
}

// Bounded wait until *ctr >= target (acquire).  Gives up after kWaitPolls polls.
__device__ __forceinline__ bool spin_count(const int* ctr, int target, int* err, volatile int* abort_flag) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        int v;
        asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
        if (v >= target) return true;
        if (*abort_flag) return false;
        if (i > 4096) __nanosleep(64);
    }
    if (err) atomicExch(err, TPTC_ERR_TIMEOUT);
    return false;
}

// Phase activation built by the CTA's consumers from p.x (written before the phase barrier,
// read through L2): optional RMSNorm with p.norm_w and quantisation into `act` in p.act's
// layout, with the norm partition and arithmetic of act_quant_kernel (same m, same codes).
// Vectors of up to 32 blocks are read once and held in registers (one L2 round trip); the
// norm gains, which no phase writes, are fetched before the caller's barrier (w_pre).
constexpr int kActHold = 2;  // blocks per warp held in registers (K <= 4096 in one pass)
__device__ __forceinline__ void prefetch_norm(const GemvParams& p, float (&w_pre)[kActHold][8]) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nb = p.K / QK_K;
    if (!p.norm_w) return;
#pragma unroll
    for (int j = 0; j < kActHold; j++) {
        const int b = warp + j * kConsumerWarps;
        if (b < nb) load8(p.norm_w + b * QK_K + 8 * lane, w_pre[j]);
    }
}

__device__ __forceinline__ void ldcg8(const float* src, float (&v)[8]) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(src + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// x / m rounded to nearest, given rm = 1 / m rounded to nearest (__frcp_rn): a product and
// one fused correction step (Markstein's final division step, P. Markstein, IBM J. Res.
// Dev. 34(1), 1990), correctly rounded for finite operands whose quotient does not
// underflow.  Replaces one __fdiv_rn per element where a whole vector is divided by the
// same m; the chain-vs-activation-kernel bit-identity test compares the two on every value.
__device__ __forceinline__ float div_by(float x, float m, float rm) {
    const float q = __fmul_rn(x, rm);
    const float e = __fmaf_rn(-q, m, x);
    return __fmaf_rn(e, rm, q);
}

__device__ void build_act_local(const GemvParams& p, uint8_t* act, float* red, const float (&w_pre)[kActHold][8]) {
    const int K = p.K, nb = K / QK_K, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool norm = p.norm_w != nullptr;
    // this warp's blocks: warp, warp + 8, ... (nbw of them), the first kActHold in registers
    const int nbw = nb > warp ? (nb - warp + kConsumerWarps - 1) / kConsumerWarps : 0;
    float v[kActHold][8];
#pragma unroll
    for (int j = 0; j < kActHold; j++)
        if (j < nbw) ldcg8(p.x + (warp + j * kConsumerWarps) * QK_K + 8 * lane, v[j]);
    float m = 1.f, rm = 1.f;
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kActHold; j++)
            if (j < nbw) ss = __fadd_rn(ss, sumsq8(v[j]));
        for (int j = kActHold; j < nbw; j++) {  // vectors over 32 blocks
            float t[8];
            ldcg8(p.x + (warp + j * kConsumerWarps) * QK_K + 8 * lane, t);
            ss = __fadd_rn(ss, sumsq8(t));
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        consumer_sync();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) tot = __fadd_rn(tot, red[w]);
        m = sqrtf(__fdiv_rn(tot, (float)K) + p.eps);
        rm = __frcp_rn(m);
#pragma unroll
        for (int j = 0; j < kActHold; j++)
            if (j < nbw)
#pragma unroll
                for (int i = 0; i < 8; i++) v[j][i] = __fmul_rn(div_by(v[j][i], m, rm), w_pre[j][i]);
    }
    // the held blocks, two at a time (a missing partner is skipped by its index)
#pragma unroll
    for (int j = 0; j < kActHold; j += 2) {
        if (j < nbw) {
            const int bb[2] = {warp + j * kConsumerWarps, j + 1 < nbw ? warp + (j + 1) * kConsumerWarps : nb};
            act_store_blocks<2>(p.act, 1, nb, act, bb, *reinterpret_cast<const float(*)[2][8]>(&v[j]), lane);
        }
    }
    // blocks beyond the held ones, two at a time
    for (int j = kActHold; j < nbw; j += 2) {
        const int bb[2] = {warp + j * kConsumerWarps, j + 1 < nbw ? warp + (j + 1) * kConsumerWarps : nb};
        float t[2][8];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            if (bb[k] < nb) {
                ldcg8(p.x + bb[k] * QK_K + 8 * lane, t[k]);
                if (norm) {
                    float w8[8];
                    load8(p.norm_w + bb[k] * QK_K + 8 * lane, w8);
#pragma unroll
                    for (int i = 0; i < 8; i++) t[k][i] = __fmul_rn(div_by(t[k][i], m, rm), w8[i]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) t[k][i] = 0.f;
            }
        }
        act_store_blocks<2>(p.act, 1, nb, act, bb, t, lane);
    }
}

template <bool WIDE>
__global__ void __launch_bounds__(kThreads, 2) gemv_chain_kernel(const __grid_constant__ ChainParams c) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kGemvMaxStages], empty[kGemvMaxStages], actbar;
    __shared__ float glu_up[2][4];
    __shared__ float red[kConsumerWarps];
    __shared__ int redi[kConsumerWarps];
    __shared__ volatile int abort_flag;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const Ring r{smem + c.act_bytes, c.stage_bytes, c.stages, full, empty};

    if (tid == 0) {
        for (int s = 0; s < r.S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(&actbar, 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        if (lane == 0) {
            int s = 0, lap = 0;
            const uint64_t policy = l2_evict_first_policy();
            for (int ph = 0; ph < c.nph; ph++)
                if (!produce_units<WIDE>(c.ph[ph], c.epi[ph], r, s, lap, policy, &abort_flag)) break;
            drain_ring(r, s, lap, &abort_flag);
        }
        return;
    }

    pdl_wait();
    int s = 0, lap = 0, unit_no = 0;
    uint32_t actphase = 0;
    bool timed_out = false;
    ArgBest best{-INFINITY, -1};
    for (int ph = 0; ph < c.nph; ph++) {
        const GemvParams& p = c.ph[ph];
        if (ph == c.nph - 1) pdl_launch_dependents();
        float w_pre[kActHold][8];
        if (!p.act_prepared) prefetch_norm(p, w_pre);
        if (ph > 0) {  // every CTA has finished the previous phase
            bool bad = false;
            if (tid == 0) bad = !spin_count(c.bar + ph - 1, gridDim.x, c.err, &abort_flag);
            if (consumer_sync_or(bad || abort_flag)) {
                abort_flag = 1;  // the producer stops at its next wait
                timed_out = true;
                break;
            }
        }
        if (p.act_prepared) {  // written by the previous kernel in this layout: one bulk copy
            if (tid == 0) {
                mbar_expect_tx(&actbar, (uint32_t)p.act.bytes);
                bulk_g2s(smem, p.act_global, (uint32_t)p.act.bytes, &actbar, 0);
            }
            if (!wait_abort(&actbar, actphase & 1, c.err, &abort_flag)) abort_flag = 1;
            actphase++;
        } else {
            build_act_local(p, smem, red, w_pre);
        }
        if (consumer_sync_or(abort_flag)) {
            abort_flag = 1;
            timed_out = true;
            break;
        }
        const Act a = act_view(p.act, smem);
        switch (c.epi[ph]) {
        case EPI_STORE:
            consume_units<EPI_STORE, WIDE>(p, a, r, s, lap, unit_no, glu_up, &best, &abort_flag, timed_out);
            break;
        case EPI_RESID:
            consume_units<EPI_RESID, WIDE>(p, a, r, s, lap, unit_no, glu_up, nullptr, &abort_flag, timed_out);
            break;
        case EPI_QKV: consume_units<EPI_QKV, WIDE>(p, a, r, s, lap, unit_no, glu_up, nullptr, &abort_flag, timed_out); break;
        default: consume_units<EPI_GLU, WIDE>(p, a, r, s, lap, unit_no, glu_up, nullptr, &abort_flag, timed_out); break;
        }
        // every warp's writes of this phase, then one arrival for the CTA
        if (ph == c.nph - 1 && c.out_tok && lane == 0) {
            red[warp] = best.v;
            redi[warp] = best.i;
        }
        if (consumer_sync_or(abort_flag)) {
            abort_flag = 1;
            timed_out = true;
            break;
        }
        if (tid == 0) {
            if (ph == c.nph - 1 && c.out_tok) {
                ArgBest b{-INFINITY, -1};
                for (int w = 0; w < kConsumerWarps; w++)
                    if (redi[w] >= 0) argbest_take(b, red[w], redi[w]);
                c.best_val[blockIdx.x] = b.v;
                c.best_idx[blockIdx.x] = b.i;
            }
            __threadfence();
            const int old = atomicAdd(c.bar + ph, 1);
            if (ph == c.nph - 1 && old == (int)gridDim.x - 1) {
                // the last CTA of the last phase: nobody waits on the counters any more
                __threadfence();
                if (c.out_tok) {
                    ArgBest b{-INFINITY, -1};
                    for (int i = 0; i < (int)gridDim.x; i++) {
                        const int bi = __ldcg(c.best_idx + i);
                        if (bi >= 0) argbest_take(b, __ldcg(c.best_val + i), bi);
                    }
                    const uint32_t t = b.i < 0 ? 0u : (uint32_t)b.i;
                    *c.out_tok = t;
                    if (c.next_tok) *c.next_tok = t;
                    if (c.pos) {
                        if (c.history) c.history[*c.pos] = t;  // token generated after position *pos
                        *c.pos += 1;
                    }
                }
                for (int q = 0; q < c.nph; q++) c.bar[q] = 0;
            }
        }
    }
    (void)timed_out;
}

}  // namespace

void gemv_prepare(GemvParams& p, int sm_count) {
    bool need_f32 = false, need_q8k = false, need_q80 = false;
    int sbb_max = 0;
    for (int s = 0; s < p.nseg; s++) {
        const int t = p.seg[s].m.type;
        if (t == TPTC_TYPE_F16) need_f32 = true;
        else if (type_q80_family(t)) need_q80 = true;
        else need_q8k = true;
        sbb_max = std::max(sbb_max, sb_bytes(t));
    }
    const int K = p.K;
    int off = 0;
    auto take = [&](int bytes) {
        int o = off;
        off += (bytes + 15) / 16 * 16;
        return o;
    };
    p.act.f32 = need_f32 ? take(K * 4) : -1;
    p.act.q8k = need_q8k ? take(K) : -1;
    p.act.q8k_d = need_q8k ? take(K / QK_K * 4) : -1;
    p.act.q8k_bs = need_q8k ? take(K / 16 * 2) : -1;
    p.act.q8k_ps = need_q8k ? take(K / 32 * 2) : -1;
    p.act.q80 = need_q80 ? take(K) : -1;
    p.act.q80_d = need_q80 ? take(K / QK8_0 * 4) : -1;
    p.act.bytes = (off + 127) / 128 * 128;
    p.act.cbs = p.seg[0].m.cbs;

    p.cbs = p.seg[0].m.cbs;
    p.nchunks = (K / QK_K + p.cbs - 1) / p.cbs;
    p.stage_bytes = kTileRows * p.cbs * sbb_max;
    int ub = 0;
    for (int s = 0; s < p.nseg; s++) {
        p.seg[s].unit_begin = ub;
        ub += p.seg[s].m.Npad / kTileRows;
    }
    p.units = ub;
    const int ring = kRingBudget - p.act.bytes;
    const int S = std::max(2, std::min(kGemvMaxStages, ring / p.stage_bytes));
    // two persistent CTAs per SM: 16 consumer warps and two producers hide shared-memory
    // and copy latency better than one
    p.grid = std::min(p.units, 2 * sm_count);
    const int needed = ((p.units + p.grid - 1) / p.grid) * p.nchunks;
    p.stages = std::max(1, std::min(S, needed));
}

size_t gemv_smem(const GemvParams& p) { return (size_t)p.act.bytes + (size_t)p.stages * p.stage_bytes; }

// True when a matrix of the launch has a format only the WIDE kernel build carries.
static bool needs_wide(const GemvParams& p) {
    for (int i = 0; i < p.nseg; i++) {
        const int t = p.seg[i].m.type;
        if (t != TPTC_TYPE_Q4_K && t != TPTC_TYPE_Q6_K && t != TPTC_TYPE_Q8_0 && t != TPTC_TYPE_F16) return true;
    }
    return false;
}

static bool chain_wide(const ChainParams& c) {
    for (int i = 0; i < c.nph; i++)
        if (needs_wide(c.ph[i])) return true;
    return false;
}

template <int EPI>
static cudaError_t launch_epi(const GemvParams& p, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = gemv_smem(p);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return needs_wide(p) ? cudaLaunchKernelEx(&cfg, gemv_kernel<EPI, true>, p)
                         : cudaLaunchKernelEx(&cfg, gemv_kernel<EPI, false>, p);
}

cudaError_t gemv_launch(const GemvParams& p, int epi, cudaStream_t st, bool pdl) {
    if (p.stages < 1 || p.stages > kGemvMaxStages || p.grid < 1 || !p.act_global) return cudaErrorInvalidValue;
    if (!p.act_prepared) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((p.K / QK_K + kActWarps - 1) / kActWarps);
        cfg.blockDim = dim3(kActWarps * 32);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        cudaError_t e = p.tp_gather ? cudaLaunchKernelEx(&cfg, act_quant_kernel<true>, p, epi == EPI_DOTS ? 0 : 1)
                                    : cudaLaunchKernelEx(&cfg, act_quant_kernel<false>, p, epi == EPI_DOTS ? 0 : 1);
        if (e != cudaSuccess) return e;
    }
    switch (epi) {
    case EPI_STORE: return launch_epi<EPI_STORE>(p, st, pdl);
    case EPI_RESID: return launch_epi<EPI_RESID>(p, st, pdl);
    case EPI_QKV: return launch_epi<EPI_QKV>(p, st, pdl);
    case EPI_GLU: return launch_epi<EPI_GLU>(p, st, pdl);
    case EPI_DOTS: return launch_epi<EPI_DOTS>(p, st, pdl);
    }
    return cudaErrorInvalidValue;
}

void chain_prepare(ChainParams& c, int sm_count) {
    int act = 0, stage = 0;
    for (int i = 0; i < c.nph; i++) {
        act = std::max(act, c.ph[i].act.bytes);
        stage = std::max(stage, c.ph[i].stage_bytes);
    }
    c.act_bytes = (act + 127) / 128 * 128;
    c.stage_bytes = stage;
    c.stages = std::max(2, std::min(kGemvMaxStages, (kRingBudget - c.act_bytes) / stage));
    c.grid = 2 * sm_count;
    for (int i = 0; i < c.nph; i++) {
        // one ring geometry and one grid for every phase (the unit pairing depends on both)
        c.ph[i].stages = c.stages;
        c.ph[i].stage_bytes = c.stage_bytes;
        c.ph[i].grid = c.grid;
    }
}

size_t chain_smem(const ChainParams& c) { return (size_t)c.act_bytes + (size_t)c.stages * c.stage_bytes; }

bool chain_fits(const ChainParams& c, int sm_count) {
    int n = 0;
    const void* fn = chain_wide(c) ? (const void*)gemv_chain_kernel<true> : (const void*)gemv_chain_kernel<false>;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, chain_smem(c)) != cudaSuccess)
        return false;
    return n * sm_count >= c.grid;
}

cudaError_t chain_launch(const ChainParams& c, cudaStream_t st, bool pdl) {
    if (c.nph < 1 || c.nph > kChainMaxPhases || c.stages < 2 || !c.bar) return cudaErrorInvalidValue;
    for (int i = 0; i < c.nph; i++)
        if (c.epi[i] == EPI_DOTS || (c.ph[i].act_prepared && !c.ph[i].act_global)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = chain_smem(c);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return chain_wide(c) ? cudaLaunchKernelEx(&cfg, gemv_chain_kernel<true>, c)
                         : cudaLaunchKernelEx(&cfg, gemv_chain_kernel<false>, c);
}

template <bool WIDE>
static cudaError_t set_smem_attrs(int max_smem) {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemv_chain_kernel<WIDE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<EPI_STORE, WIDE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<EPI_RESID, WIDE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<EPI_QKV, WIDE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    if ((e = cudaFuncSetAttribute(gemv_kernel<EPI_GLU, WIDE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem))) return e;
    return cudaFuncSetAttribute(gemv_kernel<EPI_DOTS, WIDE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
}

cudaError_t gemv_init_device() {
    const int max_smem = 200 * 1024;
    cudaError_t e = set_smem_attrs<false>(max_smem);
    return e != cudaSuccess ? e : set_smem_attrs<true>(max_smem);
}

}  // namespace tptc
