// gemm_q.cu -- prefill GEMM with the weight dequantisation fused in: C[M x N] = A[M x K] . W^T
// with A the prompt's fp16 activations and W a Q4_K / Q6_K / Q8_0 matrix in the engine's
// tiled device layout (gemv.cuh), f32 accumulation in tensor memory.
//
// Replaces, for quantised weights, the two-pass "expand the layer's matrix to fp16, then
// gemm_tc" of the batched prefill (and the reference's per-token dequant_*.wgsl + gemm.wgsl
// passes, wgpu_engine.rs:581-605): the quantised tiles go from HBM to shared memory by TMA
// and are expanded there, so a weight byte crosses HBM once in its quantised size.
//
// A persistent kernel (one CTA per SM) walks 128 x 256 tiles of C, M fastest:
//   - warp 0 (one lane): TMA producer of A, 128 x 64 fp16 tiles with 128-byte swizzle;
//   - warp 14 (one lane): TMA producer of W.  Per 256-column super-block, the quantised
//     blocks of the tile's 256 rows -- one 4-D tensor map over the device layout (bytes of a
//     block, row in its 8-row group, chunk, row group) brings 256 x block-bytes in one copy.
//     Its own ring runs ahead of the A ring, so the block loads do not wait on the tensor core;
//   - warps 6-13: dequantisation.  Thread t expands row t of the tile: per 64-column step it
//     reads the row's codes of the step with 16-byte loads, then writes its 64 fp16 values
//     into the 128-byte-swizzled K-major layout tcgen05.mma reads (2- or 3-stage ring), building
//     each value from its code with fp16 bit arithmetic (byte permute onto 1024 + code, exact
//     subtraction, one multiply or fused multiply-add with the fp16 scale and offset) -- no
//     fp32 round trip, no conversion unit;
//   - warp 1: allocates 512 TMEM columns (two 256-column accumulators) and issues
//     tcgen05.mma (M 128, N 256, K 16) from one lane, committing the A stage, the W stage and
//     each finished accumulator;
//   - warps 2-5: epilogue, as gemm_tc (store, residual add, or silu(gate) * up in fp16).
// Values: Q8_0 codes times their fp16 scale round exactly as the f32 expansion does; Q4_K and
// Q6_K scale products are rounded to fp16 before the code is applied, within one fp16 ulp of
// the f32 expansion.  Every mbarrier wait is bounded (error word, CTA abort, TMEM freed).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "gemm_epi.cuh"
#include "gemv.cuh"
#include "prefill.h"
#include "quant.cuh"
#include "tcgen05.cuh"

namespace tptc {

namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kABytes = BM * BK * 2;  // 16 KB
constexpr int kBBytes = BN * BK * 2;  // 32 KB
constexpr int kThreads = 480;
constexpr int kQWarp = 14;  // the W producer
constexpr int kAccCols = BN;
constexpr int kTmemCols = 2 * kAccCols;
constexpr int kDeqThreads = 256;  // one per row of the tile
constexpr int kDeqWarps = kDeqThreads / 32;

__host__ __device__ constexpr int q_sbm(int type) { return type == TPTC_TYPE_Q4_K ? 144 : type == TPTC_TYPE_Q6_K ? 208 : 256; }
// Ring depths within 227 KB.  Two quantised stages (8 steps of look-ahead for the W
// producer); the expanded-B ring decouples the expansion from the tensor core, three stages
// where they fit (Q4_K's 36 KB quantised stages), else two (Q6_K 52 KB, Q8_0 64 KB, which
// also leaves Q8_0 two A stages).
__host__ __device__ constexpr int q_astages(int type) { return type == TPTC_TYPE_Q8_0 ? 2 : 3; }
__host__ __device__ constexpr int q_qstages(int) { return 2; }
__host__ __device__ constexpr int q_bstages(int type) { return type == TPTC_TYPE_Q4_K ? 3 : 2; }
__host__ __device__ constexpr size_t q_smem(int type) {
    return (size_t)q_astages(type) * kABytes + (size_t)q_qstages(type) * BN * q_sbm(type) +
           (size_t)q_bstages(type) * kBBytes + 1024;
}
static_assert(q_smem(TPTC_TYPE_Q8_0) <= 227 * 1024 - 256 && q_smem(TPTC_TYPE_Q6_K) <= 227 * 1024 - 256 &&
                  q_smem(TPTC_TYPE_Q4_K) <= 227 * 1024 - 256,
              "shared memory");
static_assert(q_smem(TPTC_TYPE_Q4_K) > 116 * 1024, "one CTA per SM (the 512 TMEM columns)");

struct GemmQParams {
    GemmTcParams g;   // M, N, K, outputs, err
    DevMatrix w;      // the weight (N = its physical rows, 8-row groups)
    int nsb, cbs, nchunks, cb_last;
};

__device__ __forceinline__ bool q_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 15 && *abort_flag) return false;
    }
    if (err) atomicExch(err, TPTC_ERR_TIMEOUT);
    *abort_flag = 1;
    return false;
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ __half2 u2h2(uint32_t v) { return *reinterpret_cast<const __half2*>(&v); }
__device__ __forceinline__ uint32_t h22u(__half2 v) { return *reinterpret_cast<const uint32_t*>(&v); }

// Four unsigned byte codes (v's bytes) as two half2 of (code - bias): each code lands in the
// low byte of an fp16 whose high byte is 0x64 (= 1024 + code, exact), then bias + 1024 is
// subtracted exactly.
__device__ __forceinline__ void codes4(uint32_t v, __half2 bias, __half2& lo, __half2& hi) {
    lo = __hsub2(u2h2(prmt(v, 0x64646464u, 0x4140u)), bias);
    hi = __hsub2(u2h2(prmt(v, 0x64646464u, 0x4342u)), bias);
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// Scale and min of Q4_K sub-block j from the 12 packed scale bytes as words w0..w2
// (get_scale_min_k4, k_quants.rs).
__device__ __forceinline__ void q4k_sm(uint32_t w0, uint32_t w1, uint32_t w2, int j, int& sc, int& mn) {
    if (j < 4) {
        sc = (w0 >> (8 * j)) & 63;
        mn = (w1 >> (8 * j)) & 63;
    } else {
        const int sh = 8 * (j - 4);
        sc = ((w2 >> sh) & 0xf) | (((w0 >> sh) >> 6 & 3) << 4);
        mn = ((w2 >> sh) >> 4 & 0xf) | (((w1 >> sh) >> 6 & 3) << 4);
    }
}

// Chunk c (8 fp16 values) of the step into the row's 128-byte swizzled line.
__device__ __forceinline__ void put_chunk(uint8_t* rowp, int r7, int c, uint32_t o0, uint32_t o1, uint32_t o2,
                                          uint32_t o3) {
    *reinterpret_cast<uint4*>(rowp + ((c ^ r7) << 4)) = make_uint4(o0, o1, o2, o3);
}

// Codes 8c .. 8c + 7 (bytes of v0, v1, biased) times s plus m.
__device__ __forceinline__ void fma_chunk(uint8_t* rowp, int r7, int c, uint32_t v0, uint32_t v1, __half2 bias,
                                          __half2 s, __half2 m) {
    __half2 a, b, e, f;
    codes4(v0, bias, a, b);
    codes4(v1, bias, e, f);
    put_chunk(rowp, r7, c, h22u(__hfma2(a, s, m)), h22u(__hfma2(b, s, m)), h22u(__hfma2(e, s, m)),
              h22u(__hfma2(f, s, m)));
}
__device__ __forceinline__ void mul_chunk(uint8_t* rowp, int r7, int c, uint32_t v0, uint32_t v1, __half2 bias,
                                          __half2 s) {
    __half2 a, b, e, f;
    codes4(v0, bias, a, b);
    codes4(v1, bias, e, f);
    put_chunk(rowp, r7, c, h22u(__hmul2(a, s)), h22u(__hmul2(b, s)), h22u(__hmul2(e, s)), h22u(__hmul2(f, s)));
}

// The 64 fp16 values of 64-column step kk of one row (its block at `blk` in shared memory)
// into its swizzled line `rowp`: all of the step's codes are loaded first (16-byte loads),
// then expanded and stored.  `hdr` = the Q4_K block's first 16 bytes (d, dmin, scales);
// `aux` = Q6_K's d (low half), Q8_0's two block scales of the step.
template <int QT>
__device__ __forceinline__ void dequant_step(const uint8_t* blk, int kk, uint4 hdr, uint32_t aux, uint8_t* rowp,
                                             int r7) {
    if (QT == TPTC_TYPE_Q4_K) {
        // step kk: sub-block 2kk = low nibbles of qs[32kk .. +32), 2kk + 1 = high nibbles
        const uint4 qa = lds128(blk + 16 + 32 * kk), qb = lds128(blk + 32 + 32 * kk);
        const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        int sc0, mn0, sc1, mn1;
        q4k_sm(hdr.y, hdr.z, hdr.w, 2 * kk, sc0, mn0);
        q4k_sm(hdr.y, hdr.z, hdr.w, 2 * kk + 1, sc1, mn1);
        const float d = h2f((uint16_t)(hdr.x & 0xffffu)), dmin = h2f((uint16_t)(hdr.x >> 16));
        const __half2 s0 = __float2half2_rn(__fmul_rn(d, (float)sc0)), m0 = __float2half2_rn(-__fmul_rn(dmin, (float)mn0));
        const __half2 s1 = __float2half2_rn(__fmul_rn(d, (float)sc1)), m1 = __float2half2_rn(-__fmul_rn(dmin, (float)mn1));
        const __half2 bias = __float2half2_rn(1024.f);
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const int sh = (c >> 2) * 4, w = 2 * (c & 3);
            fma_chunk(rowp, r7, c, (q[w] >> sh) & 0x0f0f0f0fu, (q[w + 1] >> sh) & 0x0f0f0f0fu, bias, c < 4 ? s0 : s1,
                      c < 4 ? m0 : m1);
        }
    } else if (QT == TPTC_TYPE_Q6_K) {
        // elements 64kk + 8c + i: half h = kk / 2, group i4 = 2 (kk % 2) + c / 4, l = 8 (c % 4) + i;
        // low nibbles ql[64h + 32 (i4 % 2) + l] (shift 4 for i4 >= 2), high bits qh[32h + l]
        // (shift 2 i4), scale sc[(64kk + 8c) / 16]
        const int h = kk >> 1, hi = kk & 1;
        const uint4 l0 = lds128(blk + 64 * h), l1 = lds128(blk + 64 * h + 16), l2 = lds128(blk + 64 * h + 32),
                    l3 = lds128(blk + 64 * h + 48);
        const uint4 h0 = lds128(blk + 128 + 32 * h), h1 = lds128(blk + 128 + 32 * h + 16);
        const uint32_t scw = *reinterpret_cast<const uint32_t*>(blk + 192 + 4 * kk);
        const uint32_t L[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w, l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
        const uint32_t H[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const float d = h2f((uint16_t)(aux & 0xffffu));
        const int lsh = hi ? 4 : 0;
        const __half2 bias = __float2half2_rn(1056.f);  // 1024 + the +32 the codes carry
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const int lw = 8 * (c >> 2) + 2 * (c & 3), hw = 2 * (c & 3), hsh = 4 * hi + 2 * (c >> 2);
            const uint32_t v0 = ((L[lw] >> lsh) & 0x0f0f0f0fu) | (((H[hw] >> hsh) & 0x03030303u) << 4);
            const uint32_t v1 = ((L[lw + 1] >> lsh) & 0x0f0f0f0fu) | (((H[hw + 1] >> hsh) & 0x03030303u) << 4);
            const int scv = (int)(int8_t)(scw >> (8 * (c >> 1)));
            mul_chunk(rowp, r7, c, v0, v1, bias, __float2half2_rn(__fmul_rn(d, (float)scv)));
        }
    } else {  // Q8_0: int8 codes, one fp16 scale per 32 elements
        // rows are 256 bytes apart: row r reads its four 16-byte pieces in the order j + r (mod 4),
        // so a quarter warp reads two rows per bank group and stores conflict-free
        uint4 D[4];
#pragma unroll
        for (int j = 0; j < 4; j++) D[j] = lds128(blk + 64 * kk + 16 * ((j + r7) & 3));
        const __half2 slo = u2h2((aux & 0xffffu) * 0x10001u), shi = u2h2((aux >> 16) * 0x10001u);
        const __half2 bias = __float2half2_rn(1152.f);  // signed code + 128 flipped to unsigned
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int cc = (j + r7) & 3;
            const __half2 sc = cc < 2 ? slo : shi;
            mul_chunk(rowp, r7, 2 * cc, D[j].x ^ 0x80808080u, D[j].y ^ 0x80808080u, bias, sc);
            mul_chunk(rowp, r7, 2 * cc + 1, D[j].z ^ 0x80808080u, D[j].w ^ 0x80808080u, bias, sc);
        }
    }
}

template <int EPI, int QT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_q_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw,
                  const __grid_constant__ CUtensorMap tw_last, const __grid_constant__ GemmQParams q) {
    constexpr int SBM = q_sbm(QT);
    constexpr int kQBytes = BN * SBM;
    constexpr int kAStages = q_astages(QT);
    constexpr int kQStages = q_qstages(QT);
    constexpr int kBStages = q_bstages(QT);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + kAStages * kABytes;
    uint8_t* sQ = sB + kBStages * kBBytes;
    __shared__ uint64_t a_full[3], a_empty[3], q_full[3], q_empty[3];
    __shared__ uint64_t b_full[3], b_empty[3], tfull[2], tempty[2], drain;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    const GemmTcParams& p = q.g;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (p.M + BM - 1) / BM, num_n = (p.N + BN - 1) / BN, tiles = num_m * num_n, nk = p.K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kAStages; s++) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < kQStages; s++) {
            mbar_init(&q_full[s], 1);
            mbar_init(&q_empty[s], kDeqWarps);  // one arrival per dequantisation warp
        }
        for (int s = 0; s < kBStages; s++) {
            mbar_init(&b_full[s], kDeqWarps);
            mbar_init(&b_empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);
        }
        mbar_init(&drain, 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    if (warp == 1) tmem_alloc(&tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer of A, one 128 x 64 tile per step
            uint32_t ai = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int m0 = (t % num_m) * BM;
                for (int kb = 0; kb < nk; kb++) {
                    const int s = ai % kAStages;
                    if (ai >= kAStages && !q_wait(&a_empty[s], ((ai / kAStages) - 1) & 1, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&a_full[s], kABytes);
                    tma_load_2d(sA + s * kABytes, &ta, kb * BK, m0, &a_full[s]);
                    ai++;
                }
            }
            // the copies still in flight land before the CTA exits (only after an abort can
            // one be unconsumed)
            if (abort_flag)
                for (uint32_t j = ai > (uint32_t)kAStages ? ai - kAStages : 0; j < ai; j++)
                    mbar_wait_backoff(&a_full[j % kAStages], (j / kAStages) & 1, nullptr);
        }
    } else if (warp == kQWarp) {
        if (lane == 0) {  // TMA producer of W, one super-block column of the tile's rows per copy
            uint32_t qi = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int n0 = (t / num_m) * BN;
                for (int sb = 0; sb < q.nsb; sb++) {
                    const int qs = qi % kQStages, c = sb / q.cbs, j = sb - c * q.cbs;
                    if (qi >= kQStages && !q_wait(&q_empty[qs], ((qi / kQStages) - 1) & 1, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&q_full[qs], kQBytes);
                    if (c == q.nchunks - 1 && q.cb_last != q.cbs)
                        tma_load_4d(sQ + qs * kQBytes, &tw_last, j * SBM, 0, 0, n0 / kTileRows, &q_full[qs]);
                    else
                        tma_load_4d(sQ + qs * kQBytes, &tw, j * SBM, 0, c, n0 / kTileRows, &q_full[qs]);
                    qi++;
                }
            }
            if (abort_flag)
                for (uint32_t j = qi > (uint32_t)kQStages ? qi - kQStages : 0; j < qi; j++)
                    mbar_wait_backoff(&q_full[j % kQStages], (j / kQStages) & 1, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            const uint32_t idesc = mma_idesc(BM, BN);
            uint32_t ai = 0, bi = 0, tc = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, tc++) {
                const uint32_t acc = tc & 1, d = tmem + acc * kAccCols;
                if (tc >= 2 && !q_wait(&tempty[acc], ((tc >> 1) - 1) & 1, p.err, &abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < nk; kb++, ai++, bi++) {
                    const int s = ai % kAStages, bs = bi % kBStages;
                    if (!q_wait(&a_full[s], (ai / kAStages) & 1, p.err, &abort_flag) ||
                        !q_wait(&b_full[bs], (bi / kBStages) & 1, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(sA + s * kABytes), b = smem_u32(sB + bs * kBBytes);
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        mma_f16(d, sw128_desc(a + 32 * k), sw128_desc(b + 32 * k), idesc, (kb | k) != 0);
                    mma_commit(&a_empty[s]);
                    mma_commit(&b_empty[bs]);
                }
                if (ok) mma_commit(&tfull[acc]);
            }
            mma_commit(&drain);
            mbar_wait_bounded(&drain, 0, p.err);
        }
    } else if (warp < 6) {  // epilogue warps 2..5
        const int qq = warp & 3;
        uint32_t tc = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, tc++) {
            const uint32_t acc = tc & 1;
            if (!q_wait(&tfull[acc], (tc >> 1) & 1, p.err, &abort_flag)) break;
            tc_fence_after();
            const int m0 = (t % num_m) * BM, n0 = (t / num_m) * BN;
            const int row = m0 + 32 * qq + lane;
            const uint32_t base = tmem + acc * kAccCols + ((uint32_t)(32 * qq) << 16);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(base + (uint32_t)c0, r);
                if (c0 + 32 == BN) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[acc]);
                }
                store_cols<EPI>(p, row, n0 + c0, r);
            }
        }
    } else {  // dequantisation warps 6..13: thread dt expands row dt of the tile
        const int dt = threadIdx.x - 6 * 32, r7 = dt & 7;
        uint32_t qi = 0, bi = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            const int n0 = (t / num_m) * BN;
            // scales kept outside the blocks (the tile's scale section, in HBM): Q6_K's d,
            // Q8_0's eight block scales of the super-block
            const int prow = min(n0 + dt, q.w.Npad - 1);
            uint4 sc8 = make_uint4(0, 0, 0, 0), hdr = make_uint4(0, 0, 0, 0);
            bool ok = true;
            for (int kb = 0; kb < nk; kb++, bi++) {
                const int kk = kb & 3, qs = qi % kQStages, bs = bi % kBStages;
                const uint8_t* blk = sQ + qs * kQBytes + dt * SBM;
                if (kk == 0) {
                    if (!q_wait(&q_full[qs], (qi / kQStages) & 1, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint16_t* sc = dm_scales(q.w, prow, kb >> 2);
                    if (QT == TPTC_TYPE_Q6_K) sc8.x = sc[0];
                    if (QT == TPTC_TYPE_Q8_0) sc8 = *reinterpret_cast<const uint4*>(sc);
                    if (QT == TPTC_TYPE_Q4_K) hdr = lds128(blk);
                }
                if (bi >= kBStages && !q_wait(&b_empty[bs], ((bi / kBStages) - 1) & 1, p.err, &abort_flag)) {
                    ok = false;
                    break;
                }
                const uint32_t aux = QT == TPTC_TYPE_Q8_0 ? (kk == 0 ? sc8.x : kk == 1 ? sc8.y : kk == 2 ? sc8.z : sc8.w)
                                                          : sc8.x;
                dequant_step<QT>(blk, kk, hdr, aux, sB + bs * kBBytes + (dt >> 3) * 1024 + r7 * 128, r7);
                fence_proxy_async_smem();  // generic writes before the tensor core reads them
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&b_full[bs]);
                    if (kk == 3) mbar_arrive(&q_empty[qs]);
                }
                if (kk == 3) qi++;
            }
            if (!ok) break;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 q_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

// The quantised blocks of one super-block column of 256 rows as a 4-D box over the device
// layout: (block bytes, row in its 8-row group, chunk, row group).  `chunk_base` / `cb`
// select the regular chunks or the shorter last one.
cudaError_t make_wmap(CUtensorMap* map, const DevMatrix& w, int64_t chunk_off, int cb, int nchunks) {
    auto enc = q_encode();
    if (!enc) return cudaErrorNotSupported;
    const int sbm = sb_main_bytes(w.type), sbb = sb_bytes(w.type);
    const cuuint64_t dims[4] = {(cuuint64_t)cb * sbm, 8, (cuuint64_t)nchunks, (cuuint64_t)(w.Npad / kTileRows)};
    const cuuint64_t strides[3] = {(cuuint64_t)cb * sbm, (cuuint64_t)kTileRows * w.cbs * sbb,
                                   (cuuint64_t)kTileRows * w.main_row_bytes};
    const cuuint32_t box[4] = {(cuuint32_t)sbm, 8, 1, (cuuint32_t)(BN / kTileRows)};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, w.main + chunk_off, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int EPI, int QT>
cudaError_t launch_q(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& twl, const GemmQParams& q,
                     unsigned grid, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = q_smem(QT);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_q_kernel<EPI, QT>, ta, tw, twl, q);
}

template <int QT>
cudaError_t set_attrs() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemm_q_kernel<GEMM_STORE, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)q_smem(QT))))
        return e;
    if ((e = cudaFuncSetAttribute(gemm_q_kernel<GEMM_RESID, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)q_smem(QT))))
        return e;
    return cudaFuncSetAttribute(gemm_q_kernel<GEMM_GLU, QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)q_smem(QT));
}

int q_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        n <= 0)
        return 148;
    return n;
}

}  // namespace

bool gemm_q_supported(const DevMatrix& w) {
    return (w.type == TPTC_TYPE_Q4_K || w.type == TPTC_TYPE_Q6_K || w.type == TPTC_TYPE_Q8_0) && w.Npad % kTileRows == 0 &&
           w.K % QK_K == 0;
}

bool gemm_q_preferred(const DevMatrix& w, int M, int N, int sms) {
    if (!gemm_q_supported(w) || M <= 0 || N <= 0 || sms <= 0) return false;
    // Both paths walk 128 x 256 tiles, one CTA per SM; per 64-column step a CTA of this kernel
    // takes about 0.9 us (the expansion in shared memory bounds it), one of gemm_tc about
    // 0.5 us, and the separate expansion of the matrix to fp16 about 0.7 ns per 1000
    // elements -- B200 measurements over Q4_K / Q6_K / Q8_0 and M = 128 .. 8192.
    const double nk = w.K / 64.0;
    const long tiles = (long)((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const double waves = (double)((tiles + sms - 1) / sms);
    const double fused_us = waves * nk * 0.9;
    const double two_pass_us = (double)N * w.K * 0.73e-6 + waves * nk * 0.5;
    return fused_us < two_pass_us;
}

cudaError_t gemm_q_init_device() {
    cudaError_t e;
    if ((e = set_attrs<TPTC_TYPE_Q4_K>())) return e;
    if ((e = set_attrs<TPTC_TYPE_Q6_K>())) return e;
    return set_attrs<TPTC_TYPE_Q8_0>();
}

cudaError_t gemm_q(int epi, const __half* a, int lda, const DevMatrix& w, const GemmTcParams& p, cudaStream_t st,
                   bool pdl) {
    if (!gemm_q_supported(w) || p.M <= 0 || p.N <= 0 || p.N > w.Npad || p.K != w.K || lda % 8 ||
        (reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(w.main) & 15) ||
        (epi == GEMM_GLU && p.N % 8))
        return cudaErrorInvalidValue;
    GemmQParams q = {};
    q.g = p;
    q.w = w;
    q.nsb = w.K / QK_K;
    q.cbs = w.cbs;
    q.nchunks = (q.nsb + w.cbs - 1) / w.cbs;
    q.cb_last = q.nsb - (q.nchunks - 1) * w.cbs;
    CUtensorMap ta, tw, twl;
    cudaError_t e = make_tmap_f16(&ta, a, p.M, p.K, lda, BM);
    // the regular map spans the whole chunks only; with none (fewer super-blocks than a
    // chunk) it is a copy of the last chunk's map and never used
    if (e == cudaSuccess)
        e = make_wmap(&twl, w, (int64_t)(q.nchunks - 1) * kTileRows * w.cbs * sb_bytes(w.type), q.cb_last, 1);
    if (e == cudaSuccess) {
        if (q.nsb >= w.cbs) e = make_wmap(&tw, w, 0, w.cbs, q.nsb / w.cbs);
        else tw = twl;
    }
    if (e != cudaSuccess) return e;
    const long tiles = (long)((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
    const unsigned grid = (unsigned)std::min<long>(tiles, q_sms());
    const int t = w.type;
#define GQ(E)                                                                                           \
    (t == TPTC_TYPE_Q4_K ? launch_q<E, TPTC_TYPE_Q4_K>(ta, tw, twl, q, grid, st, pdl)                   \
     : t == TPTC_TYPE_Q6_K ? launch_q<E, TPTC_TYPE_Q6_K>(ta, tw, twl, q, grid, st, pdl)                 \
                           : launch_q<E, TPTC_TYPE_Q8_0>(ta, tw, twl, q, grid, st, pdl))
    switch (epi) {
    case GEMM_STORE: return GQ(GEMM_STORE);
    case GEMM_RESID: return GQ(GEMM_RESID);
    case GEMM_GLU: return GQ(GEMM_GLU);
    }
#undef GQ
    return cudaErrorInvalidValue;
}

}  // namespace tptc
