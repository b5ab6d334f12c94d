// attn_prefill.cu -- causal GQA attention for a prompt chunk (prefill) on the tensor cores.
//
// Replaces the reference's per-token attention passes during its prefill loop
// (attention.wgsl:31-170 once per prompt token, wgpu_engine.rs:254-261) with one kernel over
// the chunk: query rows t (absolute position start + t) attend to keys 0 .. start + t of the
// KV cache (the chunk's own keys already written there), score = q.k / sqrt(hd), softmax,
// P.V; head h reads kv head h / (n_heads / n_kv).
//
// A CTA of 4 warps owns 64 query rows of one head (16 per warp) and streams the key/value
// positions in 64-row tiles through a double-buffered shared-memory ring (cp.async): scores
// S = Q K^T and the update O += P V run on mma.sync m16n8k16 (fp16 inputs, f32 accumulate),
// with an online softmax in base 2 in registers (flash-attention, one pass).  Q and the
// probabilities enter the tensor cores as fp16; the KV cache is fp16.
#include "prefill.h"
#include "tcgen05.cuh"

namespace tptc {

namespace {

constexpr int BQ = 64, BKV = 64, kThreads = 128;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int HD>
__global__ void __launch_bounds__(kThreads) attn_prefill_kernel(const __grid_constant__ AttnPrefillParams p) {
    constexpr int LD = HD + 8;  // padded row (halves): conflict-free ldmatrix
    constexpr int KS = HD / 16, NB = HD / 8;
    extern __shared__ __align__(16) uint8_t smem[];
    __half* sq = reinterpret_cast<__half*>(smem);  // [BQ][LD]
    __half* skv = sq + BQ * LD;                    // [2][K|V][BKV][LD]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int h = blockIdx.y, q0 = blockIdx.x * BQ, G = p.n_heads / p.n_kv, kvh = h / G;
    const int rows = min(BQ, p.T - q0);
    const __half* kc = p.kcache + (size_t)kvh * p.max_seq * HD;
    const __half* vc = p.vcache + (size_t)kvh * p.max_seq * HD;
    const int last = p.start + q0 + rows - 1;   // last key any row of the block attends to
    const int ntiles = last / BKV + 1;

    pdl_wait();
    pdl_launch_dependents();

    // Q tile (rows past the chunk are zero) and the first K/V tile
    constexpr int CH = HD / 8;  // 16-byte chunks per row
    for (int i = tid; i < BQ * CH; i += kThreads) {
        const int r = i / CH, c = i % CH;
        __half* dst = sq + r * LD + c * 8;
        if (r < rows) cp_async16(dst, p.q + ((size_t)(q0 + r) * p.n_heads + h) * HD + c * 8);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    auto load_kv = [&](int tile, int buf) {
        __half* dk = skv + buf * 2 * BKV * LD;
        __half* dv = dk + BKV * LD;
        const int p0 = tile * BKV;
        for (int i = tid; i < BKV * CH; i += kThreads) {
            const int r = i / CH, c = i % CH;
            if (p0 + r <= last) {
                cp_async16(dk + r * LD + c * 8, kc + (size_t)(p0 + r) * HD + c * 8);
                cp_async16(dv + r * LD + c * 8, vc + (size_t)(p0 + r) * HD + c * 8);
            } else {
                *reinterpret_cast<uint4*>(dk + r * LD + c * 8) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(dv + r * LD + c * 8) = make_uint4(0, 0, 0, 0);
            }
        }
    };
    load_kv(0, 0);
    cp_async_commit();

    const int g = lane >> 2, t4 = lane & 3;
    const float sl2 = p.scale * 1.4426950408889634f;
    // this thread's two rows: warp * 16 + g and + 8 (absolute positions)
    const int pos_a = p.start + q0 + warp * 16 + g, pos_b = pos_a + 8;
    float o[NB][4];
#pragma unroll
    for (int j = 0; j < NB; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    uint32_t qf[KS][4];

    for (int tile = 0; tile < ntiles; tile++) {
        const int buf = tile & 1;
        if (tile + 1 < ntiles) load_kv(tile + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (tile == 0) {
#pragma unroll
            for (int k = 0; k < KS; k++)
                ldsm_x4(qf[k], sq + (warp * 16 + (lane & 15)) * LD + k * 16 + (lane >> 4) * 8);
        }
        const __half* tk = skv + buf * 2 * BKV * LD;
        const __half* tv = tk + BKV * LD;
        // S = Q K^T for this warp's 16 rows x 64 positions
        float s[BKV / 8][4];
#pragma unroll
        for (int j = 0; j < BKV / 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int j = 0; j < BKV / 8; j += 2) {
#pragma unroll
            for (int k = 0; k < KS; k++) {
                uint32_t b[4];
                ldsm_x4(b, tk + (j * 8 + (lane & 7) + 8 * (lane >> 4)) * LD + k * 16 + 8 * ((lane >> 3) & 1));
                mma16816(s[j], qf[k], b[0], b[1]);
                mma16816(s[j + 1], qf[k], b[2], b[3]);
            }
        }
        // causal mask (only the last tiles reach past a row's position) and the online softmax
        const int p0 = tile * BKV;
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int j = 0; j < BKV / 8; j++) {
            const int c0 = p0 + j * 8 + 2 * t4;
            s[j][0] = c0 <= pos_a ? s[j][0] * sl2 : -INFINITY;
            s[j][1] = c0 + 1 <= pos_a ? s[j][1] * sl2 : -INFINITY;
            s[j][2] = c0 <= pos_b ? s[j][2] * sl2 : -INFINITY;
            s[j][3] = c0 + 1 <= pos_b ? s[j][3] * sl2 : -INFINITY;
            mx_a = fmaxf(mx_a, fmaxf(s[j][0], s[j][1]));
            mx_b = fmaxf(mx_b, fmaxf(s[j][2], s[j][3]));
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        const float mu_a = mn_a == -INFINITY ? 0.f : mn_a, mu_b = mn_b == -INFINITY ? 0.f : mn_b;
        const float al_a = fast_exp2(m_a - mu_a), al_b = fast_exp2(m_b - mu_b);
        m_a = mn_a;
        m_b = mn_b;
        float ls_a = 0.f, ls_b = 0.f;
#pragma unroll
        for (int j = 0; j < BKV / 8; j++) {
            s[j][0] = fast_exp2(s[j][0] - mu_a);
            s[j][1] = fast_exp2(s[j][1] - mu_a);
            s[j][2] = fast_exp2(s[j][2] - mu_b);
            s[j][3] = fast_exp2(s[j][3] - mu_b);
            ls_a += s[j][0] + s[j][1];
            ls_b += s[j][2] + s[j][3];
        }
        l_a = l_a * al_a + ls_a;  // quad partials: reduced across the 4 lanes at the end
        l_b = l_b * al_b + ls_b;
#pragma unroll
        for (int j = 0; j < NB; j++) {
            o[j][0] *= al_a;
            o[j][1] *= al_a;
            o[j][2] *= al_b;
            o[j][3] *= al_b;
        }
        // O += P V: P (fp16) from the score fragments, V through ldmatrix.trans
#pragma unroll
        for (int kk = 0; kk < BKV / 16; kk++) {
            uint32_t a[4];
            a[0] = pack_half2(s[2 * kk][0], s[2 * kk][1]);
            a[1] = pack_half2(s[2 * kk][2], s[2 * kk][3]);
            a[2] = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            a[3] = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int j = 0; j < NB; j += 2) {
                uint32_t b[4];
                ldsm_x4_t(b, tv + (kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * LD + j * 8 + 8 * (lane >> 4));
                mma16816(o[j], a, b[0], b[1]);
                mma16816(o[j + 1], a, b[2], b[3]);
            }
        }
        __syncthreads();  // the buffer is refilled by the next iteration's loads
    }
    cp_async_wait<0>();

    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    const float ia = 1.f / l_a, ib = 1.f / l_b;
    const int ra = warp * 16 + g, rb = ra + 8;
#pragma unroll
    for (int j = 0; j < NB; j++) {
        const int col = j * 8 + 2 * t4;
        if (ra < rows)
            *reinterpret_cast<uint32_t*>(p.out + ((size_t)(q0 + ra) * p.n_heads + h) * HD + col) =
                pack_half2(o[j][0] * ia, o[j][1] * ia);
        if (rb < rows)
            *reinterpret_cast<uint32_t*>(p.out + ((size_t)(q0 + rb) * p.n_heads + h) * HD + col) =
                pack_half2(o[j][2] * ib, o[j][3] * ib);
    }
}

// ---------------------------------------------------------------- tcgen05 kernel

namespace tc {

constexpr int BM = 128;         // query rows per tile (TMEM lanes); a CTA runs two tiles
constexpr int BN = 64;          // key positions per K/V tile
constexpr int kStages = 3;      // K/V ring
constexpr int kThreads = 320;   // producer, MMA, two softmax warpgroups
constexpr int kTmemCols = 512;  // S_A 0..63, S_B 64..127, O_A 128.., O_B 256..

template <int HD>
struct Lay {
    static constexpr int kQBytes = BM * HD * 2;   // one query tile: HD / 64 blocks [128 x 128 B]
    static constexpr int kKVBytes = BN * HD * 2;  // one K or V tile: HD / 64 blocks [64 x 128 B]
    static constexpr int kPBytes = BM * BN * 2;   // one P tile [128 x 128 B]
    static constexpr int kQ = 0;
    static constexpr int kK = kQ + 2 * kQBytes;
    static constexpr int kV = kK + kStages * kKVBytes;
    static constexpr int kP = kV + kStages * kKVBytes;
    static constexpr int kBytes = kP + 2 * kPBytes;
};

}  // namespace tc

__device__ __forceinline__ bool attn_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    if (err) atomicExch(err, TPTC_ERR_TIMEOUT);
    *abort_flag = 1;
    return false;
}

// Two query tiles (A: rows q0 .. q0 + 127, B: the next 128) share every K/V tile: while one
// tile's warpgroup runs its softmax the tensor core works on the other tile's products.
// Issue order per key tile j: P V_A(j), S_A(j + 1), P V_B(j), S_B(j + 1); every commit
// also covers the MMAs issued before it, so when a tile's S(j) lands its P V(j - 1) -- and so
// its O and its P buffer -- is complete.
// HD is the head dimension, HP the width of the shared-memory and TMEM layout (a multiple of
// 64).  For HD = 96 the kernel runs the 128-wide layout: the second 64-column TMA box of a
// K or V row reaches past the tensor's 96 columns and the copy fills those columns with
// zeros; the Q box of a head then also covers the next head's first 32 values, which meet
// those zero keys (S is unchanged), P V leaves the padded output columns at zero, and only
// the HD real columns are written.
template <int HD, int HP>
__global__ void __launch_bounds__(tc::kThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                           const __grid_constant__ CUtensorMap tv, const __grid_constant__ AttnPrefillParams p) {
    static_assert(HP % 64 == 0 && HD <= HP && HD % 32 == 0, "layout width");
    using L = tc::Lay<HP>;
    using tc::BM;
    using tc::BN;
    constexpr int NC = HP / 64;  // 64-column blocks of a (padded) row
    constexpr int S = tc::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t q_full, kv_full[S], kv_empty[S], s_full[2], p_full[2], o_done[2], drain;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = gridDim.x - 1 - blockIdx.x;  // the longest (latest) query pairs first
    const int h = blockIdx.y, kvh = h / (p.n_heads / p.n_kv);
    const int q0 = qt * 2 * BM;
    int rows[2], nt[2];
    for (int t = 0; t < 2; t++) {
        rows[t] = max(0, min(BM, p.T - q0 - t * BM));
        nt[t] = rows[t] > 0 ? (p.start + q0 + t * BM + rows[t] - 1) / BN + 1 : 0;
    }
    const int ntot = max(nt[0], nt[1]);
    const int last = p.start + q0 + (rows[1] > 0 ? BM + rows[1] : rows[0]) - 1;  // last key the CTA needs
    const int kvrow0 = kvh * p.max_seq;

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int s = 0; s < S; s++) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int t = 0; t < 2; t++) {
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], 4);  // one arrival per softmax warp of the tile
            mbar_init(&o_done[t], 1);
        }
        mbar_init(&drain, 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    if (warp == 1) tmem_alloc(&tmem_slot, tc::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            mbar_expect_tx(&q_full, (rows[1] > 0 ? 2 : 1) * L::kQBytes);
            for (int t = 0; t < 2; t++) {
                if (rows[t] == 0) continue;
#pragma unroll
                for (int c = 0; c < NC; c++)
                    tma_load_2d(smem + L::kQ + t * L::kQBytes + c * BM * 128, &tq, h * HD + c * 64, q0 + t * BM,
                                &q_full);
            }
            int j = 0;
            for (; j < ntot; j++) {
                const int s = j % S;
                if (j >= S && !attn_wait(&kv_empty[s], ((j / S) - 1) & 1, p.err, &abort_flag)) break;
                mbar_expect_tx(&kv_full[s], 2 * L::kKVBytes);
#pragma unroll
                for (int c = 0; c < NC; c++) {
                    tma_load_2d(smem + L::kK + s * L::kKVBytes + c * BN * 128, &tk, c * 64, kvrow0 + j * BN, &kv_full[s]);
                    tma_load_2d(smem + L::kV + s * L::kKVBytes + c * BN * 128, &tv, c * 64, kvrow0 + j * BN, &kv_full[s]);
                }
            }
            // the copies still in flight land before the CTA exits
            mbar_wait_bounded(&q_full, 0, nullptr);
            for (int jj = j > S ? j - S : 0; jj < j; jj++) mbar_wait_bounded(&kv_full[jj % S], (jj / S) & 1, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            const uint32_t id_s = mma_idesc(BM, BN), id_o = mma_idesc(BM, HP) | kIdescBMajorMN;
            auto issue_s = [&](int t, int j) {
                const uint32_t qa = smem_u32(smem + L::kQ + t * L::kQBytes);
                const uint32_t ka = smem_u32(smem + L::kK + (j % S) * L::kKVBytes);
#pragma unroll
                for (int c = 0; c < NC; c++)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_f16(tmem + 64 * t, sw128_desc(qa + c * BM * 128 + 32 * kk),
                                sw128_desc(ka + c * BN * 128 + 32 * kk), id_s, (c | kk) != 0);
                mma_commit(&s_full[t]);
            };
            auto issue_pv = [&](int t, int j) {
                const uint32_t pa = smem_u32(smem + L::kP + t * L::kPBytes);
                const uint32_t va = smem_u32(smem + L::kV + (j % S) * L::kKVBytes);
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++)
                    mma_f16(tmem + 128 * (t + 1), sw128_desc(pa + 32 * kk), sw128_desc_mn(va + kk * 2048, BN * 128),
                            id_o, (j | kk) != 0);
            };
            bool ok = attn_wait(&q_full, 0, p.err, &abort_flag) && attn_wait(&kv_full[0], 0, p.err, &abort_flag);
            if (ok) {
                tc_fence_after();
                for (int t = 0; t < 2; t++)
                    if (nt[t] > 0) issue_s(t, 0);
            }
            for (int j = 0; j < ntot && ok; j++) {
                bool next_ready = false;  // K/V tile j + 1 landed (waited for before its first S)
                for (int t = 0; t < 2 && ok; t++) {
                    if (j >= nt[t]) continue;
                    if (!attn_wait(&p_full[t], j & 1, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv(t, j);
                    if (j + 1 < nt[t]) {
                        if (!next_ready) {
                            if (!attn_wait(&kv_full[(j + 1) % S], ((j + 1) / S) & 1, p.err, &abort_flag)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            next_ready = true;
                        }
                        issue_s(t, j + 1);
                    } else {
                        mma_commit(&o_done[t]);
                    }
                }
                if (ok) mma_commit(&kv_empty[j % S]);  // K_j and V_j consumed by both tiles
            }
            // every MMA issued has completed before TMEM is freed
            mma_commit(&drain);
            mbar_wait_bounded(&drain, 0, nullptr);
        }
    } else {  // warps 2..5: tile A, warps 6..9: tile B; one thread per query row
        const int t = (warp - 2) >> 2, qq = warp & 3, r = 32 * qq + lane;
        const uint32_t loff = (uint32_t)(32 * qq) << 16;
        const uint32_t tS = tmem + 64 * t, tO = tmem + 128 * (t + 1);
        const int pos = p.start + q0 + t * BM + r;
        const float sl2 = p.scale * 1.4426950408889634f;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        uint8_t* prow = smem + L::kP + t * L::kPBytes + (r >> 3) * 1024 + (r & 7) * 128;
        for (int j = 0; j < nt[t]; j++) {
            if (!attn_wait(&s_full[t], j & 1, p.err, &abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sv[BN];
            tmem_ld32(tS + loff, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
            tmem_ld32(tS + loff + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
            const int p0 = j * BN;
            float mt = -INFINITY;
#pragma unroll
            for (int k = 0; k < BN; k++) {
                const float x = p0 + k <= pos ? __uint_as_float(sv[k]) * sl2 : -INFINITY;
                sv[k] = __float_as_uint(x);
                mt = fmaxf(mt, x);
            }
            // the reference max moves only past 2^8 above the current one (P stays <= 256)
            const bool move = mt > m_ref + 8.f;
            float alpha = 1.f;
            if (move) {
                alpha = fast_exp2(m_ref - mt);
                l *= alpha;
                m_ref = mt;
            }
            if (j > 0 && __any_sync(0xffffffffu, move)) {
#pragma unroll 1
                for (int c0 = 0; c0 < HD; c0 += 32) {
                    uint32_t o[32];
                    tmem_ld32(tO + loff + c0, o);
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(tO + loff + c0, o);
                }
            }
            // P = 2^(s - m_ref) as fp16, K-major with 128-byte swizzle: row r's 16-byte chunk
            // c (keys 8c .. 8c + 7) sits at chunk c ^ (r % 8) of the row
            float ps = 0.f;
#pragma unroll
            for (int c = 0; c < BN / 8; c++) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float a = fast_exp2(__uint_as_float(sv[8 * c + 2 * e]) - m_ref);
                    const float b = fast_exp2(__uint_as_float(sv[8 * c + 2 * e + 1]) - m_ref);
                    ps += a + b;
                    w[e] = pack_half2(a, b);
                }
                *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            l += ps;
            if (j == ntot - 1) {
                // cache rows past the CTA's last attended position may hold anything: zero them
                // in the V tile so that 0 * value cannot become NaN (both warpgroups write the
                // same zeros, each before its own P V)
                uint8_t* vb = smem + L::kV + (j % S) * L::kKVBytes;
                const int vr0 = last - p0 + 1, nclr = (BN - vr0) * NC * 8;
                for (int idx = r; idx < nclr; idx += BM) {
                    const int i = vr0 + idx / (NC * 8), rem = idx % (NC * 8), c = rem >> 3, ch = rem & 7;
                    *reinterpret_cast<uint4*>(vb + c * BN * 128 + (i >> 3) * 1024 + (i & 7) * 128 + ch * 16) =
                        make_uint4(0, 0, 0, 0);
                }
            }
            fence_proxy_async_smem();  // P (and the cleared V rows) before the tensor core reads them
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);
        }
        if (ok && nt[t] > 0 && attn_wait(&o_done[t], 0, p.err, &abort_flag)) {
            tc_fence_after();
            const float il = 1.f / l;
            __half* orow = p.out + ((size_t)(q0 + t * BM + r) * p.n_heads + h) * HD;
#pragma unroll 1
            for (int c0 = 0; c0 < HD; c0 += 32) {
                uint32_t o[32];
                tmem_ld32(tO + loff + c0, o);
                if (r < rows[t]) {
                    uint32_t w[16];
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        w[i] = pack_half2(__uint_as_float(o[2 * i]) * il, __uint_as_float(o[2 * i + 1]) * il);
                    uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
                    for (int i = 0; i < 4; i++) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, tc::kTmemCols);
    }
}

template <int HD>
size_t attn_prefill_smem() {
    return (size_t)(BQ + 4 * BKV) * (HD + 8) * sizeof(__half);
}

}  // namespace

cudaError_t attn_prefill_init_device() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(attn_prefill_tc_kernel<64, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  tc::Lay<64>::kBytes + 1024)))
        return e;
    if ((e = cudaFuncSetAttribute(attn_prefill_tc_kernel<96, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  tc::Lay<128>::kBytes + 1024)))
        return e;
    if ((e = cudaFuncSetAttribute(attn_prefill_tc_kernel<128, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  tc::Lay<128>::kBytes + 1024)))
        return e;
    if ((e = cudaFuncSetAttribute(attn_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)attn_prefill_smem<64>())))
        return e;
    if ((e = cudaFuncSetAttribute(attn_prefill_kernel<96>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)attn_prefill_smem<96>())))
        return e;
    return cudaFuncSetAttribute(attn_prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)attn_prefill_smem<128>());
}

namespace {

template <int HD, int HP>
cudaError_t launch_tc(const AttnPrefillParams& p, cudaStream_t st, bool pdl) {
    CUtensorMap tq, tk, tv;
    cudaError_t e = make_tmap_f16(&tq, p.q, p.T, (int64_t)p.n_heads * HD, (int64_t)p.n_heads * HD, tc::BM);
    if (e == cudaSuccess) e = make_tmap_f16(&tk, p.kcache, (int64_t)p.n_kv * p.max_seq, HD, HD, tc::BN);
    if (e == cudaSuccess) e = make_tmap_f16(&tv, p.vcache, (int64_t)p.n_kv * p.max_seq, HD, HD, tc::BN);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.T + 2 * tc::BM - 1) / (2 * tc::BM), p.n_heads);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = tc::Lay<HP>::kBytes + 1024;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_prefill_tc_kernel<HD, HP>, tq, tk, tv, p);
}

}  // namespace

cudaError_t launch_attn_prefill(const AttnPrefillParams& p, cudaStream_t st, bool pdl, int use_tc) {
    if (p.T <= 0 || p.n_kv <= 0 || p.n_heads % p.n_kv || p.start < 0 || p.start + p.T > p.max_seq)
        return cudaErrorInvalidValue;
    const uintptr_t align = reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.kcache) |
                            reinterpret_cast<uintptr_t>(p.vcache);
    if (use_tc && (align & 15) == 0) {
        if (p.hd == 64) return launch_tc<64, 64>(p, st, pdl);
        if (p.hd == 96) return launch_tc<96, 128>(p, st, pdl);
        if (p.hd == 128) return launch_tc<128, 128>(p, st, pdl);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.T + BQ - 1) / BQ, p.n_heads);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (p.hd) {
    case 64: cfg.dynamicSmemBytes = attn_prefill_smem<64>(); return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<64>, p);
    case 96: cfg.dynamicSmemBytes = attn_prefill_smem<96>(); return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<96>, p);
    case 128:
        cfg.dynamicSmemBytes = attn_prefill_smem<128>();
        return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<128>, p);
    }
    return cudaErrorInvalidValue;
}

}  // namespace tptc
