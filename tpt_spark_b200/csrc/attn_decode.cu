// attn_decode.cu -- GQA flash-decode over the HBM-resident KV cache.
//
// Replaces the reference's three attention passes (shaders/attention.wgsl:31-58 scores,
// :73-135 softmax over a materialised scores[heads, ctx] buffer, :152-170 serial P.V),
// dispatched from engine/wgpu_engine.rs:666-726, for one query position (decode).
// Semantics follow candle quantized_llama forward_attn: score = (q.k) * (1/sqrt(hd)), no
// mask for a single query (keys 0..pos), softmax, then P.V; head h reads kv head
// h / (n_heads / n_kv) (repeat_kv).
//
// Layout: per layer K and V caches are [n_kv][max_seq][hd], fp16 (default) or f32, so the
// keys of one kv head at consecutive positions are one contiguous run.
//
// Work split: grid = (n_kv, max_splits).  The kernel reads the position, uses
// S = min(max_splits, ceil(kv_len / 128)) splits of the keys 0..pos (the CTAs of higher
// splits exit at once) and gives each split a contiguous range.  A CTA of 8 warps streams
// its range through a ring of 3-6 stages, each one 1-D TMA bulk copy of 64 K rows and one of
// 64 V rows (32 of each for f32); the last warp to finish a stage refills it, so no warp is
// set aside for copies.  Warp w owns rows 8w..8w+7 of every stage and keeps its own online
// softmax for all query heads of the group: a half-warp handles one row, each of its 16
// lanes a slice of hd/16 elements with the matching q slice in registers; dot products
// reduce over the 16 lanes with shuffles, and scores and P.V use packed f32x2 FMAs.  At the
// end the warps' states are merged in shared memory in warp order.  With S = 1 the CTA
// writes the output; otherwise it writes (m, l, acc) to scratch and the last CTA of the kv
// head (atomic ticket) merges the splits in split order, so the result does not depend on
// scheduling.
#include <algorithm>

#include "act.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace tptc {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxStages = 6;
constexpr int kRingBudget = 96 * 1024;  // two CTAs per SM
constexpr int kMinPerSplit = 128;       // positions per split before another split is used
constexpr int kMaxSplits = 64;

template <typename KV>
struct KvTraits;
template <>
struct KvTraits<__half> {
    static constexpr int kRows = 64;  // rows of K (and of V) per stage
    // 2 * N2 consecutive elements at p (p aligned to 4 * N2 bytes when N2 is 4, else 4 bytes)
    template <int N2>
    __device__ static void load(const __half* p, float2 (&v)[N2]) {
        if constexpr (N2 == 4) {
            const uint4 u = *reinterpret_cast<const uint4*>(p);
            const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = __half22float2(h[i]);
        } else {
#pragma unroll
            for (int i = 0; i < N2; i++) v[i] = __half22float2(reinterpret_cast<const __half2*>(p)[i]);
        }
    }
    __device__ static void store(__half* p, float v) { *p = __float2half_rn(v); }
};
template <>
struct KvTraits<float> {
    static constexpr int kRows = 32;
    template <int N2>
    __device__ static void load(const float* p, float2 (&v)[N2]) {
        if constexpr (N2 % 2 == 0) {
#pragma unroll
            for (int i = 0; i < N2 / 2; i++) {
                const float4 f = reinterpret_cast<const float4*>(p)[i];
                v[2 * i] = make_float2(f.x, f.y);
                v[2 * i + 1] = make_float2(f.z, f.w);
            }
        } else {
#pragma unroll
            for (int i = 0; i < N2; i++) v[i] = reinterpret_cast<const float2*>(p)[i];
        }
    }
    __device__ static void store(float* p, float v) { *p = v; }
};

// 2^x (PTX ex2.approx: a few ulp of relative error; 2^-inf = 0).  Scores are kept in the
// log2 domain (scaled by log2 e), so softmax weights are 2^(s - m).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// One halving step of a reduce-scatter over lane pairs (lane, lane ^ mask): the lane with
// the mask bit clear keeps v[0, N) and the other v[N, 2N), each adding its partner's copy.
template <int N, int GM>
__device__ __forceinline__ void rs_halve(float (&v)[GM], int mask, bool upper) {
#pragma unroll
    for (int j = 0; j < N; j++) {
        const float send = upper ? v[j] : v[N + j];
        const float keep = upper ? v[N + j] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
    }
}

// Sums v[g] (g < GM) over the 16 lanes of a half-warp and returns, in every lane, the sum of
// head g = l16 / (16 / GM); the 16 / GM lanes of a head hold bit-identical sums.  Costs
// GM - 1 + 4 - log2(GM) shuffles instead of 4 * GM.
template <int GM>
__device__ __forceinline__ float reduce_scatter16(float (&v)[GM], int l16) {
    if constexpr (GM == 8) {
        rs_halve<4>(v, 8, l16 & 8);
        rs_halve<2>(v, 4, l16 & 4);
        rs_halve<1>(v, 2, l16 & 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
    } else if constexpr (GM == 4) {
        rs_halve<2>(v, 8, l16 & 8);
        rs_halve<1>(v, 4, l16 & 4);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
    } else if constexpr (GM == 2) {
        rs_halve<1>(v, 8, l16 & 8);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 4);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
    } else {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 8);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 4);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
    }
    return v[0];
}

// 16-byte global -> shared copy through L2 only (cp.async.cg), completed by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Record of one (split or warp, head) state: m, l, two pad floats, acc[hd] -- hd + 4 floats,
// a multiple of 16 bytes, so a run of split records is one bulk copy.
__host__ __device__ constexpr int attn_rec(int hd) { return hd + 4; }
// Shared memory of the merges (inside the ring): the warp states [kWarps][G][rec]; for the
// split merge, staging for split records, then weights [G][kMaxSplits] and sums of l [G].
__host__ __device__ constexpr int attn_weight_bytes(int G) { return (G * kMaxSplits + G) * 4; }
__host__ __device__ constexpr int attn_merge_bytes(int G, int hd) {
    return kWarps * G * attn_rec(hd) * 4 > G * attn_rec(hd) * 4 + attn_weight_bytes(G)
               ? kWarps * G * attn_rec(hd) * 4
               : G * attn_rec(hd) * 4 + attn_weight_bytes(G);
}

// Effective split count and this split's key range for kv_len keys.
struct SplitRange {
    int S, t_begin, t_end;
};
__device__ __forceinline__ SplitRange split_range(int kv_len, int max_splits, int split) {
    SplitRange r;
    r.S = min(max_splits, max(1, (kv_len + kMinPerSplit - 1) / kMinPerSplit));
    int per = (kv_len + r.S - 1) / r.S;
    per = (per + 15) / 16 * 16;
    r.t_begin = min(kv_len, split * per);
    r.t_end = min(kv_len, r.t_begin + per);
    return r;
}

// The kv head's outputs (G * HD floats staged at `ob`) as blocks of the next GEMV's prepared
// activation: warp w quantises block w.  All threads of the CTA call it after a barrier.
__device__ __forceinline__ void attn_store_act(const AttnDecodeParams& p, const float* ob, int kvh, int G, int HD) {
    const int nblk = G * HD / 256, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int w = warp; w < nblk; w += kWarps) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = ob[w * 256 + 8 * lane + i];
        act_store_block(p.act, p.act_transposed, p.act_nb, p.act_out, kvh * nblk + w, v, lane);
    }
}

// The CTA's end, shared by both decode kernels: the warp states [kWarps][G][rec] are in
// shared memory (written after a barrier that ended all use of the ring).  Merges them in
// warp order into the CTA's (M, L, A); with one split writes the output, else the split
// record, and the last CTA of the kv head (atomic ticket) merges the splits in split order
// and writes the output (and the next GEMV's activation).
template <int GM, int HD>
__device__ __forceinline__ void attn_finish(const AttnDecodeParams& p, uint8_t* smem, float* qs, int ring_bytes,
                                            const SplitRange& sr, int kvh, int split, int G, int* is_last_p) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rec = attn_rec(HD);
    const float* wst = reinterpret_cast<const float*>(smem);
    int& is_last = *is_last_p;
    // merge the warps in warp order: the CTA's (M, L, A)
    const int S = sr.S;
    float* part = p.partial + ((int64_t)kvh * p.splits + split) * G * rec;
    // thread c handles columns 4c .. 4c + 3 of the group's heads (float4 loads)
    for (int c = tid; c < G * HD / 4; c += kThreads) {
        const int g = 4 * c / HD, d = 4 * c % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; w++) M = fmaxf(M, wst[(w * G + g) * rec]);
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f;
        float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kWarps; w++) {
            const float* ws = wst + (w * G + g) * rec;
            const float e = ex2(ws[0] - Mu);
            const float4 v = *reinterpret_cast<const float4*>(ws + 4 + d);
            L = fmaf(ws[1], e, L);
            A.x = fmaf(v.x, e, A.x);
            A.y = fmaf(v.y, e, A.y);
            A.z = fmaf(v.z, e, A.z);
            A.w = fmaf(v.w, e, A.w);
        }
        if (S == 1) {
            const float4 o = make_float4(A.x / L, A.y / L, A.z / L, A.w / L);
            *reinterpret_cast<float4*>(p.out + (kvh * G + g) * HD + d) = o;
            *reinterpret_cast<float4*>(qs + 4 * c) = o;  // q is in registers by now: the buffer stages the outputs
        } else {
            *reinterpret_cast<float4*>(part + g * rec + 4 + d) = A;
            if (d == 0) {
                part[g * rec] = M;
                part[g * rec + 1] = L;
            }
        }
    }
    if (S == 1) {
        if (p.act_out) {
            __syncthreads();
            attn_store_act(p, qs, kvh, G, HD);
        }
        return;
    }
    // the split ticket: after the barrier one thread takes it with an acquire-release atomic.
    // Its release orders the whole CTA's record stores before the ticket (they precede it
    // through the barrier); in the last CTA its acquire orders every other CTA's records
    // before the reads that follow the next barrier.
    __syncthreads();
    if (tid == 0) {
        int prev;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(p.counters + kvh) : "memory");
        is_last = prev == S - 1;
    }
    __syncthreads();
    if (!is_last) return;
    // merge the splits in split order.  The split records come into shared memory by 16-byte
    // cp.async copies from every thread (as many whole records as fit, in chunks), all in
    // flight together; meanwhile warp g reads the (m, l) of every split of head g with plain
    // loads and turns them into weights 2^(m_s - M) and the sum of l.
    const float* base = p.partial + (int64_t)kvh * p.splits * G * rec;
    const int stage_bytes = ring_bytes - attn_weight_bytes(G);
    float* stage = reinterpret_cast<float*>(smem);
    float* wgt = reinterpret_cast<float*>(smem + stage_bytes);  // [G][kMaxSplits]
    float* lsum = wgt + G * kMaxSplits;                         // [G]
    const int Sc = max(1, stage_bytes / (G * rec * 4));          // splits per chunk
    auto fetch = [&](int c0) {  // records of splits c0 .. c0 + Sc - 1 into the stage
        const int n16 = min(Sc, S - c0) * G * rec / 4;
        const float4* src = reinterpret_cast<const float4*>(base + (int64_t)c0 * G * rec);
        for (int i = tid; i < n16; i += kThreads) cp_async16(stage + 4 * i, src + i);
        cp_async_commit();
    };
    fetch(0);
    if (warp < G) {
        const int g = warp;
        float ms[2], ls2[2];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int sp = lane + 32 * k;
            ms[k] = sp < S ? __ldcg(base + (sp * G + g) * rec) : -INFINITY;
            ls2[k] = sp < S ? __ldcg(base + (sp * G + g) * rec + 1) : 0.f;
        }
        const float M = warp_max(fmaxf(ms[0], ms[1]));
        const float Mu = M == -INFINITY ? 0.f : M;
        float L = 0.f;
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int sp = lane + 32 * k;
            const float w = ex2(ms[k] - Mu);
            if (sp < S) wgt[g * kMaxSplits + sp] = w;
            L = fmaf(ls2[k], w, L);
        }
        L = warp_sum(L);
        if (lane == 0) lsum[g] = L;
    }
    // thread t sums columns 4c .. 4c + 3 (c = t % NC4) over the splits of partition
    // t / NC4 (splits sp with sp % NP == partition), float4 loads; the partitions' sums are
    // then added in partition order
    const int NC4 = G * HD / 4, NP = max(1, kThreads / NC4);
    const int c4 = tid % NC4, part_i = tid / NC4;
    float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < S; c0 += Sc) {
        const int n0 = min(Sc, S - c0);
        cp_async_wait_all();
        __syncthreads();  // the chunk (and, the first time, the weights) in shared memory
        if (part_i < NP) {
            const int g = 4 * c4 / HD, d = 4 * c4 % HD;
            const float* wv = wgt + g * kMaxSplits + c0;
            for (int sp = part_i; sp < n0; sp += NP) {
                const float4 v = *reinterpret_cast<const float4*>(stage + (sp * G + g) * rec + 4 + d);
                const float w = wv[sp];
                acc4.x = fmaf(v.x, w, acc4.x);
                acc4.y = fmaf(v.y, w, acc4.y);
                acc4.z = fmaf(v.z, w, acc4.z);
                acc4.w = fmaf(v.w, w, acc4.w);
            }
        }
        if (c0 + Sc < S) {
            __syncthreads();  // staging consumed
            fetch(c0 + Sc);
        }
    }
    __syncthreads();  // the stage is free: it takes the partitions' sums
    float4* psum = reinterpret_cast<float4*>(stage);  // [NP][NC4]
    if (part_i < NP) psum[part_i * NC4 + c4] = acc4;
    __syncthreads();
    for (int c = tid; c < NC4; c += kThreads) {
        float4 o = psum[c];
        for (int q = 1; q < NP; q++) {
            const float4 v = psum[q * NC4 + c];
            o.x += v.x;
            o.y += v.y;
            o.z += v.z;
            o.w += v.w;
        }
        const int g = 4 * c / HD, d = 4 * c % HD;
        const float il = 1.f / lsum[g];
        o = make_float4(o.x * il, o.y * il, o.z * il, o.w * il);
        *reinterpret_cast<float4*>(p.out + (kvh * G + g) * HD + d) = o;
        *reinterpret_cast<float4*>(qs + 4 * c) = o;
    }
    if (p.act_out) {
        __syncthreads();
        attn_store_act(p, qs, kvh, G, HD);
    }
    if (tid == 0) p.counters[kvh] = 0;
}

// N2: float2 pairs of the head dimension per lane (hd = 32 * N2); GM: most query heads per
// kv head.
template <typename KV, int N2, int GM>
__global__ void __launch_bounds__(kThreads, GM <= 4 ? 2 : 1) attn_decode_kernel(const __grid_constant__ AttnDecodeParams p) {
    using Tr = KvTraits<KV>;
    constexpr int kR = Tr::kRows;
    constexpr int kRW = kR / kWarps;  // rows per warp per stage
    constexpr int kIt = kRW / 2;      // two rows (half-warps) per iteration
    constexpr int DPL = 2 * N2;       // head-dimension elements per lane
    constexpr int HD = 16 * DPL;
    constexpr int kStageElems = kR * HD;  // K (or V) elements per stage
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMaxStages];
    __shared__ int done_warps[kMaxStages];
    __shared__ int is_last, abort_s;

    const int kvh = blockIdx.x, split = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.n_heads / p.n_kv, S_ring = p.stages;
    KV* ring = reinterpret_cast<KV*>(smem);  // [S_ring][K|V][kR][HD]
    const int ring_bytes = max(S_ring * 2 * kStageElems * (int)sizeof(KV), attn_merge_bytes(G, HD));
    float* qs = reinterpret_cast<float*>(smem + ring_bytes);  // [G][HD]

    if (tid == 0) {
        for (int s = 0; s < S_ring; s++) {
            mbar_init(&full[s], 1);
            done_warps[s] = 0;
        }
        fence_mbar_init();
        abort_s = 0;
    }
    // Before waiting for the previous kernel (the q|k|v GEMV): the position (set before the
    // step began) and the key/value rows below it (written by earlier steps) are final, so
    // the range is known and every tile except the one holding `pos` can be in flight.
    const int kv_len = *p.pos + 1;
    if (kv_len < 1 || kv_len > p.max_seq) {  // position outside the cache: flag it, touch nothing
        if (tid == 0 && kvh == 0 && split == 0 && p.err) atomicExch(p.err, TPTC_ERR_ARG);
        return;
    }
    const SplitRange sr = split_range(kv_len, p.splits, split);
    if (split >= sr.S) return;
    const int t_begin = sr.t_begin, t_end = sr.t_end;
    const int ntiles = (t_end - t_begin + kR - 1) / kR;
    const int pos = kv_len - 1, half = HD / 2;
    const bool owner = pos >= t_begin && pos < t_end;  // this CTA writes the new key
    const int tile_pos = owner ? (pos - t_begin) / kR : -1;

    // Stage s of tile t holds 1-D bulk copies of kR K rows and kR V rows.  Tid 0 issues the
    // first tile before waiting for the previous kernel and the other first stages once the
    // queries are staged -- never the tile holding `pos` before this CTA has written its key
    // (its value row comes from the previous kernel); afterwards the last warp to finish a
    // stage refills it (done_warps).  Only one tile goes out before the wait: the query loads
    // that follow the wait are L2 hits, and behind a burst of every CTA's whole ring (28 MB at
    // C5) they took 3.7 us instead of about 1 (measured with globaltimer stamps per CTA).
    const KV* kh = static_cast<const KV*>(p.kcache) + (int64_t)kvh * p.max_seq * HD;
    const KV* vh = static_cast<const KV*>(p.vcache) + (int64_t)kvh * p.max_seq * HD;
    auto issue = [&](int t) {
        const int s = t % S_ring, t0 = t_begin + t * kR, n = min(kR, t_end - t0);
        const uint32_t bytes = (uint32_t)n * HD * sizeof(KV);
        KV* kb = ring + (int64_t)s * 2 * kStageElems;
        const uint64_t policy = l2_evict_first_policy();
        mbar_expect_tx(&full[s], 2 * bytes);
        bulk_g2s(kb, kh + (int64_t)t0 * HD, bytes, &full[s], policy);
        bulk_g2s(kb + kStageElems, vh + (int64_t)t0 * HD, bytes, &full[s], policy);
    };
    constexpr int kPreWait = 1;  // tiles issued before the wait
    if (tid == 0)
        for (int t = 0; t < kPreWait && t < S_ring && t < ntiles; t++)
            if (t != tile_pos) issue(t);

    pdl_wait();
    pdl_launch_dependents();

    // RoPE (candle rope_i: interleaved pairs, x0*c - x1*s, x0*s + x1*c; with rope_neox the
    // pairs are elements j and j + hd/2, candle rope) on the group's queries, staged in
    // shared memory
    const float* cs = p.rope_cos + (int64_t)pos * half;
    const float* sn = p.rope_sin + (int64_t)pos * half;
    for (int i = tid; i < G * half; i += kThreads) {
        const int g = i / half, j = i % half;
        const float* qg = p.q + (int64_t)(kvh * G + g) * HD;
        const int ia = p.rope_neox ? j : 2 * j, ib = p.rope_neox ? j + half : 2 * j + 1;  // the rotated pair
        const float q0 = qg[ia], q1 = qg[ib], c = cs[j], s = sn[j];
        const float r0 = __fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, s));
        const float r1 = __fadd_rn(__fmul_rn(q0, s), __fmul_rn(q1, c));
        qs[g * HD + ia] = r0;
        qs[g * HD + ib] = r1;
        if (p.q_out && split == 0) {
            p.q_out[(int64_t)(kvh * G + g) * HD + ia] = r0;
            p.q_out[(int64_t)(kvh * G + g) * HD + ib] = r1;
        }
    }
    // The owner rotates this step's key and stores it in the cache; the proxy fence orders
    // those generic stores before the bulk-copy read of the same row.
    if (owner) {
        KV* krow = static_cast<KV*>(p.kcache) + ((int64_t)kvh * p.max_seq + pos) * HD;
        for (int j = tid; j < half; j += kThreads) {
            const int ia = p.rope_neox ? j : 2 * j, ib = p.rope_neox ? j + half : 2 * j + 1;
            const float k0 = p.kraw[kvh * HD + ia], k1 = p.kraw[kvh * HD + ib], c = cs[j], s = sn[j];
            Tr::store(krow + ia, __fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, s)));
            Tr::store(krow + ib, __fadd_rn(__fmul_rn(k0, s), __fmul_rn(k1, c)));
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    __syncthreads();
    if (tid == 0)
        for (int t = kPreWait; t < S_ring && t < ntiles; t++)
            if (t != tile_pos) issue(t);
    if (tid == 0 && tile_pos >= 0 && tile_pos < S_ring) issue(tile_pos);

    const int hw = lane >> 4, l16 = lane & 15;
    constexpr int LPG = 16 / GM;          // lanes per head after the reduce-scatter
    const float sl2 = p.scale * 1.4426950408889634f;  // scores in log2 units
    float2 qv[GM][N2];
#pragma unroll
    for (int g = 0; g < GM; g++)
#pragma unroll
        for (int j = 0; j < N2; j++)
            qv[g][j] = g < G ? reinterpret_cast<const float2*>(qs + g * HD + l16 * DPL)[j] : make_float2(0.f, 0.f);
    // running max and sum of head l16 / LPG (identical in both half-warps), accumulators of
    // every head over this lane's slice of the head dimension
    float m_h = -INFINITY, l_h = 0.f;
    float2 acc[GM][N2];
#pragma unroll
    for (int g = 0; g < GM; g++)
#pragma unroll
        for (int j = 0; j < N2; j++) acc[g][j] = make_float2(0.f, 0.f);

    bool ok = true;
    for (int t = 0; t < ntiles; t++) {
        const int s = t % S_ring, t0 = t_begin + t * kR, n = min(kR, t_end - t0);
        ok = mbar_wait_bounded(&full[s], (t / S_ring) & 1, p.err);
        if (!ok) break;
        const KV* kt = ring + (int64_t)s * 2 * kStageElems;
        const KV* vt = kt + kStageElems;
        float sc[kIt];  // score of (row 2i + hw, head l16 / LPG)
#pragma unroll
        for (int i = 0; i < kIt; i++) {
            const int r = warp * kRW + 2 * i + hw;
            float2 kv[N2];
            Tr::template load<N2>(kt + r * HD + l16 * DPL, kv);
            float d[GM];
#pragma unroll
            for (int g = 0; g < GM; g++) {
                float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int j = 0; j < N2; j++) d2 = __ffma2_rn(qv[g][j], kv[j], d2);
                d[g] = d2.x + d2.y;
            }
            const float dot = reduce_scatter16<GM>(d, l16);
            sc[i] = r < n ? dot * sl2 : -INFINITY;
        }
        // online softmax of this warp's rows of the stage
        float mt = sc[0];
#pragma unroll
        for (int i = 1; i < kIt; i++) mt = fmaxf(mt, sc[i]);
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
        const float mn = fmaxf(m_h, mt);
        const float mu = mn == -INFINITY ? 0.f : mn;
        const float alpha = ex2(m_h - mu);
        float ls = 0.f;
#pragma unroll
        for (int i = 0; i < kIt; i++) {
            sc[i] = ex2(sc[i] - mu);
            ls += sc[i];
        }
        ls += __shfl_xor_sync(0xffffffffu, ls, 16);
        l_h = l_h * alpha + ls;
        m_h = mn;
#pragma unroll
        for (int g = 0; g < GM; g++) {
            const float a = __shfl_sync(0xffffffffu, alpha, g * LPG);
            const float2 a2 = make_float2(a, a);
#pragma unroll
            for (int j = 0; j < N2; j++) acc[g][j] = __fmul2_rn(acc[g][j], a2);
        }
        // P.V
#pragma unroll
        for (int i = 0; i < kIt; i++) {
            const int r = warp * kRW + 2 * i + hw;
            float pg[GM];
#pragma unroll
            for (int g = 0; g < GM; g++) pg[g] = __shfl_sync(0xffffffffu, sc[i], (lane & 16) + g * LPG);
            float2 vv[N2];
            if (r < n) {
                Tr::template load<N2>(vt + r * HD + l16 * DPL, vv);
            } else {
#pragma unroll
                for (int j = 0; j < N2; j++) vv[j] = make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int g = 0; g < GM; g++) {
                const float2 p2 = make_float2(pg[g], pg[g]);
#pragma unroll
                for (int j = 0; j < N2; j++) acc[g][j] = __ffma2_rn(p2, vv[j], acc[g][j]);
            }
        }
        __syncwarp();
        if (lane == 0) {  // the last warp done with stage s refills it
            __threadfence_block();
            if (atomicAdd(&done_warps[s], 1) == kWarps - 1) {
                done_warps[s] = 0;
                __threadfence_block();
                if (t + S_ring < ntiles) {
                    fence_proxy_async_smem();
                    issue(t + S_ring);
                }
            }
        }
    }
    if (!ok) abort_s = 1;

    // the two half-warps saw different rows under the same running max
#pragma unroll
    for (int g = 0; g < GM; g++)
#pragma unroll
        for (int j = 0; j < N2; j++) {
            acc[g][j].x += __shfl_xor_sync(0xffffffffu, acc[g][j].x, 16);
            acc[g][j].y += __shfl_xor_sync(0xffffffffu, acc[g][j].y, 16);
        }

    __syncthreads();  // every warp is done with the ring: reuse it for the warp states
    if (abort_s) return;
    const int rec = attn_rec(HD);
    float* wst = reinterpret_cast<float*>(smem);  // [warp][G][rec] = (m, l, -, -, acc[HD])
    if (hw == 0) {
        const int gh = l16 / LPG;
        if (l16 % LPG == 0 && gh < G) {
            wst[(warp * G + gh) * rec] = m_h;
            wst[(warp * G + gh) * rec + 1] = l_h;
        }
#pragma unroll
        for (int g = 0; g < GM; g++) {
            if (g >= G) continue;
            float* w = wst + (warp * G + g) * rec + 4 + l16 * DPL;
#pragma unroll
            for (int j = 0; j < N2; j++) {
                w[2 * j] = acc[g][j].x;
                w[2 * j + 1] = acc[g][j].y;
            }
        }
    }
    __syncthreads();

    attn_finish<GM, HD>(p, smem, qs, ring_bytes, sr, kvh, split, G, &is_last);
}

// ---------------------------------------------------------------------------------------
// Tensor-core variant for the fp16 cache.  Same split, ring, position ownership and merge as
// attn_decode_kernel; the products run on mma.sync (m16n8k16, fp16 in, f32 accumulate) with
// the keys as the M dimension:
//   S^T[key][head] = K[key][:] . Q^T[:][head]     (A = K rows by ldmatrix, B = Q^T in registers)
//   O^T[dim][head] += V^T[dim][key] . P^T[key][head]   (A = V^T by ldmatrix.trans, B = P^T)
// so the n = 8 columns hold up to 8 query heads of the group.  Each stage is a K and a V tile
// of 64 positions brought by 2-D TMA with 128-byte swizzle (64-column boxes; for head_dim 96
// the second box's last 32 columns are zero-filled and never read).  Warps 0-3 take the even
// tiles and warps 4-7 the odd ones, 16 positions each.  Q and P enter the tensor core as a
// high and a low fp16 part (x = hi + lo to about 22 bits), so scores and weights keep f32
// precision against the fp16 keys and values.  Softmax is base 2 with a lazily moved
// reference maximum per head: it moves (and O^T and l are rescaled) only when a score
// exceeds it by more than 8, so the weights stay below 256.
namespace tcd {
constexpr int kKeys = 64;         // positions per stage
constexpr int kBox = 64 * 128;    // one TMA box: 64 rows x 64 fp16 columns (128 B), swizzled
}  // namespace tcd

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 1-D bulk copy global -> shared without a cache hint; 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s_nohint(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ uint32_t half2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// (x0, x1) as a high and a low fp16 pair: hi = fp16(x), lo = fp16(x - hi)
__device__ __forceinline__ void split_half2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 f = __half22float2(h);
    hi = half2_bits(h);
    lo = half2_bits(__floats2half2_rn(x0 - f.x, x1 - f.y));
}
// Byte offset of (row, column) in a tile of 64-column boxes with 128-byte swizzle: the
// 16-byte chunk c of a row sits at chunk c ^ (row % 8).
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
    return (uint32_t)((col >> 6) * tcd::kBox + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4));
}

template <int HD, int GM>
__global__ void __launch_bounds__(kThreads, 2)
    attn_decode_tc_kernel(const __grid_constant__ AttnDecodeParams p, const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv) {
    constexpr int NB = (HD + 63) / 64;     // TMA boxes per row
    constexpr int KC = HD / 16;            // k-chunks of the scores = m-tiles of the output
    constexpr int kTile = NB * tcd::kBox;  // bytes of one K (or V) tile
    constexpr int kR = tcd::kKeys;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[kMaxStages], qbar;
    __shared__ int done_warps[kMaxStages];
    // issued[s]: the tile whose copies stage s holds or is receiving.  A warp group may run a
    // tile ahead of the other, and the previous use of a stage belongs to the other group
    // whenever the ring depth is odd; a parity wait cannot tell phase k + 2 from phase k, so
    // a consumer first sees its tile issued (its stage's previous phase is then complete).
    __shared__ volatile int issued[kMaxStages];
    __shared__ int is_last, abort_s;

    const int kvh = blockIdx.x, split = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.n_heads / p.n_kv, S_ring = p.stages;
    const int ring_bytes = max(S_ring * 2 * kTile, attn_merge_bytes(G, HD));
    float* qs = reinterpret_cast<float*>(smem + ring_bytes);  // [G][HD]
    float* csn = qs + G * HD;                                 // cos | sin of position pos
    float* kr = csn + HD;                                     // the new key before RoPE

    if (tid == 0) {
        for (int s = 0; s < S_ring; s++) {
            mbar_init(&full[s], 1);
            done_warps[s] = 0;
            issued[s] = -1;
        }
        mbar_init(&qbar, 1);
        fence_mbar_init();
        abort_s = 0;
    }
    const int kv_len = *p.pos + 1;
    if (kv_len < 1 || kv_len > p.max_seq) {  // position outside the cache: flag it, touch nothing
        if (tid == 0 && kvh == 0 && split == 0 && p.err) atomicExch(p.err, TPTC_ERR_ARG);
        return;
    }
    const SplitRange sr = split_range(kv_len, p.splits, split);
    if (split >= sr.S) return;
    const int t_begin = sr.t_begin, t_end = sr.t_end;
    const int ntiles = (t_end - t_begin + kR - 1) / kR;
    const int pos = kv_len - 1, half = HD / 2;
    const bool owner = pos >= t_begin && pos < t_end;
    const int tile_pos = owner ? (pos - t_begin) / kR : -1;
    const int row0 = kvh * p.max_seq + t_begin;  // tensor-map row of the split's first key

    // stage s of tile t: K tile then V tile, NB boxes each; rows past the split (or past the
    // tensor: zero fill) are masked (K) and zeroed (V) by the warps that own them
    auto issue = [&](int t) {
        const int s = t % S_ring;
        uint8_t* kb = smem + s * 2 * kTile;
        const uint64_t policy = l2_evict_first_policy();
        mbar_expect_tx(&full[s], 2 * kTile);
#pragma unroll
        for (int b = 0; b < NB; b++) {
            tma_load_2d_hint(kb + b * tcd::kBox, &tk, b * 64, row0 + t * kR, &full[s], policy);
            tma_load_2d_hint(kb + kTile + b * tcd::kBox, &tv, b * 64, row0 + t * kR, &full[s], policy);
        }
        __threadfence_block();
        issued[s] = t;
    };
    constexpr int kPreWait = 1;  // tiles issued before the wait (see attn_decode_kernel)
    if (tid == 0)
        for (int t = 0; t < kPreWait && t < S_ring && t < ntiles; t++)
            if (t != tile_pos) issue(t);

    pdl_wait();
    pdl_launch_dependents();

    // The group's queries, the RoPE row of `pos` and (owner) the new key come in by bulk
    // copies issued ahead of the ring's other first tiles: plain loads queued behind a burst of
    // tile copies took several microseconds.
    if (tid == 0) {
        mbar_expect_tx(&qbar, (uint32_t)((G * HD + HD + (owner ? HD : 0)) * 4));
        bulk_g2s_nohint(qs, p.q + (int64_t)kvh * G * HD, (uint32_t)(G * HD * 4), &qbar);
        bulk_g2s_nohint(csn, p.rope_cos + (int64_t)pos * half, (uint32_t)(half * 4), &qbar);
        bulk_g2s_nohint(csn + half, p.rope_sin + (int64_t)pos * half, (uint32_t)(half * 4), &qbar);
        if (owner) bulk_g2s_nohint(kr, p.kraw + (int64_t)kvh * HD, (uint32_t)(HD * 4), &qbar);
        for (int t = kPreWait; t < S_ring && t < ntiles; t++)
            if (t != tile_pos) issue(t);
    }
    bool ok = mbar_wait_bounded(&qbar, 0, p.err);
    // RoPE on the group's queries (candle rope_i, or rope with rope_neox), in place
    for (int i = tid; i < G * half && ok; i += kThreads) {
        const int g = i / half, j = i % half;
        const int ia = p.rope_neox ? j : 2 * j, ib = p.rope_neox ? j + half : 2 * j + 1;  // the rotated pair
        const float q0 = qs[g * HD + ia], q1 = qs[g * HD + ib], c = csn[j], s = csn[half + j];
        const float r0 = __fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, s));
        const float r1 = __fadd_rn(__fmul_rn(q0, s), __fmul_rn(q1, c));
        qs[g * HD + ia] = r0;
        qs[g * HD + ib] = r1;
        if (p.q_out && split == 0) {
            p.q_out[(int64_t)(kvh * G + g) * HD + ia] = r0;
            p.q_out[(int64_t)(kvh * G + g) * HD + ib] = r1;
        }
    }
    if (owner && ok) {  // this step's key, rotated, into the cache before any read of its tile
        __half* krow = static_cast<__half*>(p.kcache) + ((int64_t)kvh * p.max_seq + pos) * HD;
        for (int j = tid; j < half; j += kThreads) {
            const int ia = p.rope_neox ? j : 2 * j, ib = p.rope_neox ? j + half : 2 * j + 1;
            const float k0 = kr[ia], k1 = kr[ib], c = csn[j], s = csn[half + j];
            krow[ia] = __float2half_rn(__fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, s)));
            krow[ib] = __float2half_rn(__fadd_rn(__fmul_rn(k0, s), __fmul_rn(k1, c)));
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    __syncthreads();
    if (tid == 0 && ok && tile_pos >= 0 && tile_pos < S_ring) issue(tile_pos);

    const int g8 = lane >> 2, t4 = lane & 3;       // mma fragment coordinates
    const int grp = warp >> 2, quarter = warp & 3;  // tile parity and 16-position slice
    // Q^T as the B operand (k = head dimension, n = query head g8), high and low parts
    uint32_t qh[KC][2], ql[KC][2];
#pragma unroll
    for (int c = 0; c < KC; c++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int d = 16 * c + 2 * t4 + 8 * e;
            const float x0 = g8 < G ? qs[g8 * HD + d] : 0.f, x1 = g8 < G ? qs[g8 * HD + d + 1] : 0.f;
            split_half2(x0, x1, qh[c][e], ql[c][e]);
        }
    // ldmatrix row addresses: K (A of the scores) rows r, r + 8 at columns +0 / +8; V (A of
    // the output, transposed) rows r / r + 8 at columns +0, +8
    const int krow = 16 * quarter + (lane & 7) + ((lane >> 3) & 1) * 8, kcol = (lane >> 4) * 8;
    const int vrow = 16 * quarter + (lane & 7) + (lane >> 4) * 8, vcol = ((lane >> 3) & 1) * 8;
    const float sl2 = p.scale * 1.4426950408889634f;
    float m_ref[2] = {-INFINITY, -INFINITY}, l_part[2] = {0.f, 0.f};  // heads 2 t4, 2 t4 + 1
    float o[KC][4];
#pragma unroll
    for (int i = 0; i < KC; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    for (int t = grp; t < ntiles && ok; t += 2) {
        const int s = t % S_ring, n = min(kR, t_end - t_begin - t * kR);
        ok = false;
        for (uint32_t i = 0; i < kWaitPolls; ++i)
            if (issued[s] == t) {
                ok = true;
                break;
            }
        if (!ok) {
            if (p.err) atomicExch(p.err, TPTC_ERR_TIMEOUT);
            break;
        }
        __threadfence_block();
        ok = mbar_wait_bounded(&full[s], (t / S_ring) & 1, p.err);
        if (!ok) break;
        uint8_t* kt = smem + s * 2 * kTile;
        const uint32_t kb = smem_u32(kt), vb = kb + kTile;
        float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < KC; c++) {
            uint32_t a[4];
            ldsm_x4(kb + sw128_off(krow, 16 * c + kcol), a);
            mma_16816(sacc, a, qh[c][0], qh[c][1]);
            mma_16816(sacc, a, ql[c][0], ql[c][1]);
        }
        // scores (log2 units) of positions r and r + 8 for heads 2 t4, 2 t4 + 1
        const int r = 16 * quarter + g8;
        float sc[4];
        sc[0] = r < n ? sacc[0] * sl2 : -INFINITY;
        sc[1] = r < n ? sacc[1] * sl2 : -INFINITY;
        sc[2] = r + 8 < n ? sacc[2] * sl2 : -INFINITY;
        sc[3] = r + 8 < n ? sacc[3] * sl2 : -INFINITY;
        float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
        if (__any_sync(0xffffffffu, mx0 > m_ref[0] + 8.f || mx1 > m_ref[1] + 8.f)) {
#pragma unroll
            for (int sh = 4; sh < 32; sh <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
            }
            const float n0 = fmaxf(m_ref[0], mx0), n1 = fmaxf(m_ref[1], mx1);
            const float a0 = n0 == -INFINITY ? 1.f : ex2(m_ref[0] - n0);
            const float a1 = n1 == -INFINITY ? 1.f : ex2(m_ref[1] - n1);
            m_ref[0] = n0;
            m_ref[1] = n1;
            l_part[0] *= a0;
            l_part[1] *= a1;
#pragma unroll
            for (int i = 0; i < KC; i++) {
                o[i][0] *= a0;
                o[i][2] *= a0;
                o[i][1] *= a1;
                o[i][3] *= a1;
            }
        }
        const float mu0 = m_ref[0] == -INFINITY ? 0.f : m_ref[0];
        const float mu1 = m_ref[1] == -INFINITY ? 0.f : m_ref[1];
        const float pw0 = ex2(sc[0] - mu0), pw1 = ex2(sc[1] - mu1), pw2 = ex2(sc[2] - mu0), pw3 = ex2(sc[3] - mu1);
        l_part[0] += pw0 + pw2;
        l_part[1] += pw1 + pw3;
        // P^T (rows: positions r, r + 8; columns: heads) transposed into B fragments
        uint32_t ph0, pl0, ph1, pl1;
        split_half2(pw0, pw1, ph0, pl0);
        split_half2(pw2, pw3, ph1, pl1);
        const uint32_t bh0 = movmatrix_trans(ph0), bh1 = movmatrix_trans(ph1);
        const uint32_t bl0 = movmatrix_trans(pl0), bl1 = movmatrix_trans(pl1);
        if (16 * quarter + 16 > n) {
            // V rows of this slice past the range may hold anything: zero them (their weight is 0)
            uint8_t* vt = kt + kTile;
            for (int idx = lane; idx < 16 * NB * 8; idx += 32) {
                const int rr = 16 * quarter + idx / (NB * 8), b = (idx / 8) % NB, ch = idx & 7;
                if (rr >= n) *reinterpret_cast<uint4*>(vt + b * tcd::kBox + rr * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
            }
            fence_proxy_async_smem();  // before the stage is refilled by TMA
            __syncwarp();
        }
#pragma unroll
        for (int i = 0; i < KC; i++) {
            uint32_t a[4];
            ldsm_x4_trans(vb + sw128_off(vrow, 16 * i + vcol), a);
            mma_16816(o[i], a, bh0, bh1);
            mma_16816(o[i], a, bl0, bl1);
        }
        __syncwarp();
        if (lane == 0) {  // the last of the tile's four warps refills its stage
            __threadfence_block();
            if (atomicAdd(&done_warps[s], 1) == 3) {
                done_warps[s] = 0;
                __threadfence_block();
                if (t + S_ring < ntiles) {
                    fence_proxy_async_smem();
                    issue(t + S_ring);
                }
            }
        }
    }
    if (!ok) abort_s = 1;
#pragma unroll
    for (int sh = 4; sh < 32; sh <<= 1) {
        l_part[0] += __shfl_xor_sync(0xffffffffu, l_part[0], sh);
        l_part[1] += __shfl_xor_sync(0xffffffffu, l_part[1], sh);
    }

    __syncthreads();  // every warp is done with the ring: reuse it for the warp states
    if (abort_s) return;
    const int rec = attn_rec(HD);
    float* wst = reinterpret_cast<float*>(smem);  // [warp][G][rec] = (m, l, -, -, acc[HD])
#pragma unroll
    for (int e = 0; e < 2; e++) {
        const int h = 2 * t4 + e;
        if (h >= G) continue;
        float* w = wst + (warp * G + h) * rec;
        if (g8 == 0) {
            w[0] = m_ref[e];
            w[1] = l_part[e];
        }
#pragma unroll
        for (int i = 0; i < KC; i++) {
            w[4 + 16 * i + g8] = o[i][e];
            w[4 + 16 * i + g8 + 8] = o[i][2 + e];
        }
    }
    __syncthreads();
    attn_finish<GM, HD>(p, smem, qs, ring_bytes, sr, kvh, split, G, &is_last);
}

int attn_tc_stages(int hd) {
    const int stage = 2 * ((hd + 63) / 64) * tcd::kBox;
    return std::max(2, std::min(kMaxStages, kRingBudget / stage));
}

size_t attn_tc_smem(int n_heads, int n_kv, int hd) {
    const int G = n_heads / n_kv;
    const size_t ring = (size_t)attn_tc_stages(hd) * 2 * ((hd + 63) / 64) * tcd::kBox;
    return 1024 + std::max(ring, (size_t)attn_merge_bytes(G, hd)) + (size_t)(G + 2) * hd * 4;
}

using TcKernelFn = void (*)(AttnDecodeParams, CUtensorMap, CUtensorMap);

template <int GM>
TcKernelFn pick_tc_hd(int hd) {
    switch (hd) {
        case 64: return attn_decode_tc_kernel<64, GM>;
        case 96: return attn_decode_tc_kernel<96, GM>;
        case 128: return attn_decode_tc_kernel<128, GM>;
    }
    return nullptr;
}

TcKernelFn pick_tc_kernel(int hd, int G) {
    if (G == 1) return pick_tc_hd<1>(hd);
    if (G == 2) return pick_tc_hd<2>(hd);
    return G <= 4 ? pick_tc_hd<4>(hd) : pick_tc_hd<8>(hd);
}

template <typename KV>
int attn_stages(int hd) {
    const int stage = 2 * KvTraits<KV>::kRows * hd * (int)sizeof(KV);
    return std::max(2, std::min(kMaxStages, kRingBudget / stage));
}

template <typename KV>
size_t attn_smem(int n_heads, int n_kv, int hd) {
    const int G = n_heads / n_kv;
    const size_t ring = (size_t)attn_stages<KV>(hd) * 2 * KvTraits<KV>::kRows * hd * sizeof(KV);
    const size_t wst = (size_t)attn_merge_bytes(G, hd);
    return std::max(ring, wst) + (size_t)G * hd * 4;
}

using KernelFn = void (*)(AttnDecodeParams);

template <typename KV, int GM>
KernelFn pick_dpl(int hd) {
    switch (hd) {
        case 64: return attn_decode_kernel<KV, 2, GM>;
        case 96: return attn_decode_kernel<KV, 3, GM>;
        case 128: return attn_decode_kernel<KV, 4, GM>;
    }
    return nullptr;
}

KernelFn pick_kernel(int kv_f32, int hd, int G) {
    if (kv_f32) {
        if (G == 1) return pick_dpl<float, 1>(hd);
        if (G == 2) return pick_dpl<float, 2>(hd);
        return G <= 4 ? pick_dpl<float, 4>(hd) : pick_dpl<float, 8>(hd);
    }
    if (G == 1) return pick_dpl<__half, 1>(hd);
    if (G == 2) return pick_dpl<__half, 2>(hd);
    return G <= 4 ? pick_dpl<__half, 4>(hd) : pick_dpl<__half, 8>(hd);
}

}  // namespace

int attn_decode_splits(int n_kv, int max_seq, int sm_count) {
    // about 1.4 CTAs per SM over all kv heads at long context: at C5 (8 kv heads, 8K keys)
    // 26 splits stream the keys as fast as 37 (two per SM) and halve the split merge that the
    // last CTA of each kv head runs alone (measured per kernel with globaltimer stamps)
    const int s = std::max(1, (7 * sm_count + 5 * n_kv - 1) / (5 * n_kv));
    const int max_useful = std::max(1, (max_seq + kMinPerSplit - 1) / kMinPerSplit);
    return std::min(kMaxSplits, std::min(s, max_useful));
}

size_t attn_decode_partial_floats(int n_heads, int n_kv, int hd, int splits) {
    return (size_t)n_kv * splits * (n_heads / n_kv) * attn_rec(hd);
}

const char* attn_decode_shape_error(int n_heads, int n_kv, int hd, int max_seq) {
    if (n_heads <= 0 || n_kv <= 0 || hd <= 0 || max_seq <= 0) return "attention: sizes must be positive";
    if (n_heads % n_kv != 0) return "attention: n_heads must be a multiple of n_kv";
    if (n_heads / n_kv > 8) return "attention: at most 8 query heads per kv head";
    if (hd != 64 && hd != 96 && hd != 128) return "attention: head_dim must be 64, 96 or 128";
    return nullptr;
}

AttnScratch attn_scratch_layout(int n_heads, int n_kv, int hd, int max_seq, int sm_count) {
    AttnScratch s;
    s.splits = attn_decode_splits(n_kv, max_seq, sm_count);
    s.err = 0;
    s.counters = 256;
    s.partial = s.counters + ((size_t)n_kv * sizeof(int) + 255) / 256 * 256;
    s.total = s.partial + attn_decode_partial_floats(n_heads, n_kv, hd, s.splits) * sizeof(float);
    return s;
}

cudaError_t launch_attn_decode(const AttnDecodeParams& p_in, cudaStream_t st, bool pdl) {
    if (attn_decode_shape_error(p_in.n_heads, p_in.n_kv, p_in.hd, p_in.max_seq) || p_in.splits < 1 ||
        p_in.splits > kMaxSplits)
        return cudaErrorInvalidValue;
    AttnDecodeParams p = p_in;
    p.stages = p.kv_f32 ? attn_stages<float>(p.hd) : attn_stages<__half>(p.hd);
    // the tensor-core kernel reads the caches by TMA and q, the RoPE rows and the new key by
    // bulk copies: all 16-byte aligned
    const uintptr_t align = reinterpret_cast<uintptr_t>(p.kcache) | reinterpret_cast<uintptr_t>(p.vcache) |
                            reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.kraw) |
                            reinterpret_cast<uintptr_t>(p.rope_cos) | reinterpret_cast<uintptr_t>(p.rope_sin);
    const bool tc = !p.kv_f32 && (align & 15) == 0;
    CUtensorMap tk, tv;
    if (tc) {
        p.stages = attn_tc_stages(p.hd);
        const int64_t rows = (int64_t)p.n_kv * p.max_seq;
        cudaError_t e = make_tmap_f16(&tk, static_cast<const __half*>(p.kcache), rows, p.hd, p.hd, tcd::kKeys);
        if (e == cudaSuccess) e = make_tmap_f16(&tv, static_cast<const __half*>(p.vcache), rows, p.hd, p.hd, tcd::kKeys);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_kv, p.splits);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.kv_f32 ? attn_smem<float>(p.n_heads, p.n_kv, p.hd) : attn_smem<__half>(p.n_heads, p.n_kv, p.hd);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (tc) {
        cfg.dynamicSmemBytes = attn_tc_smem(p.n_heads, p.n_kv, p.hd);
        return cudaLaunchKernelEx(&cfg, pick_tc_kernel(p.hd, p.n_heads / p.n_kv), p, tk, tv);
    }
    return cudaLaunchKernelEx(&cfg, pick_kernel(p.kv_f32, p.hd, p.n_heads / p.n_kv), p);
}

cudaError_t attn_init_device() {
    for (int f32 = 0; f32 < 2; f32++)
        for (int hd : {64, 96, 128})
            for (int G : {1, 2, 4, 8}) {
                cudaError_t e = cudaFuncSetAttribute(pick_kernel(f32, hd, G), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     200 * 1024);
                if (e != cudaSuccess) return e;
            }
    for (int hd : {64, 96, 128})
        for (int G : {1, 2, 4, 8}) {
            cudaError_t e = cudaFuncSetAttribute(pick_tc_kernel(hd, G), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 200 * 1024);
            if (e != cudaSuccess) return e;
        }
    return cudaSuccess;
}

}  // namespace tptc
