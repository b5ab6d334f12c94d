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
// keys of one kv head at consecutive positions are one contiguous run.  Grid = (n_kv,
// splits); each CTA streams its share of positions in 64-position tiles (two threads per
// position for the scores, one output dimension per thread for P.V) through a 2-stage
// shared-memory ring filled by 1-D TMA bulk copies, keeps an online softmax for the group's
// query heads, and writes (m, l, acc) to scratch.  The last CTA of a kv head (atomic
// ticket) merges the splits in split order, so the result does not depend on scheduling;
// the merge stages every split's statistics in shared memory with parallel loads.
#include <algorithm>

#include "kernels.h"

namespace tptc {

namespace {

constexpr int kThreads = 128;
constexpr int kMaxGroup = 8;  // query heads per kv head
constexpr int kStages = 2;

template <typename KV>
struct KvTraits;
template <>
struct KvTraits<__half> {
    static constexpr int kTile = 64;  // positions per tile (64 KB ring: co-resides with a GEMV CTA)
    __device__ static float2 pair(const __half* row, int j) {
        return __half22float2(reinterpret_cast<const __half2*>(row)[j]);
    }
    __device__ static float at(const __half* p) { return __half2float(*p); }
    __device__ static void store(__half* p, float v) { *p = __float2half_rn(v); }
};
template <>
struct KvTraits<float> {
    static constexpr int kTile = 64;
    __device__ static float2 pair(const float* row, int j) { return reinterpret_cast<const float2*>(row)[j]; }
    __device__ static float at(const float* p) { return *p; }
    __device__ static void store(float* p, float v) { *p = v; }
};

template <typename KV>
__global__ void __launch_bounds__(kThreads) attn_decode_kernel(const __grid_constant__ AttnDecodeParams p) {
    using Tr = KvTraits<KV>;
    constexpr int kT = Tr::kTile;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kStages];
    __shared__ float red[kMaxGroup][kThreads / 32];
    __shared__ float mnew_s[kMaxGroup], alpha_s[kMaxGroup];
    __shared__ int is_last;

    const int kvh = blockIdx.x, split = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.n_heads / p.n_kv, hd = p.hd;
    const int tile_elems = kT * hd;
    KV* kbuf = reinterpret_cast<KV*>(smem);                             // [kStages][kT][hd]
    KV* vbuf = kbuf + kStages * tile_elems;                             // [kStages][kT][hd]
    float* qs = reinterpret_cast<float*>(vbuf + kStages * tile_elems);  // [G][hd]
    float* ps = qs + G * hd;                                            // [G][kT]

    if (tid == 0) {
        for (int s = 0; s < kStages; s++) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    pdl_wait();
    pdl_launch_dependents();

    const int kv_len = *p.pos + 1;
    if (kv_len < 1 || kv_len > p.max_seq) {  // position outside the cache: flag it, touch nothing
        if (tid == 0 && kvh == 0 && split == 0 && p.err) atomicExch(p.err, TPTC_ERR_ARG);
        return;
    }
    int per = (kv_len + p.splits - 1) / p.splits;
    per = (per + kT - 1) / kT * kT;
    const int t_begin = split * per, t_end = min(kv_len, t_begin + per);
    const int ntiles = t_end > t_begin ? (t_end - t_begin + kT - 1) / kT : 0;

    // RoPE (candle rope_i: interleaved pairs, x0*c - x1*s, x0*s + x1*c) on the group's
    // queries while they are staged in shared memory
    const int pos = kv_len - 1, half = hd / 2;
    const float* cs = p.rope_cos + (int64_t)pos * half;
    const float* sn = p.rope_sin + (int64_t)pos * half;
    for (int i = tid; i < G * half; i += kThreads) {
        const int g = i / half, j = i % half;
        const float* qg = p.q + (int64_t)(kvh * G + g) * hd;
        const float q0 = qg[2 * j], q1 = qg[2 * j + 1], c = cs[j], s = sn[j];
        const float r0 = __fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, s));
        const float r1 = __fadd_rn(__fmul_rn(q0, s), __fmul_rn(q1, c));
        qs[g * hd + 2 * j] = r0;
        qs[g * hd + 2 * j + 1] = r1;
        if (p.q_out && split == 0) {
            p.q_out[(int64_t)(kvh * G + g) * hd + 2 * j] = r0;
            p.q_out[(int64_t)(kvh * G + g) * hd + 2 * j + 1] = r1;
        }
    }
    // The CTA whose positions include `pos` rotates this step's key and stores it in the cache;
    // the proxy fence orders those generic stores before its own bulk-copy reads of them.
    if (pos >= t_begin && pos < t_end) {
        KV* krow = static_cast<KV*>(p.kcache) + ((int64_t)kvh * p.max_seq + pos) * hd;
        for (int j = tid; j < half; j += kThreads) {
            const float k0 = p.kraw[kvh * hd + 2 * j], k1 = p.kraw[kvh * hd + 2 * j + 1], c = cs[j], s = sn[j];
            Tr::store(krow + 2 * j, __fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, s)));
            Tr::store(krow + 2 * j + 1, __fadd_rn(__fmul_rn(k0, s), __fmul_rn(k1, c)));
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    __syncthreads();

    const KV* kh = static_cast<const KV*>(p.kcache) + (int64_t)kvh * p.max_seq * hd;
    const KV* vh = static_cast<const KV*>(p.vcache) + (int64_t)kvh * p.max_seq * hd;
    uint64_t policy = 0;
    auto issue = [&](int tile) {
        const int s = tile % kStages, t0 = t_begin + tile * kT, n = min(kT, t_end - t0);
        const uint32_t bytes = (uint32_t)n * hd * sizeof(KV);
        mbar_expect_tx(&full[s], 2 * bytes);
        bulk_g2s(kbuf + s * tile_elems, kh + (int64_t)t0 * hd, bytes, &full[s], policy);
        bulk_g2s(vbuf + s * tile_elems, vh + (int64_t)t0 * hd, bytes, &full[s], policy);
    };
    if (tid == 0) {
        policy = l2_evict_first_policy();
        for (int t = 0; t < kStages && t < ntiles; t++) issue(t);
    }

    float m_run[kMaxGroup], l_run[kMaxGroup], acc[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; g++) {
        m_run[g] = -INFINITY;
        l_run[g] = 0.f;
        acc[g] = 0.f;
    }
    // scores: two threads per position (kThreads = 2 * kT), each half of the head dimension
    const int my_pos = tid >> 1, my_half = tid & 1;
    const int hp = hd / 2, hq = hp / 2;  // half2 pairs per row, per half-row
    bool timed_out = false;
    for (int tile = 0; tile < ntiles; tile++) {
        const int s = tile % kStages, t0 = t_begin + tile * kT, n = min(kT, t_end - t0);
        if (!mbar_wait_bounded(&full[s], (tile / kStages) & 1, p.err)) timed_out = true;
        if (__syncthreads_or(timed_out)) return;
        float sc[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) sc[g] = 0.f;
        if (my_pos < n) {
            const KV* krow = kbuf + s * tile_elems + my_pos * hd;
            // start column rotated by position so neighbouring threads hit different banks
            int jj = my_half * hq + (my_pos % hq);
            const int lo = my_half * hq, hi = lo + hq;
            for (int j = 0; j < hq; j++) {
                const float2 kv = Tr::pair(krow, jj);
#pragma unroll
                for (int g = 0; g < kMaxGroup; g++) {
                    if (g < G) {
                        const float2 qv = reinterpret_cast<const float2*>(qs + g * hd)[jj];
                        sc[g] = fmaf(qv.x, kv.x, sc[g]);
                        sc[g] = fmaf(qv.y, kv.y, sc[g]);
                    }
                }
                jj = (jj + 1 == hi) ? lo : jj + 1;
            }
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], 1);
            sc[g] = my_pos < n ? sc[g] * p.scale : -INFINITY;
        }
        // tile max per head
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g < G) {
                const float mx = warp_max(sc[g]);
                if (lane == 0) red[g][warp] = mx;
            }
        }
        __syncthreads();
        if (tid < G) {
            float mx = red[tid][0];
            for (int w = 1; w < kThreads / 32; w++) mx = fmaxf(mx, red[tid][w]);
            const float mn = fmaxf(m_run[tid], mx);
            mnew_s[tid] = mn;
            alpha_s[tid] = m_run[tid] == -INFINITY ? 0.f : expf(m_run[tid] - mn);
        }
        __syncthreads();
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g < G) {
                const float pv = my_pos < n ? expf(sc[g] - mnew_s[g]) : 0.f;
                if (my_half == 0) ps[g * kT + my_pos] = pv;
                const float ls = warp_sum(my_half == 0 ? pv : 0.f);
                if (lane == 0) red[g][warp] = ls;
            }
        }
        __syncthreads();
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g < G) {
                float ls = 0.f;
                for (int w = 0; w < kThreads / 32; w++) ls += red[g][w];
                l_run[g] = l_run[g] * alpha_s[g] + ls;
                m_run[g] = mnew_s[g];
                acc[g] *= alpha_s[g];
            }
        }
        // P.V: thread = output dimension
        if (tid < hd) {
            const KV* vcol = vbuf + s * tile_elems + tid;
            for (int t = 0; t < n; t++) {
                const float v = Tr::at(vcol + t * hd);
#pragma unroll
                for (int g = 0; g < kMaxGroup; g++)
                    if (g < G) acc[g] = fmaf(ps[g * kT + t], v, acc[g]);
            }
        }
        __syncthreads();  // stage s fully consumed
        if (tid == 0 && tile + kStages < ntiles) {
            fence_proxy_async_smem();
            issue(tile + kStages);
        }
    }

    // partial results: [kvh][split][g][2 + hd] = (m, l, acc[hd])
    const int rec = 2 + hd;
    float* part = p.partial + ((int64_t)kvh * p.splits + split) * G * rec;
    if (tid < hd) {
        for (int g = 0; g < G; g++) part[g * rec + 2 + tid] = acc[g];
    }
    if (tid == 0) {
        for (int g = 0; g < G; g++) {
            part[g * rec] = m_run[g];
            part[g * rec + 1] = l_run[g];
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&p.counters[kvh], 1) == p.splits - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // merge: stage every split's (m, l) in shared memory with parallel loads, then each
    // thread reduces one output dimension in split order (deterministic)
    const float* base = p.partial + (int64_t)kvh * p.splits * G * rec;
    float* wgt = ps;             // reuse: [G][splits] m_s, then weights exp(m_s - M); splits <= kT
    float* lsp = qs;             // reuse: [G][splits] l_s (splits <= 64 <= hd)
    float* lsum = mnew_s;        // [G] totals
    for (int i = tid; i < G * p.splits; i += kThreads) {
        const int g = i / p.splits, s = i % p.splits;
        wgt[g * kT + s] = base[(s * G + g) * rec];
        lsp[g * p.splits + s] = base[(s * G + g) * rec + 1];
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int s = 0; s < p.splits; s++) M = fmaxf(M, wgt[tid * kT + s]);
        float L = 0.f;
        for (int s = 0; s < p.splits; s++) {
            const float w = wgt[tid * kT + s] == -INFINITY ? 0.f : expf(wgt[tid * kT + s] - M);
            wgt[tid * kT + s] = w;
            L = fmaf(lsp[tid * p.splits + s], w, L);
        }
        lsum[tid] = L;
    }
    __syncthreads();
    if (tid < hd) {
        for (int g = 0; g < G; g++) {
            float o = 0.f;
            for (int s0 = 0; s0 < p.splits; s0 += 16) {  // 16 independent loads in flight
                float v[16];
#pragma unroll
                for (int k = 0; k < 16; k++)
                    v[k] = s0 + k < p.splits ? base[((s0 + k) * G + g) * rec + 2 + tid] : 0.f;
#pragma unroll
                for (int k = 0; k < 16; k++)
                    if (s0 + k < p.splits) o = fmaf(v[k], wgt[g * kT + s0 + k], o);
            }
            p.out[(kvh * G + g) * hd + tid] = o / lsum[g];
        }
    }
    if (tid == 0) p.counters[kvh] = 0;
}

template <typename KV>
size_t attn_smem(int n_heads, int n_kv, int hd) {
    const int G = n_heads / n_kv, kT = KvTraits<KV>::kTile;
    return (size_t)2 * kStages * kT * hd * sizeof(KV) + (size_t)G * hd * 4 + (size_t)G * kT * 4;
}

}  // namespace

int attn_decode_splits(int n_kv, int max_seq, int sm_count) {
    int s = std::max(1, sm_count / n_kv);
    const int max_useful = (max_seq + 63) / 64;
    // the merge stages one weight per split in a 64-entry shared array
    return std::min(64, std::min(s, std::max(1, max_useful)));
}

size_t attn_decode_partial_floats(int n_heads, int n_kv, int hd, int splits) {
    return (size_t)n_kv * splits * (n_heads / n_kv) * (2 + hd);
}

const char* attn_decode_shape_error(int n_heads, int n_kv, int hd, int max_seq) {
    if (n_heads <= 0 || n_kv <= 0 || hd <= 0 || max_seq <= 0) return "attention: sizes must be positive";
    if (n_heads % n_kv != 0) return "attention: n_heads must be a multiple of n_kv";
    if (n_heads / n_kv > kMaxGroup) return "attention: at most 8 query heads per kv head";
    if (hd > kThreads || hd % 16 != 0) return "attention: head_dim must be a multiple of 16, at most 128";
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

cudaError_t launch_attn_decode(const AttnDecodeParams& p, cudaStream_t st, bool pdl) {
    if (attn_decode_shape_error(p.n_heads, p.n_kv, p.hd, p.max_seq)) return cudaErrorInvalidValue;
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
    if (p.kv_f32) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<float>, p);
    return cudaLaunchKernelEx(&cfg, attn_decode_kernel<__half>, p);
}

cudaError_t attn_init_device() {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
}

}  // namespace tptc
