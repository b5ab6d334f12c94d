// prefill.cu -- prompt processing (prefill).
//
// Two paths behind Engine::prefill (tptc_prefill):
//   * batched: the whole chunk of prompt tokens goes through each layer at once -- weights
//     expanded to dense fp16 per layer, projections on the tcgen05 GEMM (gemm_tc.cu), causal
//     attention over the chunk on the tensor cores (attn_prefill.cu).  This is candle's batched
//     `forward(&input, 0)` (candle_engine.rs:272-281) in the form its CUDA backend takes for
//     batches (dequantise to f16, then a dense matmul), and replaces the reference GPU
//     engine's token-by-token prefill (wgpu_engine.rs:252-261).  Activations enter the GEMMs
//     as fp16 (not Q8_K), so the logits differ from the integer-dot decode path by fp16
//     rounding; the KV cache must be fp16.
//   * per token: each prompt position through the decode step (bit-identical to decoding the
//     prompt; the only path for the f32 KV cache and for prompts below the batched threshold).
#include <algorithm>
#include <vector>

#include "engine.h"
#include "kernels.h"
#include "moe.h"
#include "prefill.h"
#include "quant.cuh"
#include "tp.h"

namespace tptc {

namespace {

#define PF_RET_IF(st)                \
    do {                             \
        Status _s = (st);            \
        if (!_s.ok()) return _s;     \
    } while (0)

// x[t][:] = dequantised row ids[t] of token_embd (device layout); one CTA per token.
__global__ void embed_rows_kernel(DevMatrix emb, const uint32_t* __restrict__ ids, float* __restrict__ x, float scale) {
    const int t = blockIdx.x, row = (int)ids[t], K = emb.K;
    float* xr = x + (size_t)t * K;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float v = dm_elem(emb, row, i);
        xr[i] = scale == 1.f ? v : __fmul_rn(v, scale);
    }
}

// out[t][:] = fp16(x[t] / sqrt(mean(x[t]^2) + eps) * w) (candle rms_norm: x / m * alpha);
// one CTA of 256 threads per token, dim a multiple of 4.
__global__ void __launch_bounds__(256) rmsnorm_f16_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          int dim, float eps, __half* __restrict__ out) {
    __shared__ float red[8];
    const int t = blockIdx.x;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)t * dim);
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) {
        const float4 v = xr[i];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += red[i];
    const float m = sqrtf(tot / (float)dim + eps);
    __half2* o2 = reinterpret_cast<__half2*>(out + (size_t)t * dim);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) {
        const float4 v = xr[i], g = w4[i];
        o2[2 * i] = __floats2half2_rn(__fdiv_rn(v.x, m) * g.x, __fdiv_rn(v.y, m) * g.y);
        o2[2 * i + 1] = __floats2half2_rn(__fdiv_rn(v.z, m) * g.z, __fdiv_rn(v.w, m) * g.w);
    }
}

// The q|k|v GEMM output row of token t -> RoPE (candle rope_i: interleaved pairs) on q and
// k, q as fp16 [T][n_heads][hd], k and v into this layer's fp16 cache at position start + t.
// Same rotation arithmetic as the decode attention kernel.  One CTA per token.
struct QkvPostParams {
    const float* qkv;  // [T][(n_heads + 2 n_kv) hd]
    __half* q;
    __half* kc;
    __half* vc;
    const float* cos;
    const float* sin;
    int start, n_heads, n_kv, hd, max_seq;
    const float* bq;  // optional q / k / v biases (qwen2), added in f32 before RoPE
    const float* bk;
    const float* bv;
    int neox;         // 1: RoPE pairs element j with j + hd/2 (candle rope), 0: 2j with 2j+1 (rope_i)
};
// Per token: the q and k heads rotated pair by pair (q -> fp16 for the attention GEMMs, k ->
// the fp16 cache) and v copied to the cache, each value plus its bias when there is one.
__global__ void qkv_post_kernel(const QkvPostParams p) {
    const int t = blockIdx.x, pos = p.start + t, half = p.hd / 2;
    const int nq = p.n_heads * p.hd, nk = p.n_kv * p.hd, n = nq + 2 * nk;
    const float* row = p.qkv + (size_t)t * n;
    const float* cs = p.cos + (size_t)pos * half;
    const float* sn = p.sin + (size_t)pos * half;
    for (int i = threadIdx.x; i < (p.n_heads + p.n_kv) * half; i += blockDim.x) {
        const int head = i / half, j = i % half;
        const int e0 = p.neox ? j : 2 * j, e1 = p.neox ? j + half : 2 * j + 1;  // within the head
        const int col = head * p.hd;  // the head's first column in [q | k]
        float x0 = row[col + e0], x1 = row[col + e1];
        const float* b = head < p.n_heads ? (p.bq ? p.bq + col : nullptr) : (p.bk ? p.bk + (col - nq) : nullptr);
        if (b) {
            x0 = __fadd_rn(x0, b[e0]);
            x1 = __fadd_rn(x1, b[e1]);
        }
        const float c = cs[j], s = sn[j];
        const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float r1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        if (head < p.n_heads) {
            __half* dq = p.q + (size_t)t * nq + col;
            dq[e0] = __float2half_rn(r0);
            dq[e1] = __float2half_rn(r1);
        } else {
            __half* dk = p.kc + ((size_t)(head - p.n_heads) * p.max_seq + pos) * p.hd;
            dk[e0] = __float2half_rn(r0);
            dk[e1] = __float2half_rn(r1);
        }
    }
    for (int i = threadIdx.x; i < nk; i += blockDim.x) {
        float v = row[nq + nk + i];
        if (p.bv) v = __fadd_rn(v, p.bv[i]);
        const int vh = i / p.hd, e = i % p.hd;
        p.vc[((size_t)vh * p.max_seq + pos) * p.hd + e] = __float2half_rn(v);
    }
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

cudaError_t prefill_init_device() {
    cudaError_t e = gemm_tc_init_device();
    if (e == cudaSuccess) e = gemm_q_init_device();
    if (e != cudaSuccess) return e;
    return attn_prefill_init_device();
}

// Scratch of the batched path for chunks of up to `chunk` tokens (one allocation).
Status Engine::prefill_buffers(int chunk) {
    if (chunk <= pf_chunk_) return {};
    const ModelMeta& m = meta_;
    const int hd = m.head_dim, ffn_l = m.ffn / tp_size_;
    const size_t nq = (size_t)n_heads_l_ * hd, nqkv = nq + 2 * (size_t)n_kv_l_ * hd;
    const size_t T = (size_t)chunk;
    const size_t eff = (size_t)m.expert_ffn, sffn = (size_t)m.shared_ffn, TK = T * (size_t)m.n_expert_used;
    const size_t w_elems = std::max({nqkv * m.dim, (size_t)2 * ffn_l * m.dim, (size_t)m.dim * ffn_l,
                                     (size_t)m.dim * nq, 2 * eff * m.dim, 2 * sffn * m.dim});
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off = align256(off + bytes);
        return o;
    };
    const size_t o_ids = take(T * 4), o_x = take(T * m.dim * 4), o_xn = take(T * m.dim * 2);
    const size_t o_qkv = take(T * nqkv * 4), o_q = take(T * nq * 2), o_o = take(T * nq * 2);
    const size_t o_h = take(T * ffn_l * 2), o_w = take(w_elems * 2);
    // row-parallel partial sums under tensor parallelism (the decode step's own partial
    // buffer is baked into its graph and is not resized here)
    const size_t o_part = tp_ ? take(T * m.dim * 4) : 0;
    const bool moe = m.n_expert > 0;
    const size_t o_rsel = moe ? take(TK * 4) : 0, o_rw = moe ? take(TK * 4) : 0;
    const size_t o_gidx = moe ? take(TK * 4) : 0, o_rowof = moe ? take(TK * 4) : 0;
    const size_t o_ga = moe ? take(TK * m.dim * 2) : 0, o_gh = moe ? take(TK * eff * 2) : 0;
    const size_t o_gy = moe ? take(TK * m.dim * 4) : 0;
    const size_t o_shh = sffn ? take(T * sffn * 2) : 0, o_shy = sffn ? take(T * m.dim * 4) : 0;
    if (pf_) {
        TPTC_CUDA_RET(cudaStreamSynchronize(stream_));
        cudaFree(pf_);
    }
    pf_ = nullptr;
    pf_size_ = 0;
    pf_chunk_ = 0;
    cudaError_t ce = cudaMalloc(&pf_, off);
    if (ce != cudaSuccess) {
        pf_ = nullptr;
        return Status{TPTC_ERR_OOM, "prefill buffers for " + std::to_string(chunk) + " tokens need " +
                                        std::to_string(off >> 20) + " MiB: " + cuda_msg(ce, "cudaMalloc")};
    }
    pf_size_ = off;
    pf_chunk_ = chunk;
    pf_ids_ = reinterpret_cast<uint32_t*>(pf_ + o_ids);
    pf_x_ = reinterpret_cast<float*>(pf_ + o_x);
    pf_xn_ = reinterpret_cast<__half*>(pf_ + o_xn);
    pf_qkv_ = reinterpret_cast<float*>(pf_ + o_qkv);
    pf_q_ = reinterpret_cast<__half*>(pf_ + o_q);
    pf_o_ = reinterpret_cast<__half*>(pf_ + o_o);
    pf_h_ = reinterpret_cast<__half*>(pf_ + o_h);
    pf_w_ = reinterpret_cast<__half*>(pf_ + o_w);
    pf_part_ = tp_ ? reinterpret_cast<float*>(pf_ + o_part) : nullptr;
    pf_rsel_ = moe ? reinterpret_cast<int*>(pf_ + o_rsel) : nullptr;
    pf_rw_ = moe ? reinterpret_cast<float*>(pf_ + o_rw) : nullptr;
    pf_gidx_ = moe ? reinterpret_cast<int*>(pf_ + o_gidx) : nullptr;
    pf_rowof_ = moe ? reinterpret_cast<int*>(pf_ + o_rowof) : nullptr;
    pf_ga_ = moe ? reinterpret_cast<__half*>(pf_ + o_ga) : nullptr;
    pf_gh_ = moe ? reinterpret_cast<__half*>(pf_ + o_gh) : nullptr;
    pf_gy_ = moe ? reinterpret_cast<float*>(pf_ + o_gy) : nullptr;
    pf_sh_h_ = sffn ? reinterpret_cast<__half*>(pf_ + o_shh) : nullptr;
    pf_sh_y_ = sffn ? reinterpret_cast<float*>(pf_ + o_shy) : nullptr;
    return {};
}

// One chunk of T prompt tokens at positions start .. start + T - 1 (ids already in pf_ids_).
Status Engine::enqueue_prefill_chunk(int T, int start) {
    const ModelMeta& m = meta_;
    const int hd = m.head_dim, dim = m.dim, ffn_l = m.ffn / tp_size_;
    const int nq = n_heads_l_ * hd, nk = n_kv_l_ * hd, nqkv = nq + 2 * nk;
    const size_t layer_kv = (size_t)2 * n_kv_l_ * max_seq_ * hd * 2;  // bytes (fp16 cache)
    cudaStream_t st = stream_;
    // A quantised weight is contracted by the fused-dequant GEMM (its blocks expanded in shared
    // memory) where the wave model expects that to be faster (TPTC_FUSED_AUTO) or always
    // (TPTC_FUSED_ALWAYS); otherwise it is expanded to fp16 in pf_w_ first (one pass over the
    // matrix) and contracted by gemm_tc.  A gate|up matrix is used in its physical row order
    // (4 gate rows, then the 4 matching up rows), which the GLU epilogue expects.
    auto fused = [&](const DevMatrix& w, int M) {
        if (prefill_fused_ == TPTC_FUSED_NEVER || !gemm_q_supported(w)) return false;
        return prefill_fused_ == TPTC_FUSED_ALWAYS || gemm_q_preferred(w, M, w.N, sm_count_);
    };
    auto matmul = [&](int epi, const __half* a, const DevMatrix& w, const GemmTcParams& g) -> cudaError_t {
        if (fused(w, g.M)) return gemm_q(epi, a, g.K, w, g, st, false);
        cudaError_t e = launch_dequant_rows_f16(w, 0, g.N, pf_w_, st, w.glu != 0);
        return e != cudaSuccess ? e : gemm_tc(epi, a, g.K, pf_w_, g.K, g, st, false);
    };
    embed_rows_kernel<<<T, 256, 0, st>>>(embd_, pf_ids_, pf_x_, m.embd_scale);
    TPTC_CUDA_RET(cudaGetLastError());
    for (int l = 0; l < m.n_layers; l++) {
        const LayerWeights& L = layers_[l];
        __half* kc = reinterpret_cast<__half*>(kv_ + l * layer_kv);
        __half* vc = reinterpret_cast<__half*>(kv_ + l * layer_kv + layer_kv / 2);
        // attention block
        rmsnorm_f16_kernel<<<T, 256, 0, st>>>(pf_x_, L.attn_norm, dim, m.rms_eps, pf_xn_);
        TPTC_CUDA_RET(cudaGetLastError());
        GemmTcParams g = {};
        g.M = T;
        g.N = nqkv;
        g.K = dim;
        g.c = pf_qkv_;
        g.ldc = nqkv;
        g.err = err_;
        if (fused(L.q, T) && fused(L.k, T) && fused(L.v, T)) {  // three GEMMs into the column ranges
            GemmTcParams gq = g;
            gq.N = nq;
            TPTC_CUDA_RET(gemm_q(GEMM_STORE, pf_xn_, dim, L.q, gq, st, false));
            gq.N = nk;
            gq.c = pf_qkv_ + nq;
            TPTC_CUDA_RET(gemm_q(GEMM_STORE, pf_xn_, dim, L.k, gq, st, false));
            gq.c = pf_qkv_ + nq + nk;
            TPTC_CUDA_RET(gemm_q(GEMM_STORE, pf_xn_, dim, L.v, gq, st, false));
        } else {
            TPTC_CUDA_RET(launch_dequant_rows_f16(L.q, 0, nq, pf_w_, st));
            TPTC_CUDA_RET(launch_dequant_rows_f16(L.k, 0, nk, pf_w_ + (size_t)nq * dim, st));
            TPTC_CUDA_RET(launch_dequant_rows_f16(L.v, 0, nk, pf_w_ + (size_t)(nq + nk) * dim, st));
            TPTC_CUDA_RET(gemm_tc(GEMM_STORE, pf_xn_, dim, pf_w_, dim, g, st, false));
        }
        QkvPostParams qp = {pf_qkv_, pf_q_, kc, vc, rope_cos_, rope_sin_, start, n_heads_l_, n_kv_l_, hd, max_seq_,
                            L.bq, L.bk, L.bv, meta_.rope_neox ? 1 : 0};
        qkv_post_kernel<<<T, 256, 0, st>>>(qp);
        TPTC_CUDA_RET(cudaGetLastError());
        AttnPrefillParams ap = {};
        ap.q = pf_q_;
        ap.kcache = kc;
        ap.vcache = vc;
        ap.out = pf_o_;
        ap.T = T;
        ap.start = start;
        ap.n_heads = n_heads_l_;
        ap.n_kv = n_kv_l_;
        ap.hd = hd;
        ap.max_seq = max_seq_;
        ap.scale = (float)(1.0 / sqrt((double)hd));
        ap.err = err_;
        TPTC_CUDA_RET(launch_attn_prefill(ap, st, false));
        g.N = dim;
        g.K = nq;
        g.ldc = dim;
        if (tp_) {  // row-parallel o: partial sums of every token, then one allreduce
            g.c = pf_part_;
            TPTC_CUDA_RET(matmul(GEMM_STORE, pf_o_, L.o, g));
            PF_RET_IF(tp_->allreduce_add(g.c, pf_x_, (size_t)T * dim, st));
        } else {
            g.c = pf_x_;
            TPTC_CUDA_RET(matmul(GEMM_RESID, pf_o_, L.o, g));
        }
        // feed-forward block: gate|up in the device tile order, silu(gate) * up in the epilogue
        rmsnorm_f16_kernel<<<T, 256, 0, st>>>(pf_x_, L.ffn_norm, dim, m.rms_eps, pf_xn_);
        TPTC_CUDA_RET(cudaGetLastError());
        if (L.moe) {
            // Mixture of experts: every token routed on the device (the decode path's routing);
            // the choices come to the host once per layer to group the chosen (token, expert)
            // rows by expert; each expert's rows then go through the same GEMMs as a dense
            // layer, and the combine kernel adds the outputs back in candle's order.
            const int E = m.n_expert, K = m.n_expert_used, eff = m.expert_ffn, TK = T * K;
            MoeRouteParams r = {};
            r.x = pf_x_;
            r.norm_w = L.ffn_norm;
            r.eps = m.rms_eps;
            r.router = L.router;
            r.router_f16 = L.router_type == TPTC_TYPE_F16 ? 1 : 0;
            r.dim = dim;
            r.n_expert = E;
            r.n_used = K;
            r.sel = pf_rsel_;
            r.w = pf_rw_;
            TPTC_CUDA_RET(launch_moe_route_rows(r, T, st));
            std::vector<int> sel((size_t)TK), cnt(E, 0), off(E + 1, 0), gidx((size_t)TK), rowof((size_t)TK);
            TPTC_CUDA_RET(cudaMemcpyAsync(sel.data(), pf_rsel_, (size_t)TK * 4, cudaMemcpyDeviceToHost, st));
            TPTC_CUDA_RET(cudaStreamSynchronize(st));
            for (int i = 0; i < TK; i++) {
                if (sel[i] < 0 || sel[i] >= E) return Status{TPTC_ERR_CUDA, "expert routing out of range"};
                cnt[sel[i]]++;
            }
            for (int e = 0; e < E; e++) off[e + 1] = off[e] + cnt[e];
            std::vector<int> fill(off.begin(), off.end() - 1);
            for (int t = 0; t < T; t++)
                for (int k = 0; k < K; k++) {
                    const int row = fill[sel[(size_t)t * K + k]]++;
                    gidx[row] = t;
                    rowof[(size_t)t * K + k] = row;
                }
            TPTC_CUDA_RET(cudaMemcpyAsync(pf_gidx_, gidx.data(), (size_t)TK * 4, cudaMemcpyHostToDevice, st));
            TPTC_CUDA_RET(cudaMemcpyAsync(pf_rowof_, rowof.data(), (size_t)TK * 4, cudaMemcpyHostToDevice, st));
            TPTC_CUDA_RET(launch_gather_rows_f16(pf_xn_, pf_gidx_, TK, dim, pf_ga_, st));
            for (int e = 0; e < E; e++) {
                if (!cnt[e]) continue;
                DevMatrix wg = L.eglu, wd = L.edown;
                wg.main += (int64_t)e * L.eglu_stride;
                wd.main += (int64_t)e * L.edown_stride;
                GemmTcParams ge = {};
                ge.M = cnt[e];
                ge.N = 2 * eff;
                ge.K = dim;
                ge.h = pf_gh_ + (size_t)off[e] * eff;
                ge.ldh = eff;
                ge.err = err_;
                ge.geglu = m.geglu ? 1 : 0;
                TPTC_CUDA_RET(matmul(GEMM_GLU, pf_ga_ + (size_t)off[e] * dim, wg, ge));
                GemmTcParams gd = {};
                gd.M = cnt[e];
                gd.N = dim;
                gd.K = eff;
                gd.c = pf_gy_ + (size_t)off[e] * dim;
                gd.ldc = dim;
                gd.err = err_;
                TPTC_CUDA_RET(matmul(GEMM_STORE, pf_gh_ + (size_t)off[e] * eff, wd, gd));
            }
            if (L.shexp) {  // the shared expert on every token
                const int sffn = m.shared_ffn;
                GemmTcParams gs = {};
                gs.M = T;
                gs.N = 2 * sffn;
                gs.K = dim;
                gs.h = pf_sh_h_;
                gs.ldh = sffn;
                gs.err = err_;
                gs.geglu = m.geglu ? 1 : 0;
                TPTC_CUDA_RET(matmul(GEMM_GLU, pf_xn_, L.glu, gs));
                GemmTcParams gd = {};
                gd.M = T;
                gd.N = dim;
                gd.K = sffn;
                gd.c = pf_sh_y_;
                gd.ldc = dim;
                gd.err = err_;
                TPTC_CUDA_RET(matmul(GEMM_STORE, pf_sh_h_, L.down, gd));
            }
            TPTC_CUDA_RET(launch_moe_combine_rows(pf_x_, pf_gy_, pf_rowof_, pf_rw_, K, L.shexp ? pf_sh_y_ : nullptr,
                                                  T, dim, st));
            continue;
        }
        GemmTcParams gg = {};
        gg.M = T;
        gg.N = 2 * ffn_l;
        gg.K = dim;
        gg.h = pf_h_;
        gg.ldh = ffn_l;
        gg.err = err_;
        gg.geglu = m.geglu ? 1 : 0;
        TPTC_CUDA_RET(matmul(GEMM_GLU, pf_xn_, L.glu, gg));
        g.N = dim;
        g.K = ffn_l;
        g.ldc = dim;
        if (tp_) {
            g.c = pf_part_;
            TPTC_CUDA_RET(matmul(GEMM_STORE, pf_h_, L.down, g));
            PF_RET_IF(tp_->allreduce_add(g.c, pf_x_, (size_t)T * dim, st));
        } else {
            g.c = pf_x_;
            TPTC_CUDA_RET(matmul(GEMM_RESID, pf_h_, L.down, g));
        }
    }
    return {};
}

bool Engine::prefill_uses_gemm(int n) const {
    if (kv_f32_ || prefill_gemm_min_ <= 0 || n < prefill_gemm_min_) return false;
    const ModelMeta& m = meta_;
    const int ffn_l = m.ffn / tp_size_;
    // GEMM operands: K a multiple of 64, the gate|up tile order whole 8-row groups
    return m.dim % 64 == 0 && (n_heads_l_ * m.head_dim) % 64 == 0 && ffn_l % 64 == 0 &&
           (m.head_dim == 64 || m.head_dim == 96 || m.head_dim == 128);
}

Status Engine::run_prefill_batched(const uint32_t* ids, int n, int start_pos, float* last_logits) {
    if (!prefill_uses_gemm(n)) {
        // Prompt positions one at a time through the decode graph (the reference's prefill
        // loop, wgpu_engine.rs:254-261); the last step's logits are returned.
        for (int i = 0; i < n; i++) {
            uint32_t am;
            Status s = decode(ids[i], start_pos + i, i + 1 == n ? last_logits : nullptr, &am);
            if (!s.ok()) return s;
        }
        return {};
    }
    const int chunk = std::min(n, kPrefillChunk);
    PF_RET_IF(prefill_buffers(chunk));
    const ModelMeta& m = meta_;
    for (int c0 = 0; c0 < n; c0 += chunk) {
        const int T = std::min(chunk, n - c0);
        TPTC_CUDA_RET(cudaMemcpyAsync(pf_ids_, ids + c0, (size_t)T * 4, cudaMemcpyHostToDevice, stream_));
        PF_RET_IF(enqueue_prefill_chunk(T, start_pos + c0));
        if (c0 + T == n) {
            // the last token's row -> final norm + lm_head (the decode GEMV)
            TPTC_CUDA_RET(cudaMemcpyAsync(x_, pf_x_ + (size_t)(T - 1) * m.dim, (size_t)m.dim * 4,
                                          cudaMemcpyDeviceToDevice, stream_));
            GemvParams h = {};
            h.K = m.dim;
            h.err = err_;
            h.act_global = act_;
            h.eps = m.rms_eps;
            h.nseg = 1;
            h.seg[0] = GemvSeg{output_, 0};
            h.x = x_;
            h.norm_w = out_norm_;
            h.out = logits_ + head_row0_;
            gemv_prepare(h, sm_count_);
            TPTC_CUDA_RET(gemv_launch(h, EPI_STORE, stream_, false));
            if (last_logits) {
                PF_RET_IF(gather_logits());
                TPTC_CUDA_RET(cudaMemcpyAsync(last_logits, logits_, (size_t)m.vocab * 4, cudaMemcpyDeviceToHost,
                                              stream_));
            }
        }
        // the ids buffer is reused by the next chunk: wait for this one
        PF_RET_IF(sync());
        cached_tokens_.insert(cached_tokens_.end(), ids + c0, ids + c0 + T);
    }
    return {};
}

}  // namespace tptc
