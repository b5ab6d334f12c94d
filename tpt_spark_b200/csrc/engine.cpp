// engine.cpp -- model load, KV cache, CUDA-graph decode step, prefill and the infer loop.
#include "engine.h"

#include <math.h>
#include <string.h>

#include <algorithm>
#include <chrono>

#include "kernels.h"
#include "moe.h"
#include "prefill.h"
#include "tp.h"

namespace tptc {

std::string cuda_msg(cudaError_t e, const char* what) {
    return std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
}

namespace {

Status err(int code, const std::string& m) { return Status{code, m}; }

#define RET_IF(st)            \
    do {                      \
        Status _s = (st);     \
        if (!_s.ok()) return _s; \
    } while (0)

#define CU(call)                                                                      \
    do {                                                                              \
        cudaError_t _e = (call);                                                      \
        if (_e != cudaSuccess) return Status{TPTC_ERR_CUDA, cuda_msg(_e, #call)};     \
    } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int64_t raw_row_bytes(int type, int K) {
    switch (type) {
    case TPTC_TYPE_Q4_K: return (int64_t)K / QK_K * Q4K_BYTES;
    case TPTC_TYPE_Q6_K: return (int64_t)K / QK_K * Q6K_BYTES;
    case TPTC_TYPE_Q8_0: return (int64_t)K / QK8_0 * Q80_BYTES;
    case TPTC_TYPE_Q5_K: return (int64_t)K / QK_K * Q5K_BYTES;
    case TPTC_TYPE_Q2_K: return (int64_t)K / QK_K * Q2K_BYTES;
    case TPTC_TYPE_Q3_K: return (int64_t)K / QK_K * Q3K_BYTES;
    case TPTC_TYPE_Q4_0: return (int64_t)K / QK8_0 * Q40_BYTES;
    case TPTC_TYPE_Q5_0: return (int64_t)K / QK8_0 * Q50_BYTES;
    case TPTC_TYPE_Q4_1: return (int64_t)K / QK8_0 * Q41_BYTES;
    case TPTC_TYPE_Q5_1: return (int64_t)K / QK8_0 * Q51_BYTES;
    case TPTC_TYPE_F16: return (int64_t)K * 2;
    case TPTC_TYPE_F32: return (int64_t)K * 4;
    }
    return 0;
}

bool matrix_type_ok(int t) {
    return t == TPTC_TYPE_Q2_K || t == TPTC_TYPE_Q3_K || t == TPTC_TYPE_Q4_K || t == TPTC_TYPE_Q5_K ||
           t == TPTC_TYPE_Q6_K || t == TPTC_TYPE_Q4_0 || t == TPTC_TYPE_Q5_0 || t == TPTC_TYPE_Q4_1 ||
           t == TPTC_TYPE_Q5_1 || t == TPTC_TYPE_Q8_0 || t == TPTC_TYPE_F16;
}

// Streams host bytes into device memory through two pinned buffers (the reference uploads
// with wgpu create_buffer_init, wgpu_loader.rs:175; here: mmap -> pinned -> cudaMemcpyAsync).
struct Stager {
    static constexpr size_t kChunk = 64ull << 20;
    uint8_t* pinned[2] = {nullptr, nullptr};
    uint8_t* dtmp[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int cur = 0;
    cudaStream_t st;

    explicit Stager(cudaStream_t s) : st(s) {}
    ~Stager() {
        for (int i = 0; i < 2; i++) {
            if (ev[i]) {
                cudaEventSynchronize(ev[i]);
                cudaEventDestroy(ev[i]);
            }
            if (pinned[i]) cudaFreeHost(pinned[i]);
            if (dtmp[i]) cudaFree(dtmp[i]);
        }
    }
    Status init() {
        for (int i = 0; i < 2; i++) {
            CU(cudaHostAlloc(&pinned[i], kChunk, cudaHostAllocDefault));
            CU(cudaMalloc(&dtmp[i], kChunk));
            CU(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
            CU(cudaEventRecord(ev[i], st));
        }
        return {};
    }
    // Next free buffer index (waits for its previous transfer).
    Status acquire(int& i) {
        i = cur;
        cur ^= 1;
        CU(cudaEventSynchronize(ev[i]));
        return {};
    }
    Status release(int i) {
        CU(cudaEventRecord(ev[i], st));
        return {};
    }
};

// Copy rows [r0, r1) x raw-bytes [c0, c1) of a row-major host tensor into device memory,
// repacking into the tiled layout as logical rows first_row.. of `m`.  Used whole (c0 = 0,
// c1 = row bytes) on one GPU; the column window selects a K-slice for row-parallel tensor
// sharding.  m.type == F32 (norm vectors) is copied as is.
Status upload_rows(Stager& sg, const uint8_t* host, int64_t host_row_bytes, int r0, int r1, int64_t c0, int64_t c1,
                   const DevMatrix& m, int first_row) {
    const int64_t rb = c1 - c0;
    int rows_per = (int)std::max<int64_t>(1, (int64_t)Stager::kChunk / rb);
    for (int r = r0; r < r1; r += rows_per) {
        const int nr = std::min(rows_per, r1 - r);
        int b;
        RET_IF(sg.acquire(b));
        if (c0 == 0 && rb == host_row_bytes) {
            memcpy(sg.pinned[b], host + (int64_t)r * host_row_bytes, (size_t)nr * rb);
        } else {
            for (int i = 0; i < nr; i++)
                memcpy(sg.pinned[b] + (int64_t)i * rb, host + (int64_t)(r + i) * host_row_bytes + c0, (size_t)rb);
        }
        if (m.type == TPTC_TYPE_F32) {
            CU(cudaMemcpyAsync(m.main + (int64_t)(r - r0) * rb, sg.pinned[b], (size_t)nr * rb, cudaMemcpyHostToDevice,
                               sg.st));
        } else {
            CU(cudaMemcpyAsync(sg.dtmp[b], sg.pinned[b], (size_t)nr * rb, cudaMemcpyHostToDevice, sg.st));
            CU(launch_repack(sg.dtmp[b], rb, nr, first_row + (r - r0), m, sg.st));
        }
        RET_IF(sg.release(b));
    }
    return {};
}

}  // namespace

// ------------------------------------------------------------------------------------------

Engine::Engine(int device, int tp_rank, int tp_size) : device_(device), tp_rank_(tp_rank), tp_size_(tp_size) {}

Engine::~Engine() {
    unload();
    if (stream_) {
        cudaSetDevice(device_);
        cudaStreamDestroy(stream_);
    }
    if (ev0_) cudaEventDestroy(ev0_);
    if (ev1_) cudaEventDestroy(ev1_);
    if (h_tok_) cudaFreeHost(h_tok_);
    if (h_pos_) cudaFreeHost(h_pos_);
    if (h_err_) cudaFreeHost(h_err_);
}

Status Engine::init(const void* nccl_uid) {
    int n = 0;
    CU(cudaGetDeviceCount(&n));
    if (device_ < 0 || device_ >= n) return err(TPTC_ERR_ARG, "device " + std::to_string(device_) + " not present");
    if (tp_size_ < 1 || tp_rank_ < 0 || tp_rank_ >= tp_size_) return err(TPTC_ERR_ARG, "bad tp rank/size");
    CU(cudaSetDevice(device_));
    cudaDeviceProp prop;
    CU(cudaGetDeviceProperties(&prop, device_));
    if (prop.major < 10) return err(TPTC_ERR_UNSUPPORTED, std::string("libtptc needs sm_100 (B200); found ") + prop.name);
    sm_count_ = prop.multiProcessorCount;
    CU(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    CU(cudaEventCreate(&ev0_));
    CU(cudaEventCreate(&ev1_));
    CU(kernels_init_device());
    CU(cudaHostAlloc(&h_tok_, 64 * sizeof(uint32_t), cudaHostAllocDefault));
    CU(cudaHostAlloc(&h_pos_, 64 * sizeof(int), cudaHostAllocDefault));
    CU(cudaHostAlloc(&h_err_, 64 * sizeof(int), cudaHostAllocDefault));
    const char* e = getenv("TPTC_PDL");
    pdl_ = !(e && e[0] == '0');
    const char* ch = getenv("TPTC_DECODE_CHAIN");
    chain_ = ch && ch[0] == '1';
    if (tp_size_ > 1) {
        tp_.reset(new Tp());
        RET_IF(tp_->init(tp_rank_, tp_size_, nccl_uid, stream_));
    }
    return {};
}

void Engine::unload() {
    if (device_ >= 0) cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    if (graph_plain_) cudaGraphExecDestroy(graph_plain_);
    if (graph_chained_) cudaGraphExecDestroy(graph_chained_);
    graph_plain_ = graph_chained_ = nullptr;
    if (arena_) cudaFree(arena_);
    if (rt_) cudaFree(rt_);
    if (pf_) cudaFree(pf_);
    arena_ = rt_ = pf_ = nullptr;
    arena_size_ = rt_size_ = pf_size_ = 0;
    pf_chunk_ = 0;
    layers_.clear();
    cached_tokens_.clear();
    loaded_ = false;
    device_bytes_ = 0;
}

Status Engine::load(const std::string& path, tptc_progress_cb cb, void* user) {
    if (!stream_) return err(TPTC_ERR_STATE, "context not initialised");
    CU(cudaSetDevice(device_));
    unload();
    GgufFile f;
    std::string emsg;
    int rc = f.open(path, emsg);
    if (rc != TPTC_OK) return err(rc, emsg);

    // ---- metadata (wgpu_loader.rs:305-406; candle_engine.rs:145-165 arch check).  qwen2 is
    // llama's forward with q / k / v biases and RoPE on head halves (candle quantized_qwen2;
    // the reference runs it on its wgpu path, wgpu_loader.rs:270, bias_add.wgsl).
    // phi3 (candle quantized_phi3): one fused attn_qkv tensor (rows q | k | v, the reference's
    // wgpu_engine.rs:385-397) and one fused ffn_up tensor (rows gate | up), RoPE on head halves.
    // gemma (the reference's arch table gives it GEGLU and a tied lm_head, wgpu_loader.rs:220,270)
    // follows its model definition: GEGLU with the tanh gelu, embeddings scaled by sqrt(dim),
    // RoPE on head halves; its GGUF norm gains already carry the +1.  gemma2 / gemma3 add
    // post-norms and logit soft-capping, which this forward pass does not have.
    ModelMeta m;
    f.get_str("general.architecture", m.architecture);
    if (m.architecture != "llama" && m.architecture != "mistral" && m.architecture != "qwen2" &&
        m.architecture != "phi3" && m.architecture != "gemma")
        return err(TPTC_ERR_UNSUPPORTED, "Architecture '" + m.architecture +
                                             "' is not yet supported. Supported: llama, mistral, qwen2, phi3, gemma.");
    m.rope_neox = m.architecture == "qwen2" || m.architecture == "phi3" || m.architecture == "gemma";
    m.geglu = m.architecture == "gemma";
    f.get_str("general.name", m.name);
    const std::string a = m.architecture;
    uint64_t u;
    auto getu = [&](const std::string& k, int def) { return f.get_u64(a + "." + k, u) ? (int)u : def; };
    m.context_length = getu("context_length", 4096);
    m.n_layers = getu("block_count", 32);
    m.n_heads = getu("attention.head_count", 32);
    m.n_kv_heads = getu("attention.head_count_kv", m.n_heads);
    m.dim = getu("embedding_length", 4096);
    const GgufTensor* te = f.find("token_embd.weight");
    if (!te || te->ne.size() != 2) return err(TPTC_ERR_FORMAT, "missing or malformed token_embd.weight");
    m.vocab = getu("vocab_size", (int)te->ne[1]);
    float fv;
    if (f.get_f32(a + ".rope.freq_base", fv)) m.rope_freq_base = fv;
    if (f.get_f32(a + ".attention.layer_norm_rms_epsilon", fv)) m.rms_eps = fv;
    {
        std::string st;
        float factor = 1.f;
        f.get_str(a + ".rope.scaling.type", st);
        f.get_f32(a + ".rope.scaling.factor", factor);
        if (st == "linear" || st == "longrope") m.rope_scale = std::max(1.f, factor);
    }
    if (m.n_heads <= 0 || m.dim % m.n_heads) return err(TPTC_ERR_FORMAT, "embedding_length not divisible by head_count");
    m.head_dim = m.dim / m.n_heads;
    {
        int est = (m.dim * 8 + 2) / 3;
        est = (est + 255) / 256 * 256;
        m.ffn = getu("feed_forward_length", est);
    }
    if (m.n_kv_heads <= 0 || m.n_heads % m.n_kv_heads) return err(TPTC_ERR_UNSUPPORTED, "head_count not a multiple of head_count_kv");
    if (m.head_dim != 64 && m.head_dim != 96 && m.head_dim != 128)
        return err(TPTC_ERR_UNSUPPORTED, "head_dim must be 64, 96 or 128");
    if (m.dim % QK_K || m.ffn % QK_K) return err(TPTC_ERR_UNSUPPORTED, "embedding/ffn sizes must be multiples of 256");
    if (m.geglu) m.embd_scale = sqrtf((float)m.dim);
    // mixture of experts (wgpu_loader.rs:367-377: expert_used_count defaults to 2 when absent)
    m.n_expert = getu("expert_count", 0);
    if (m.n_expert > 1) {
        m.n_expert_used = getu("expert_used_count", 2);
        m.expert_ffn = getu("expert_feed_forward_length", m.ffn);
        if (m.n_expert > kMoeMaxExperts || m.n_expert_used < 1 || m.n_expert_used > kMoeMaxUsed ||
            m.n_expert_used > m.n_expert)
            return err(TPTC_ERR_UNSUPPORTED, "expert_count / expert_used_count out of range (at most " +
                                                 std::to_string(kMoeMaxExperts) + " experts, " +
                                                 std::to_string(kMoeMaxUsed) + " chosen per token)");
        if (m.expert_ffn % QK_K || m.dim > kMoeMaxDim)
            return err(TPTC_ERR_UNSUPPORTED, "expert feed-forward size must be a multiple of 256");
        if (tp_size_ > 1) return err(TPTC_ERR_UNSUPPORTED, "mixture-of-experts models run on one GPU (tp_size 1)");
    } else {
        m.n_expert = 0;
    }
    int sh[7][4];
    for (int w = 0; w < 7; w++)
        if (!tp_shard(w, m.n_heads, m.n_kv_heads, m.head_dim, m.dim, m.ffn, tp_rank_, tp_size_, sh[w][0], sh[w][1],
                      sh[w][2], sh[w][3]))
            return err(TPTC_ERR_UNSUPPORTED, "model does not shard evenly over tp_size=" + std::to_string(tp_size_));
    m.tied = f.find("output.weight") == nullptr;
    m.qkv_bias = f.find("blk.0.attn_q.bias") != nullptr;
    m.fused_qkv = f.find("blk.0.attn_qkv.weight") != nullptr;
    m.fused_gate_up = f.find("blk.0.ffn_gate.weight") == nullptr && f.find("blk.0.ffn_up.weight") != nullptr;
    meta_ = m;
    path_ = path;
    file_bytes_ = f.size;

    n_heads_l_ = m.n_heads / tp_size_;
    n_kv_l_ = m.n_kv_heads / tp_size_;
    const int hd = m.head_dim, ffn_l = m.ffn / tp_size_;

    // ---- tensor plan: name, expected shape, rows/cols this rank keeps, destination.
    // gate and up land in one fused gate|up matrix (logical rows [0, ffn_l) and [ffn_l,
    // 2 ffn_l)), so the decode GEMV streams matching gate and up rows as one tile.
    struct Plan {
        std::string name;
        int N, K;            // full shape
        int r0, r1;          // rows kept (column parallel)
        int k0, k1;          // K range kept (row parallel)
        DevMatrix* mat;      // nullptr for f32 vectors
        float** vec;
        int first_row;       // logical row of r0 in `mat`
        int glu_rows;        // > 0: `mat` is a fused gate|up matrix of this many rows
        int expert = -1;     // >= 0: this expert's [N x K] slice of a stacked [n_stack][N][K] tensor
        int n_stack = 0;
        const void** raw = nullptr;  // F32 / F16 rows copied as they are (the MoE router)
        int* raw_type = nullptr;
    };
    std::vector<Plan> plans;
    layers_.assign(m.n_layers, LayerWeights{});
    plans.push_back({"token_embd.weight", m.vocab, m.dim, 0, m.vocab, 0, m.dim, &embd_, nullptr, 0, 0});
    for (int l = 0; l < m.n_layers; l++) {
        LayerWeights& L = layers_[l];
        const std::string p = "blk." + std::to_string(l) + ".";
        plans.push_back({p + "attn_norm.weight", 1, m.dim, 0, 1, 0, m.dim, nullptr, &L.attn_norm, 0, 0});
        // rows / K windows from tp_shard (the same plan tptc_tp_shard exposes); a fused tensor
        // (phi3 attn_qkv, ffn_up) is read as its row blocks, `row_off` rows into it
        auto W = [&](int w, const char* name, int N, int K, DevMatrix* mat, int first_row, int glu_rows,
                     int row_off = 0, int fused_rows = 0) {
            plans.push_back({p + name, fused_rows ? fused_rows : N, K, row_off + sh[w][0], row_off + sh[w][1], sh[w][2],
                             sh[w][3], mat, nullptr, first_row, glu_rows});
        };
        const int nq = m.n_heads * hd, nkv = m.n_kv_heads * hd;
        if (m.fused_qkv) {
            W(TPTC_SHARD_Q, "attn_qkv.weight", nq, m.dim, &L.q, 0, 0, 0, nq + 2 * nkv);
            W(TPTC_SHARD_K, "attn_qkv.weight", nkv, m.dim, &L.k, 0, 0, nq, nq + 2 * nkv);
            W(TPTC_SHARD_V, "attn_qkv.weight", nkv, m.dim, &L.v, 0, 0, nq + nkv, nq + 2 * nkv);
        } else {
            W(TPTC_SHARD_Q, "attn_q.weight", nq, m.dim, &L.q, 0, 0);
            W(TPTC_SHARD_K, "attn_k.weight", nkv, m.dim, &L.k, 0, 0);
            W(TPTC_SHARD_V, "attn_v.weight", nkv, m.dim, &L.v, 0, 0);
        }
        if (m.qkv_bias) {  // f32 vectors: this rank keeps the rows of its weight window
            auto B = [&](int w, const char* name, int N, float** dst) {
                plans.push_back({p + name, 1, N, 0, 1, sh[w][0], sh[w][1], nullptr, dst, 0, 0});
            };
            B(TPTC_SHARD_Q, "attn_q.bias", m.n_heads * hd, &L.bq);
            B(TPTC_SHARD_K, "attn_k.bias", m.n_kv_heads * hd, &L.bk);
            B(TPTC_SHARD_V, "attn_v.bias", m.n_kv_heads * hd, &L.bv);
        }
        W(TPTC_SHARD_O, "attn_output.weight", m.dim, m.n_heads * hd, &L.o, 0, 0);
        plans.push_back({p + "ffn_norm.weight", 1, m.dim, 0, 1, 0, m.dim, nullptr, &L.ffn_norm, 0, 0});
        L.moe = m.n_expert > 1 && f.find(p + "ffn_gate_inp.weight") != nullptr;
        if (L.moe) {
            // router [n_expert][dim]; the experts stacked (ffn_*_exps, llama.cpp's layout, split per
            // expert as wgpu_loader.rs:151-173 does) or one tensor each (ffn_*.E, candle's
            // quantized_llama names); gate|up of every expert first, then every down, so each
            // group lands at a uniform stride in the arena
            Plan rp{p + "ffn_gate_inp.weight", m.n_expert, m.dim, 0, m.n_expert, 0, m.dim, nullptr, nullptr, 0, 0};
            rp.raw = &L.router;
            rp.raw_type = &L.router_type;
            plans.push_back(rp);
            const int E = m.n_expert, eff = m.expert_ffn;
            const bool stacked = f.find(p + "ffn_gate_exps.weight") != nullptr;
            L.eglu_all.assign(E, DevMatrix{});
            L.edown_all.assign(E, DevMatrix{});
            auto X = [&](const char* stem, int e, int N, int K, DevMatrix* mat, int first_row, int glu_rows) {
                Plan q{stacked ? p + stem + "_exps.weight" : p + stem + "." + std::to_string(e) + ".weight",
                       N, K, 0, N, 0, K, mat, nullptr, first_row, glu_rows};
                if (stacked) {
                    q.expert = e;
                    q.n_stack = E;
                }
                plans.push_back(q);
            };
            for (int e = 0; e < E; e++) {
                X("ffn_gate", e, eff, m.dim, &L.eglu_all[e], 0, 2 * eff);
                X("ffn_up", e, eff, m.dim, &L.eglu_all[e], eff, 2 * eff);
            }
            for (int e = 0; e < E; e++) X("ffn_down", e, m.dim, eff, &L.edown_all[e], 0, 0);
            // an always-on shared expert (the reference's wgpu_engine.rs:840-853)
            if (const GgufTensor* sg = f.find(p + "ffn_gate_shexp.weight")) {
                const int sffn = sg->ne.size() == 2 ? (int)sg->ne[1] : 0;
                if (sffn <= 0 || sffn % QK_K)
                    return err(TPTC_ERR_UNSUPPORTED, "shared expert rows must be a multiple of 256");
                if (meta_.shared_ffn && meta_.shared_ffn != sffn)
                    return err(TPTC_ERR_UNSUPPORTED, "shared experts of different sizes");
                meta_.shared_ffn = sffn;
                L.shexp = true;
                plans.push_back({p + "ffn_gate_shexp.weight", sffn, m.dim, 0, sffn, 0, m.dim, &L.glu, nullptr, 0, 2 * sffn});
                plans.push_back({p + "ffn_up_shexp.weight", sffn, m.dim, 0, sffn, 0, m.dim, &L.glu, nullptr, sffn, 2 * sffn});
                plans.push_back({p + "ffn_down_shexp.weight", m.dim, sffn, 0, m.dim, 0, sffn, &L.down, nullptr, 0, 0});
            }
        } else if (m.fused_gate_up) {  // ffn_up rows [0, ffn) gate, [ffn, 2 ffn) up
            W(TPTC_SHARD_GATE, "ffn_up.weight", m.ffn, m.dim, &L.glu, 0, 2 * ffn_l, 0, 2 * m.ffn);
            W(TPTC_SHARD_UP, "ffn_up.weight", m.ffn, m.dim, &L.glu, ffn_l, 2 * ffn_l, m.ffn, 2 * m.ffn);
        } else {
            W(TPTC_SHARD_GATE, "ffn_gate.weight", m.ffn, m.dim, &L.glu, 0, 2 * ffn_l);
            W(TPTC_SHARD_UP, "ffn_up.weight", m.ffn, m.dim, &L.glu, ffn_l, 2 * ffn_l);
        }
        if (!L.moe) W(TPTC_SHARD_DOWN, "ffn_down.weight", m.dim, m.ffn, &L.down, 0, 0);
    }
    plans.push_back({"output_norm.weight", 1, m.dim, 0, 1, 0, m.dim, nullptr, &out_norm_, 0, 0});
    // lm_head: vocab-parallel under tensor parallelism when the vocabulary splits evenly (each
    // rank its rows; with tied embeddings those rows of token_embd, which stays whole for the
    // embedding lookup), replicated otherwise
    head_rows_ = m.vocab;
    head_row0_ = 0;
    if (tp_size_ > 1 && m.vocab % tp_size_ == 0) {
        head_rows_ = m.vocab / tp_size_;
        head_row0_ = tp_rank_ * head_rows_;
    }
    const bool head_sliced = head_rows_ < m.vocab;
    if (!m.tied || head_sliced)
        plans.push_back({m.tied ? "token_embd.weight" : "output.weight", m.vocab, m.dim, head_row0_,
                         head_row0_ + head_rows_, 0, m.dim, &output_, nullptr, 0, 0});

    // ---- validate and lay out the arena
    size_t off = 0;
    std::vector<size_t> offs(plans.size(), 0);
    std::vector<const GgufTensor*> tens(plans.size());
    for (size_t i = 0; i < plans.size(); i++) {
        Plan& p = plans[i];
        const GgufTensor* t = f.find(p.name);
        if (!t) return err(TPTC_ERR_FORMAT, "missing tensor '" + p.name + "'");
        tens[i] = t;
        const bool vec = p.mat == nullptr && p.raw == nullptr;
        const uint64_t want0 = (uint64_t)p.K, want1 = (uint64_t)p.N;
        bool shape_ok = vec ? (t->ne.size() == 1 && t->ne[0] == want0)
                        : p.n_stack ? (t->ne.size() == 3 && t->ne[0] == want0 && t->ne[1] == want1 &&
                                       t->ne[2] == (uint64_t)p.n_stack)
                                    : (t->ne.size() == 2 && t->ne[0] == want0 && t->ne[1] == want1);
        if (!shape_ok) return err(TPTC_ERR_FORMAT, "tensor '" + p.name + "' has an unexpected shape");
        if (p.raw) {  // the MoE router: f32 or f16 rows, used as they are (candle dequantises to f32)
            if (t->type != TPTC_TYPE_F32 && t->type != TPTC_TYPE_F16)
                return err(TPTC_ERR_UNSUPPORTED, "router tensor '" + p.name + "' must be F32 or F16");
            *p.raw_type = (int)t->type;
            offs[i] = off;
            off = align_up(off + (size_t)p.N * p.K * (t->type == TPTC_TYPE_F32 ? 4 : 2), 256);
            continue;
        }
        if (vec) {
            if (t->type != TPTC_TYPE_F32) return err(TPTC_ERR_UNSUPPORTED, "vector tensor '" + p.name + "' must be F32");
            offs[i] = off;
            off = align_up(off + (size_t)(p.k1 - p.k0) * 4, 256);
            continue;
        }
        if (!matrix_type_ok((int)t->type))
            return err(TPTC_ERR_UNSUPPORTED, "tensor '" + p.name + "' has unsupported GGML type " + std::to_string(t->type));
        if (p.glu_rows && p.first_row > 0) {  // second half of a fused gate|up matrix
            if ((int)t->type != p.mat->type)
                return err(TPTC_ERR_UNSUPPORTED, "ffn_gate and ffn_up must share a GGML type (" + p.name + ")");
            continue;
        }
        DevMatrix& d = *p.mat;
        d = dm_geometry((int)t->type, p.glu_rows ? p.glu_rows : p.r1 - p.r0, p.k1 - p.k0, p.glu_rows ? 1 : 0);
        offs[i] = off;
        off = align_up(off + (size_t)d.main_bytes(), 256);
    }
    arena_size_ = off;
    cudaError_t ce = cudaMalloc(&arena_, arena_size_);
    if (ce != cudaSuccess) {
        arena_ = nullptr;
        return err(TPTC_ERR_OOM, "weights need " + std::to_string(arena_size_ >> 20) + " MiB: " + cuda_msg(ce, "cudaMalloc"));
    }
    device_bytes_ = arena_size_;
    CU(cudaMemsetAsync(arena_, 0, arena_size_, stream_));  // tile padding rows stay zero

    // ---- upload
    Stager sg(stream_);
    RET_IF(sg.init());
    weight_bytes_ = 0;
    for (size_t i = 0; i < plans.size(); i++) {
        Plan& p = plans[i];
        const GgufTensor* t = tens[i];
        const uint8_t* src = f.tensor_data(*t);
        if (p.raw) {
            const int64_t rb = (int64_t)p.K * (*p.raw_type == TPTC_TYPE_F32 ? 4 : 2);
            *p.raw = arena_ + offs[i];
            DevMatrix tmp;
            tmp.type = TPTC_TYPE_F32;  // copied as is
            tmp.main = arena_ + offs[i];
            RET_IF(upload_rows(sg, src, rb, 0, p.N, 0, rb, tmp, 0));
            weight_bytes_ += (uint64_t)p.N * rb;
        } else if (!p.mat) {
            *p.vec = reinterpret_cast<float*>(arena_ + offs[i]);
            DevMatrix tmp;
            tmp.type = TPTC_TYPE_F32;
            tmp.main = arena_ + offs[i];
            RET_IF(upload_rows(sg, src, (int64_t)p.K * 4, 0, 1, (int64_t)p.k0 * 4, (int64_t)p.k1 * 4, tmp, 0));
            weight_bytes_ += (uint64_t)(p.k1 - p.k0) * 4;
        } else {
            DevMatrix& d = *p.mat;
            if (!(p.glu_rows && p.first_row > 0)) {
                d.main = arena_ + offs[i];
            }
            const int64_t rrb = raw_row_bytes(d.type, p.K);
            const int64_t c0 = raw_row_bytes(d.type, p.k0), c1 = raw_row_bytes(d.type, p.k1);
            if (p.expert >= 0) src += (int64_t)p.expert * p.N * rrb;  // this expert's slice of the stack
            RET_IF(upload_rows(sg, src, rrb, p.r0, p.r1, c0, c1, d, p.first_row));
            weight_bytes_ += (uint64_t)(p.r1 - p.r0) * d.main_row_bytes;
        }
        if (cb) cb((uint32_t)(i + 1), (uint32_t)plans.size(), user);
    }
    if (m.tied && !head_sliced) output_ = embd_;
    // every expert of a layer: one type and shape, at a uniform stride (the GEMVs address
    // expert e as expert 0's matrix plus e strides)
    for (LayerWeights& L : layers_) {
        if (!L.moe) continue;
        auto stack = [&](const std::vector<DevMatrix>& all, DevMatrix& first, int64_t& stride) -> bool {
            first = all[0];
            stride = all.size() > 1 ? (int64_t)(all[1].main - all[0].main) : 0;
            for (size_t e = 1; e < all.size(); e++)
                if (all[e].type != first.type || all[e].N != first.N || all[e].K != first.K ||
                    all[e].main != first.main + (int64_t)e * stride)
                    return false;
            return true;
        };
        if (!stack(L.eglu_all, L.eglu, L.eglu_stride) || !stack(L.edown_all, L.edown, L.edown_stride))
            return err(TPTC_ERR_UNSUPPORTED, "the experts of a layer must share one GGML type per projection");
    }
    CU(cudaStreamSynchronize(stream_));
    RET_IF(alloc_runtime());
    loaded_ = true;
    return {};
}

Status Engine::alloc_runtime() {
    const ModelMeta& m = meta_;
    const int hd = m.head_dim, L = m.n_layers;
    max_seq_ = m.context_length;
    attn_splits_ = attn_decode_splits(n_kv_l_, max_seq_, sm_count_);
    const size_t kv_elems = (size_t)L * 2 * n_kv_l_ * max_seq_ * hd;
    const int half = hd / 2;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const size_t o_kv = take(kv_elems * kv_elem_bytes());
    const size_t o_cos = take((size_t)max_seq_ * half * 4), o_sin = take((size_t)max_seq_ * half * 4);
    const size_t o_x = take((size_t)m.dim * 4), o_x2 = take((size_t)m.dim * 4);
    const size_t o_q = take((size_t)n_heads_l_ * hd * 4), o_att = take((size_t)n_heads_l_ * hd * 4);
    const size_t o_qr = take((size_t)n_heads_l_ * hd * 4), o_kr = take((size_t)n_kv_l_ * hd * 4);
    // h: [2 ffn_l] (gate|up products); under MoE the selected experts' products side by side,
    // then the shared expert's
    const size_t h_floats = std::max((size_t)2 * (m.ffn / tp_size_),
                                     (size_t)m.n_expert_used * m.expert_ffn + (size_t)m.shared_ffn);
    const size_t o_h = take(h_floats * 4), o_lg = take((size_t)m.vocab * 4);
    const size_t o_mlg = take((size_t)std::max(1, m.n_expert) * 4), o_msel = take((size_t)kMoeMaxUsed * 4);
    const size_t o_mw = take((size_t)kMoeMaxUsed * 4), o_macc = take((size_t)m.dim * 4), o_mcnt = take(64);
    const size_t o_ti = take(64), o_to = take(64), o_pos = take(64), o_err = take(64), o_step = take(64);
    const size_t o_hist = take((size_t)max_seq_ * 4 + 64);
    const size_t o_part = take(attn_decode_partial_floats(n_heads_l_, n_kv_l_, hd, attn_splits_) * 4);
    const size_t o_cnt = take((size_t)n_kv_l_ * 4);
    const int k_max = std::max(std::max(m.dim, std::max(m.ffn / tp_size_, n_heads_l_ * hd)),
                               std::max(m.expert_ffn, m.shared_ffn));
    const size_t o_act = take(gemv_act_bytes_max(k_max));
    const size_t o_cbar = take((size_t)(L + 1) * kChainMaxPhases * 4);
    const size_t o_bval = take((size_t)2 * sm_count_ * 4), o_bidx = take((size_t)2 * sm_count_ * 4);
    const size_t o_scnt = take((size_t)m.vocab * 4), o_sscr = take((size_t)m.vocab * 4), o_sstep = take(64);
    const size_t o_swork = take(kSampleWorkBytes);
    rt_size_ = off;
    cudaError_t ce = cudaMalloc(&rt_, rt_size_);
    if (ce != cudaSuccess) {
        rt_ = nullptr;
        return err(TPTC_ERR_OOM, "KV cache / runtime buffers need " + std::to_string(rt_size_ >> 20) +
                                     " MiB: " + cuda_msg(ce, "cudaMalloc"));
    }
    device_bytes_ += rt_size_;
    CU(cudaMemsetAsync(rt_, 0, rt_size_, stream_));
    kv_ = rt_ + o_kv;
    rope_cos_ = reinterpret_cast<float*>(rt_ + o_cos);
    rope_sin_ = reinterpret_cast<float*>(rt_ + o_sin);
    x_ = reinterpret_cast<float*>(rt_ + o_x);
    x2_ = reinterpret_cast<float*>(rt_ + o_x2);
    qbuf_ = reinterpret_cast<float*>(rt_ + o_q);
    attn_ = reinterpret_cast<float*>(rt_ + o_att);
    qrot_ = reinterpret_cast<float*>(rt_ + o_qr);
    kraw_ = reinterpret_cast<float*>(rt_ + o_kr);
    h_ = reinterpret_cast<float*>(rt_ + o_h);
    moe_logits_ = reinterpret_cast<float*>(rt_ + o_mlg);
    moe_sel_ = reinterpret_cast<int*>(rt_ + o_msel);
    moe_w_ = reinterpret_cast<float*>(rt_ + o_mw);
    moe_acc_ = reinterpret_cast<float*>(rt_ + o_macc);
    moe_count_ = reinterpret_cast<int*>(rt_ + o_mcnt);
    logits_ = reinterpret_cast<float*>(rt_ + o_lg);
    tok_in_ = reinterpret_cast<uint32_t*>(rt_ + o_ti);
    tok_out_ = reinterpret_cast<uint32_t*>(rt_ + o_to);
    pos_ = reinterpret_cast<int*>(rt_ + o_pos);
    err_ = reinterpret_cast<int*>(rt_ + o_err);
    step_ = reinterpret_cast<int*>(rt_ + o_step);
    history_ = reinterpret_cast<uint32_t*>(rt_ + o_hist);
    attn_partial_ = reinterpret_cast<float*>(rt_ + o_part);
    attn_counters_ = reinterpret_cast<int*>(rt_ + o_cnt);
    act_ = rt_ + o_act;
    chain_bar_ = reinterpret_cast<int*>(rt_ + o_cbar);
    best_val_ = reinterpret_cast<float*>(rt_ + o_bval);
    best_idx_ = reinterpret_cast<int*>(rt_ + o_bidx);
    sample_counts_ = reinterpret_cast<int*>(rt_ + o_scnt);
    sample_scratch_ = reinterpret_cast<float*>(rt_ + o_sscr);
    sample_work_ = rt_ + o_swork;
    sample_step_ = reinterpret_cast<int*>(rt_ + o_sstep);

    // candle quantized_llama precomput_freqs_cis: theta_i = 1/base^(2i/hd) (f32 powf),
    // angle = pos * theta_i, cos/sin in f32 -- built on the host with the C library's powf,
    // cosf and sinf (rope.wgsl:37-50 computes the same rotation per dispatch).
    std::vector<float> c((size_t)max_seq_ * half), s((size_t)max_seq_ * half);
    for (int p = 0; p < max_seq_; p++) {
        float pf = (float)p;
        if (m.rope_scale != 1.f) pf = pf / m.rope_scale;
        for (int i = 0; i < half; i++) {
            const float theta = 1.f / powf(m.rope_freq_base, (float)(2 * i) / (float)hd);
            const float ang = pf * theta;
            c[(size_t)p * half + i] = cosf(ang);
            s[(size_t)p * half + i] = sinf(ang);
        }
    }
    CU(cudaMemcpyAsync(rope_cos_, c.data(), c.size() * 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaMemcpyAsync(rope_sin_, s.data(), s.size() * 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaStreamSynchronize(stream_));
    // the peer-memory inboxes are baked into the graphs: map them before capture
    if (tp_) RET_IF(tp_->init_p2p(m.dim, m.n_layers, step_, tp_wait_polls_, stream_));
    RET_IF(build_decode_graph(false, &graph_plain_));
    RET_IF(build_decode_graph(true, &graph_chained_));
    return {};
}

// One decode step: embed -> L x (QKV+RoPE+KV write, flash-decode, O+residual,
// gate/up+SiLU, down+residual) -> norm + lm_head -> argmax.  All positions come from the
// device scalar pos_, so one captured graph serves every step.
Status Engine::enqueue_decode(cudaStream_t st, bool chained, float* trace) {
    const ModelMeta& m = meta_;
    const int hd = m.head_dim, L = m.n_layers;
    const size_t layer_kv = (size_t)2 * n_kv_l_ * max_seq_ * hd * kv_elem_bytes();  // bytes
    auto kcache = [&](int l) { return kv_ + l * layer_kv; };
    auto vcache = [&](int l) { return kv_ + l * layer_kv + layer_kv / 2; };
    auto base = [&](int K) {
        GemvParams p = {};
        p.K = K;
        p.err = err_;
        p.act_global = act_;
        p.eps = m.rms_eps;
        p.nseg = 1;
        return p;
    };
    // q | k | v with fused RMSNorm; v goes straight into the cache, q and k are rotated by
    // the attention kernel
    // Tensor parallelism: the residual stream alternates between x_ and x2_.  A layer starts
    // with x in x_; o scatters its partial rows (slot 0) and the gate|up activation gathers
    // them into x2_; down scatters (slot 1) and the next q|k|v (or the head) activation
    // gathers them back into x_ (TpLink, gemv.cuh).
    const TpLink* link = tp_ ? tp_->link_dev : nullptr;
    auto gather = [&](GemvParams& p, int slot, int use, float* from, float* to) {
        p.x = from;
        p.tp = link;
        p.tp_slot = slot;
        p.tp_use = use;
        p.tp_gather = 1;
        p.x_out = to;
    };
    auto qkv_params = [&](int l) {
        const LayerWeights& W = layers_[l];
        GemvParams p = base(m.dim);
        p.nseg = 3;
        const DevMatrix* qkv[3] = {&W.q, &W.k, &W.v};
        for (int i = 0; i < 3; i++) p.seg[i] = GemvSeg{*qkv[i], 0};
        p.x = x_;
        if (link && l > 0) gather(p, 1, 2 * (l - 1) + 1, x2_, x_);
        p.norm_w = W.attn_norm;
        p.out = qbuf_;
        p.kraw = kraw_;
        p.vcache = vcache(l);
        p.kv_f32 = kv_f32_ ? 1 : 0;
        p.pos = pos_;
        p.hd = hd;
        p.max_seq = max_seq_;
        p.bias[0] = W.bq;
        p.bias[1] = W.bk;
        p.bias[2] = W.bv;
        gemv_prepare(p, sm_count_);
        return p;
    };
    auto o_params = [&](int l) {
        GemvParams p = base(n_heads_l_ * hd);
        p.seg[0] = GemvSeg{layers_[l].o, 0};
        p.x = attn_;
        p.out = x_;
        if (link) {  // row-parallel: partial rows into every rank's inbox
            p.tp = link;
            p.tp_slot = 0;
            p.tp_use = 2 * l;
        }
        gemv_prepare(p, sm_count_);
        return p;
    };
    auto glu_params = [&](int l) {
        GemvParams p = base(m.dim);
        p.seg[0] = GemvSeg{layers_[l].glu, 0};
        p.x = x_;
        if (link) gather(p, 0, 2 * l, x_, x2_);
        p.norm_w = layers_[l].ffn_norm;
        p.out = h_;
        p.glu_act = m.geglu ? 1 : 0;
        gemv_prepare(p, sm_count_);
        return p;
    };
    // Mixture-of-experts feed-forward of layer l (candle MlpOrMoe::MoE): routing on the device,
    // gate|up of the selected experts (up to three per launch, one activation build), then one
    // down launch per expert accumulating the weighted sum, the last adding it to x; a shared
    // expert runs after the routed ones with weight 1.
    auto enqueue_moe = [&](int l) -> Status {
        const LayerWeights& W = layers_[l];
        const int K = m.n_expert_used, eff = m.expert_ffn;
        MoeRouteParams r = {};
        r.x = x_;
        r.norm_w = W.ffn_norm;
        r.eps = m.rms_eps;
        r.router = W.router;
        r.router_f16 = W.router_type == TPTC_TYPE_F16 ? 1 : 0;
        r.dim = m.dim;
        r.n_expert = m.n_expert;
        r.n_used = K;
        r.logits = moe_logits_;
        r.sel = moe_sel_;
        r.w = moe_w_;
        r.count = moe_count_;
        CU(launch_moe_route(r, st, pdl_));
        bool act_ready = false;
        for (int k0 = 0; k0 < K; k0 += kGemvMaxSeg) {
            GemvParams g = base(m.dim);
            g.nseg = std::min(kGemvMaxSeg, K - k0);
            for (int i = 0; i < g.nseg; i++) {
                g.seg[i] = GemvSeg{W.eglu, 0};
                g.seg[i].out_off = (k0 + i) * eff;
                g.seg[i].sel = k0 + i;
            }
            g.moe_sel = moe_sel_;
            g.moe_stride = W.eglu_stride;
            g.moe_nexp = m.n_expert;
            g.x = x_;
            g.norm_w = W.ffn_norm;
            g.out = h_;
            g.glu_act = m.geglu ? 1 : 0;
            g.act_prepared = act_ready ? 1 : 0;  // the first launch's activation is still in act_
            gemv_prepare(g, sm_count_);
            CU(gemv_launch(g, EPI_GLU, st, pdl_));
            act_ready = true;
        }
        if (W.shexp) {
            GemvParams g = base(m.dim);
            g.seg[0] = GemvSeg{W.glu, 0};
            g.seg[0].out_off = K * eff;
            g.x = x_;
            g.norm_w = W.ffn_norm;
            g.out = h_;
            g.glu_act = m.geglu ? 1 : 0;
            g.act_prepared = W.glu.type == W.eglu.type ? 1 : 0;  // same layout as the experts' activation
            gemv_prepare(g, sm_count_);
            CU(gemv_launch(g, EPI_GLU, st, pdl_));
        }
        for (int k = 0; k <= K; k++) {
            if (k == K && !W.shexp) break;
            const bool shared = k == K;
            GemvParams d = base(shared ? m.shared_ffn : eff);
            d.seg[0] = GemvSeg{shared ? W.down : W.edown, 0};
            if (!shared) {
                d.seg[0].sel = k;
                d.moe_sel = moe_sel_;
                d.moe_stride = W.edown_stride;
                d.moe_nexp = m.n_expert;
            }
            d.x = h_ + (size_t)k * eff;
            d.out = x_;
            d.moe_acc = moe_acc_;
            d.moe_w = moe_w_;
            d.moe_slot = shared ? -1 : k;
            d.moe_first = k == 0 ? 1 : 0;
            d.moe_last = (shared || (k == K - 1 && !W.shexp)) ? 1 : 0;
            gemv_prepare(d, sm_count_);
            CU(gemv_launch(d, EPI_RESID, st, pdl_));
        }
        return {};
    };
    auto down_params = [&](int l) {
        GemvParams p = base(m.ffn / tp_size_);
        p.seg[0] = GemvSeg{layers_[l].down, 0};
        p.x = h_;
        p.out = x_;
        if (link) {
            p.tp = link;
            p.tp_slot = 1;
            p.tp_use = 2 * l + 1;
        }
        gemv_prepare(p, sm_count_);
        return p;
    };
    auto head_params = [&]() {
        GemvParams p = base(m.dim);
        p.seg[0] = GemvSeg{output_, 0};
        p.x = x_;
        if (link) gather(p, 1, 2 * (m.n_layers - 1) + 1, x2_, x_);
        p.norm_w = out_norm_;
        p.out = logits_ + head_row0_;  // this rank's rows of the vocabulary
        gemv_prepare(p, sm_count_);
        return p;
    };
    // attention of layer l; when every kv head's output is whole 256-blocks the kernel also
    // writes the o projection's activation itself (q8k / q80 / f32 as the o matrix needs)
    auto attn_params = [&](int l, GemvParams& o) {
        AttnDecodeParams a = {};
        a.q = qbuf_;
        a.kraw = kraw_;
        a.kcache = kcache(l);
        a.vcache = vcache(l);
        a.kv_f32 = kv_f32_ ? 1 : 0;
        a.rope_cos = rope_cos_;
        a.rope_sin = rope_sin_;
        a.q_out = qrot_;
        a.pos = pos_;
        a.out = attn_;
        a.partial = attn_partial_;
        a.counters = attn_counters_;
        a.n_heads = n_heads_l_;
        a.n_kv = n_kv_l_;
        a.hd = hd;
        a.max_seq = max_seq_;
        a.splits = attn_splits_;
        a.scale = (float)(1.0 / sqrt((double)hd));
        a.err = err_;
        a.rope_neox = m.rope_neox ? 1 : 0;
        if ((n_heads_l_ / n_kv_l_) * hd % 256 == 0) {
            a.act_out = act_;
            a.act = o.act;
            a.act_transposed = 1;
            a.act_nb = o.K / 256;
            o.act_prepared = 1;
        }
        return a;
    };
    auto trace_layer = [&](int l) -> Status {
        if (!trace) return {};
        CU(cudaMemcpyAsync(trace + (size_t)(l * 3 + 0) * m.dim, qrot_, (size_t)n_heads_l_ * hd * 4,
                           cudaMemcpyDeviceToHost, st));
        CU(cudaMemcpyAsync(trace + (size_t)(l * 3 + 1) * m.dim, attn_, (size_t)n_heads_l_ * hd * 4,
                           cudaMemcpyDeviceToHost, st));
        CU(cudaMemcpyAsync(trace + (size_t)(l * 3 + 2) * m.dim, x_, (size_t)m.dim * 4, cudaMemcpyDeviceToHost, st));
        return {};
    };

    bool use_chain = chain_ && !tp_ && m.n_expert == 0;
    if (use_chain) {  // the chains with the largest activation / stage (the widest layer, the head)
        ChainParams t = {};
        t.ph[0] = o_params(L - 1);
        t.ph[1] = glu_params(L - 1);
        t.ph[2] = down_params(L - 1);
        t.ph[3] = head_params();
        t.nph = 4;
        chain_prepare(t, sm_count_);
        use_chain = chain_fits(t, sm_count_);
        t.ph[3] = qkv_params(0);
        chain_prepare(t, sm_count_);
        use_chain = use_chain && chain_fits(t, sm_count_);
    }
    CU(launch_embed_row(embd_, tok_in_, x_, st, false, link ? step_ : nullptr, m.embd_scale));
    if (use_chain) {
        // GEMV chains: [q|k|v(0)], then per layer attention(l) and one chain
        // [o(l), gate|up(l), down(l), q|k|v(l+1) or lm_head + argmax]
        ChainParams c0 = {};
        c0.ph[0] = qkv_params(0);
        c0.epi[0] = EPI_QKV;
        c0.nph = 1;
        c0.bar = chain_bar_;
        c0.err = err_;
        chain_prepare(c0, sm_count_);
        CU(chain_launch(c0, st, pdl_));
        for (int l = 0; l < L; l++) {
            GemvParams o = o_params(l);
            const AttnDecodeParams a = attn_params(l, o);
            CU(launch_attn_decode(a, st, pdl_));
            ChainParams c = {};
            c.ph[0] = o;
            c.epi[0] = EPI_RESID;
            c.ph[1] = glu_params(l);
            c.epi[1] = EPI_GLU;
            c.ph[2] = down_params(l);
            c.epi[2] = EPI_RESID;
            if (l + 1 < L) {
                c.ph[3] = qkv_params(l + 1);
                c.epi[3] = EPI_QKV;
            } else {
                c.ph[3] = head_params();
                c.epi[3] = EPI_STORE;
                c.best_val = best_val_;
                c.best_idx = best_idx_;
                c.out_tok = tok_out_;
                c.next_tok = chained ? tok_in_ : nullptr;
                c.pos = chained ? pos_ : nullptr;
                c.history = chained ? history_ : nullptr;
            }
            c.nph = 4;
            c.bar = chain_bar_ + (size_t)(l + 1) * kChainMaxPhases;
            c.err = err_;
            chain_prepare(c, sm_count_);
            CU(chain_launch(c, st, pdl_));
            RET_IF(trace_layer(l));
        }
        return {};
    }
    for (int l = 0; l < L; l++) {
        GemvParams p = qkv_params(l);
        CU(gemv_launch(p, EPI_QKV, st, pdl_));
        GemvParams o = o_params(l);
        const AttnDecodeParams a = attn_params(l, o);
        CU(launch_attn_decode(a, st, pdl_));
        CU(gemv_launch(o, EPI_RESID, st, pdl_));  // under TP: scatter to every rank's inbox
        if (layers_[l].moe) {
            RET_IF(enqueue_moe(l));
        } else {
            GemvParams g = glu_params(l);
            CU(gemv_launch(g, EPI_GLU, st, pdl_));
            GemvParams d = down_params(l);
            CU(gemv_launch(d, EPI_RESID, st, pdl_));
        }
        RET_IF(trace_layer(l));
    }
    GemvParams h = head_params();
    CU(gemv_launch(h, EPI_STORE, st, pdl_));
    if (head_rows_ < m.vocab)  // vocab-parallel: the ranks exchange their best over peer memory
        CU(launch_argmax_tp(logits_ + head_row0_, head_rows_, head_row0_, link, err_, tok_out_,
                            chained ? tok_in_ : nullptr, chained ? pos_ : nullptr, chained ? history_ : nullptr, st,
                            pdl_));
    else
        CU(launch_argmax(logits_, m.vocab, tok_out_, chained ? tok_in_ : nullptr, chained ? pos_ : nullptr,
                         chained ? history_ : nullptr, st, pdl_));
    return {};
}

Status Engine::build_decode_graph(bool chained, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    CU(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    Status s = enqueue_decode(stream_, chained);
    cudaError_t ce = cudaStreamEndCapture(stream_, &g);
    if (!s.ok()) {
        if (g) cudaGraphDestroy(g);
        return s;
    }
    if (ce != cudaSuccess) return err(TPTC_ERR_CUDA, cuda_msg(ce, "cudaStreamEndCapture"));
    size_t nn = 0;
    if (cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess && nn) {
        std::vector<cudaGraphNode_t> nodes(nn);
        int kernels = 0;
        if (cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
            for (size_t i = 0; i < nn; i++) {
                cudaGraphNodeType t;
                if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) kernels++;
            }
        graph_kernels_ = kernels;
    }
    ce = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return err(TPTC_ERR_CUDA, cuda_msg(ce, "cudaGraphInstantiate"));
    return {};
}

Status Engine::check_err() {
    CU(cudaMemcpyAsync(h_err_, err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    CU(cudaStreamSynchronize(stream_));
    if (*h_err_ != 0) {
        const int code = *h_err_;
        cudaMemsetAsync(err_, 0, sizeof(int), stream_);
        // a chain that gave up leaves its arrival counters mid-count
        if (chain_bar_) cudaMemsetAsync(chain_bar_, 0, (size_t)(meta_.n_layers + 1) * kChainMaxPhases * 4, stream_);
        cudaStreamSynchronize(stream_);
        return err(code == TPTC_ERR_TIMEOUT ? TPTC_ERR_TIMEOUT : TPTC_ERR_CUDA,
                   "a device-side bounded wait gave up (status " + std::to_string(code) + ")");
    }
    return {};
}

Status Engine::sync() {
    CU(cudaStreamSynchronize(stream_));
    return check_err();
}

Status Engine::kv_reset() {
    cached_tokens_.clear();
    return {};
}

int common_prefix_len(const uint32_t* cached, int n_cached, const uint32_t* ids, int n) {
    int i = 0;
    const int lim = std::min(n, n_cached);
    while (i < lim && cached[i] == ids[i]) i++;
    return i;
}

int Engine::prefix_len(const uint32_t* ids, int n) const {
    return common_prefix_len(cached_tokens_.data(), (int)cached_tokens_.size(), ids, n);
}

Status Engine::decode(uint32_t id, int pos, float* logits, uint32_t* argmax) {
    if (!loaded_) return err(TPTC_ERR_STATE, "no model loaded");
    if (id >= (uint32_t)meta_.vocab) return err(TPTC_ERR_ARG, "token id out of range");
    if (pos < 0 || pos >= max_seq_) return err(TPTC_ERR_ARG, "position outside the context window");
    if (pos != (int)cached_tokens_.size())
        return err(TPTC_ERR_ARG, "decode position must equal the KV length (" + std::to_string(cached_tokens_.size()) + ")");
    CU(cudaSetDevice(device_));
    h_tok_[0] = id;
    h_pos_[0] = pos;
    CU(cudaMemcpyAsync(tok_in_, h_tok_, 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaMemcpyAsync(pos_, h_pos_, 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaGraphLaunch(graph_plain_, stream_));
    if (logits) {
        RET_IF(gather_logits());
        CU(cudaMemcpyAsync(logits, logits_, (size_t)meta_.vocab * 4, cudaMemcpyDeviceToHost, stream_));
    }
    if (argmax) CU(cudaMemcpyAsync(h_tok_ + 1, tok_out_, 4, cudaMemcpyDeviceToHost, stream_));
    RET_IF(sync());
    if (argmax) *argmax = h_tok_[1];
    cached_tokens_.push_back(id);
    return {};
}

Status Engine::sample_reset(const uint32_t* context, int n) {
    std::vector<int> counts(meta_.vocab, 0);
    for (int i = 0; i < n; i++)
        if (context[i] < (uint32_t)meta_.vocab) counts[context[i]]++;
    CU(cudaMemcpyAsync(sample_counts_, counts.data(), (size_t)meta_.vocab * 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaMemsetAsync(sample_step_, 0, 4, stream_));
    return sync();
}

Status Engine::gather_logits() {
    if (!tp_ || head_rows_ == meta_.vocab) return {};
    return tp_->allgather(logits_, (size_t)head_rows_, stream_);
}

Status Engine::enqueue_sample(const tptc_infer_params& p) {
    RET_IF(gather_logits());  // every rank samples the whole vocabulary, the same draw
    SampleParams s = {};
    s.logits = logits_;
    s.vocab = meta_.vocab;
    s.counts = sample_counts_;
    s.penalty = p.repeat_penalty;
    s.temperature = p.temperature;
    s.top_p = p.top_p;
    s.seed = p.seed;
    s.step = sample_step_;
    s.scratch = sample_scratch_;
    s.work = sample_work_;
    s.out_tok = tok_out_;
    CU(launch_sample(s, stream_, false));
    CU(cudaMemcpyAsync(h_tok_ + 1, tok_out_, 4, cudaMemcpyDeviceToHost, stream_));
    return {};
}

Status Engine::sample_logits(const tptc_infer_params& p, uint32_t* out) {
    RET_IF(enqueue_sample(p));
    RET_IF(sync());
    *out = h_tok_[1];
    return {};
}

Status Engine::decode_sample(uint32_t id, int pos, const tptc_infer_params& p, uint32_t* out) {
    // decode()'s step followed by the selection kernel, one host synchronisation per token
    if (id >= (uint32_t)meta_.vocab) return err(TPTC_ERR_ARG, "token id out of range");
    if (pos < 0 || pos >= max_seq_ || pos != (int)cached_tokens_.size())
        return err(TPTC_ERR_ARG, "decode position must equal the KV length and lie in the context window");
    h_tok_[0] = id;
    h_pos_[0] = pos;
    CU(cudaMemcpyAsync(tok_in_, h_tok_, 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaMemcpyAsync(pos_, h_pos_, 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaGraphLaunch(graph_plain_, stream_));
    RET_IF(enqueue_sample(p));
    RET_IF(sync());
    cached_tokens_.push_back(id);
    *out = h_tok_[1];
    return {};
}

Status Engine::debug_trace(uint32_t id, int pos, float* trace) {
    if (!loaded_) return err(TPTC_ERR_STATE, "no model loaded");
    if (id >= (uint32_t)meta_.vocab || pos != (int)cached_tokens_.size() || pos >= max_seq_)
        return err(TPTC_ERR_ARG, "bad token or position");
    CU(cudaSetDevice(device_));
    h_tok_[0] = id;
    h_pos_[0] = pos;
    CU(cudaMemcpyAsync(tok_in_, h_tok_, 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaMemcpyAsync(pos_, h_pos_, 4, cudaMemcpyHostToDevice, stream_));
    RET_IF(enqueue_decode(stream_, false, trace));
    RET_IF(sync());
    cached_tokens_.push_back(id);
    return {};
}

Status Engine::decode_greedy(uint32_t id, int pos, int n, uint32_t* out_ids) {
    if (!loaded_) return err(TPTC_ERR_STATE, "no model loaded");
    if (n <= 0) return {};
    if (id >= (uint32_t)meta_.vocab) return err(TPTC_ERR_ARG, "token id out of range");
    if (pos < 0 || pos + n > max_seq_) return err(TPTC_ERR_ARG, "steps run past the context window");
    if (pos != (int)cached_tokens_.size()) return err(TPTC_ERR_ARG, "decode position must equal the KV length");
    CU(cudaSetDevice(device_));
    h_tok_[0] = id;
    h_pos_[0] = pos;
    CU(cudaMemcpyAsync(tok_in_, h_tok_, 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaMemcpyAsync(pos_, h_pos_, 4, cudaMemcpyHostToDevice, stream_));
    CU(cudaEventRecord(ev0_, stream_));
    for (int i = 0; i < n; i++) CU(cudaGraphLaunch(graph_chained_, stream_));
    CU(cudaEventRecord(ev1_, stream_));
    std::vector<uint32_t> toks(n);
    CU(cudaMemcpyAsync(toks.data(), history_ + pos, (size_t)n * 4, cudaMemcpyDeviceToHost, stream_));
    RET_IF(sync());
    float ms = 0.f;
    CU(cudaEventElapsedTime(&ms, ev0_, ev1_));
    last_device_ms = ms;
    if (out_ids) memcpy(out_ids, toks.data(), (size_t)n * 4);
    cached_tokens_.push_back(id);
    for (int i = 0; i + 1 < n; i++) cached_tokens_.push_back(toks[i]);
    return {};
}

Status Engine::prefill(const uint32_t* ids, int n, int start_pos, float* last_logits) {
    if (!loaded_) return err(TPTC_ERR_STATE, "no model loaded");
    if (n <= 0) return err(TPTC_ERR_ARG, "prefill of zero tokens");
    if (start_pos != (int)cached_tokens_.size())
        return err(TPTC_ERR_ARG, "start_pos must equal the KV length (" + std::to_string(cached_tokens_.size()) + ")");
    if (start_pos + n > max_seq_) return err(TPTC_ERR_ARG, "prompt runs past the context window");
    for (int i = 0; i < n; i++)
        if (ids[i] >= (uint32_t)meta_.vocab) return err(TPTC_ERR_ARG, "token id out of range");
    CU(cudaSetDevice(device_));
    CU(cudaEventRecord(ev0_, stream_));
    RET_IF(run_prefill_batched(ids, n, start_pos, last_logits));
    CU(cudaEventRecord(ev1_, stream_));
    CU(cudaEventSynchronize(ev1_));
    float ms = 0.f;
    CU(cudaEventElapsedTime(&ms, ev0_, ev1_));
    last_device_ms = ms;
    return {};
}

// ---- LlmEngine::infer over token ids (wgpu_engine.rs:165-334, candle_engine.rs:205-334)

Status Engine::infer(const uint32_t* prompt, int n, const tptc_infer_params& p, tptc_token_cb cb, void* user) {
    using clk = std::chrono::steady_clock;
    if (!loaded_) return err(TPTC_ERR_STATE, "no model loaded");
    if (!cb) return err(TPTC_ERR_ARG, "on_token callback is required");
    CU(cudaSetDevice(device_));
    std::vector<uint32_t> tokens(prompt, prompt + std::max(0, n));
    for (uint32_t t : tokens)
        if (t >= (uint32_t)meta_.vocab) return err(TPTC_ERR_ARG, "token id out of range");
    // truncate from the front (wgpu_engine.rs:188-197)
    const int max_prompt = std::max(0, meta_.context_length - (int)p.max_tokens);
    if ((int)tokens.size() > max_prompt) {
        tokens.erase(tokens.begin(), tokens.begin() + ((int)tokens.size() - max_prompt));
        cached_tokens_.clear();
    }
    if (tokens.empty()) return err(TPTC_ERR_ARG, "prompt is empty after tokenization");
    // prefix reuse (wgpu_engine.rs:199-206); the last prompt token is always recomputed so
    // that its logits exist (the reference reads stale logits when the whole prompt hits).
    int prefix = prefix_len(tokens.data(), (int)tokens.size());
    if (prefix >= (int)tokens.size()) prefix = (int)tokens.size() - 1;
    cached_tokens_.resize(prefix);

    // next-token selection on the device (sample.cu): the context counts feed the repeat
    // penalty; greedy without a penalty keeps the argmax inside the decode graph
    const bool greedy = !(p.temperature >= 1e-7f);  // candle: temperature < 1e-7 is argmax
    const bool penalty = fabsf(p.repeat_penalty - 1.f) >= 1.1920929e-7f;

    auto t0 = clk::now();
    RET_IF(prefill(tokens.data() + prefix, (int)tokens.size() - prefix, prefix, nullptr));
    RET_IF(sample_reset(tokens.data(), (int)tokens.size()));
    uint32_t next = 0;
    RET_IF(sample_logits(p, &next));
    auto t1 = clk::now();
    last_prefill_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    last_n_prompt = (int)tokens.size() - prefix;

    int pos = (int)tokens.size();
    uint32_t generated = 0;
    auto td = clk::now();
    for (;;) {
        if (p.eos_token_id >= 0 && next == (uint32_t)p.eos_token_id) break;
        if (generated >= p.max_tokens) break;
        if (pos >= meta_.context_length) break;
        if (cb(next, 0, user) != 0) {
            cb(0, 1, user);
            last_decode_ms = std::chrono::duration<double, std::milli>(clk::now() - td).count();
            last_n_generated = (int)generated;
            return err(TPTC_ERR_CANCELLED, "inference cancelled by the token callback");
        }
        tokens.push_back(next);
        generated++;
        if (greedy && !penalty) {
            uint32_t am;
            RET_IF(decode(next, pos, nullptr, &am));
            next = am;
        } else {
            // the sampled token was counted by the kernel; `next` enters the context here
            RET_IF(decode_sample(next, pos, p, &next));
        }
        pos++;
    }
    last_decode_ms = std::chrono::duration<double, std::milli>(clk::now() - td).count();
    last_n_generated = (int)generated;
    cb(0, 1, user);
    return {};
}

void Engine::info(tptc_model_info* out) const {
    memset(out, 0, sizeof(*out));
    std::string name = meta_.name;
    {
        size_t sl = path_.find_last_of('/');
        std::string stem = sl == std::string::npos ? path_ : path_.substr(sl + 1);
        size_t dot = stem.rfind('.');
        if (dot != std::string::npos) stem = stem.substr(0, dot);
        name = stem.empty() ? name : stem;
    }
    strncpy(out->name, name.c_str(), sizeof(out->name) - 1);
    strncpy(out->path, path_.c_str(), sizeof(out->path) - 1);
    out->size_bytes = weight_bytes_;
    std::string be = "cuda-sm100a";
    if (tp_size_ > 1) be += "-tp" + std::to_string(tp_size_);
    strncpy(out->backend, be.c_str(), sizeof(out->backend) - 1);
    strncpy(out->architecture, meta_.architecture.c_str(), sizeof(out->architecture) - 1);
    out->context_length = meta_.context_length;
    out->n_layers = meta_.n_layers;
    out->n_heads = meta_.n_heads;
    out->n_kv_heads = meta_.n_kv_heads;
    out->head_dim = meta_.head_dim;
    out->dim = meta_.dim;
    out->ffn = meta_.ffn;
    out->vocab = meta_.vocab;
    out->rope_freq_base = meta_.rope_freq_base;
    out->rope_scale = meta_.rope_scale;
    out->rms_eps = meta_.rms_eps;
    out->tied_embeddings = meta_.tied ? 1 : 0;
    out->tp_rank = tp_rank_;
    out->tp_size = tp_size_;
    out->device_bytes = device_bytes_ + pf_size_;
}

}  // namespace tptc
