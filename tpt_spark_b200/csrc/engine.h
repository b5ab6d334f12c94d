// engine.h -- the CUDA engine behind the C ABI: the counterpart of the reference's WgpuEngine
// (src-tauri/src/engine/wgpu_engine.rs) + GpuModel + KvCache (wgpu_kvcache.rs) + loader
// (wgpu_loader.rs), implementing LlmEngine's semantics (engine/mod.rs:62-82).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemv.cuh"
#include "gguf.h"
#include "tptc.h"

namespace tptc {

// GgufMeta (wgpu_loader.rs:41-67), the fields the dense Llama path uses.
struct ModelMeta {
    std::string architecture = "llama";
    std::string name;
    int context_length = 4096, n_layers = 0, n_heads = 0, n_kv_heads = 0, head_dim = 0, dim = 0, ffn = 0, vocab = 0;
    float rope_freq_base = 10000.f, rope_scale = 1.f, rms_eps = 1e-5f;
    bool tied = false;
    bool rope_neox = false;  // qwen2: RoPE pairs element i with i + head_dim / 2 (candle rope)
    bool qkv_bias = false;   // qwen2: f32 attn_q / attn_k / attn_v biases
    bool fused_qkv = false;      // phi3: one attn_qkv tensor, rows q | k | v
    bool fused_gate_up = false;  // phi3: one ffn_up tensor, rows gate | up
    bool geglu = false;          // gemma: GEGLU feed-forward (tanh-form gelu(gate) * up)
    float embd_scale = 1.f;      // gemma: embedding rows times sqrt(dim)
    // mixture of experts (wgpu_loader.rs:367-377): experts per MoE layer, chosen per token,
    // rows of each expert's gate / up (and down's K); shared-expert rows (0: none)
    int n_expert = 0, n_expert_used = 0, expert_ffn = 0, shared_ffn = 0;
};

struct LayerWeights {
    DevMatrix q, k, v, o, down;
    DevMatrix glu;  // fused ffn_gate | ffn_up (gemv.cuh): logical rows [0, ffn) gate, [ffn, 2 ffn) up
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    float* bq = nullptr;  // this rank's rows of the q / k / v biases (qwen2), or nullptr
    float* bk = nullptr;
    float* bv = nullptr;
    // mixture of experts (a layer with blk.N.ffn_gate_inp.weight): the router's raw rows
    // [n_expert][dim] (F32 or F16); every expert's gate|up and down matrix in the device layout,
    // expert e at eglu.main + e * eglu_stride (edown likewise); an optional shared expert in
    // glu / down (the dense layer's matrices)
    bool moe = false;
    const void* router = nullptr;
    int router_type = 0;
    DevMatrix eglu, edown;
    int64_t eglu_stride = 0, edown_stride = 0;
    bool shexp = false;
    std::vector<DevMatrix> eglu_all, edown_all;  // per expert (load-time bookkeeping)
};

struct Tp;  // tensor-parallel communicator (tp.cpp)

// KvCache::common_prefix_len (wgpu_kvcache.rs:63-69): leading ids shared by both sequences.
int common_prefix_len(const uint32_t* cached, int n_cached, const uint32_t* ids, int n);

class Engine {
   public:
    Engine(int device, int tp_rank, int tp_size);
    ~Engine();
    Status init(const void* nccl_uid);
    Status load(const std::string& path, tptc_progress_cb cb, void* user);
    void unload();
    bool loaded() const { return loaded_; }
    void info(tptc_model_info* out) const;

    Status kv_reset();
    int kv_len() const { return (int)cached_tokens_.size(); }
    void kv_truncate(int n) { cached_tokens_.resize(n); }
    // KV cache element type, chosen before load: fp16 (default) or f32 (candle's precision).
    Status set_kv_f32(bool f32) {
        if (loaded_) return Status{TPTC_ERR_STATE, "the KV cache type must be set before load"};
        kv_f32_ = f32;
        return {};
    }
    bool kv_f32() const { return kv_f32_; }
    // Prompts of at least n tokens take the batched tensor-core prefill (fp16 KV cache only);
    // shorter ones, or all when n <= 0, run token by token through the decode step.
    void set_prefill_gemm_min(int n) { prefill_gemm_min_ = n; }
    // When the batched prefill contracts quantised weights with the fused-dequant GEMM
    // (TPTC_FUSED_NEVER / AUTO / ALWAYS) instead of expanding each matrix to fp16 first.
    void set_prefill_fused(int mode) { prefill_fused_ = mode; }
    // Reads a tensor-parallel wait makes before it gives up (set before load; 0 = default).
    Status set_tp_wait_polls(uint32_t polls) {
        if (loaded_) return Status{TPTC_ERR_STATE, "the wait bound must be set before load"};
        tp_wait_polls_ = polls;
        return {};
    }
    bool prefill_uses_gemm(int n) const;
    int prefix_len(const uint32_t* ids, int n) const;

    Status prefill(const uint32_t* ids, int n, int start_pos, float* last_logits);
    Status decode(uint32_t id, int pos, float* logits, uint32_t* argmax);
    Status decode_greedy(uint32_t id, int pos, int n, uint32_t* out_ids);
    // Device next-token selection (sample.cu) over the last logits: sample_reset loads the
    // context's token counts (repeat penalty) and zeroes the draw counter; sample_logits picks
    // from logits_ (the kernel counts the pick); decode_sample = decode + sample_logits.
    Status sample_reset(const uint32_t* context, int n);
    Status sample_logits(const tptc_infer_params& p, uint32_t* out);
    Status enqueue_sample(const tptc_infer_params& p);  // kernel + token copy, no sync
    Status decode_sample(uint32_t id, int pos, const tptc_infer_params& p, uint32_t* out);
    Status infer(const uint32_t* prompt, int n, const tptc_infer_params& p, tptc_token_cb cb, void* user);

    double last_prefill_ms = 0, last_decode_ms = 0, last_device_ms = 0;
    int graph_kernels_ = 0;  // kernel launches in one decode step (nodes of the captured graph)
    int last_n_prompt = 0, last_n_generated = 0;
    std::string last_error;
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

   private:
    Status alloc_runtime();
    Status build_decode_graph(bool chained, cudaGraphExec_t* out);
    // trace (host, pinned or pageable; null in graphs): per layer l, rows 3l..3l+2 of width
    // dim receive q (after RoPE), the attention output and the residual stream x.
    Status enqueue_decode(cudaStream_t st, bool chained, float* trace = nullptr);

   public:
    // One decode step outside the graph, recording the per-layer trace above (test hook).
    Status debug_trace(uint32_t id, int pos, float* trace);

   private:
    // prefill.cu
    Status prefill_buffers(int chunk);
    Status enqueue_prefill_chunk(int T, int start);
    Status run_prefill_batched(const uint32_t* ids, int n, int start_pos, float* last_logits);
    Status check_err();
    Status sync();
    // Under a vocab-parallel lm_head every rank holds the logits of its rows; the full vector
    // (host copies, sampling) is an NCCL all-gather, made by every rank at the same calls.
    Status gather_logits();

    int device_, tp_rank_, tp_size_;
    int sm_count_ = 148;
    bool loaded_ = false;
    bool pdl_ = true;
    bool chain_ = false;  // single-GPU decode step as GEMV chains (TPTC_DECODE_CHAIN=1; default: one launch per GEMV)
    cudaStream_t stream_ = nullptr;
    ModelMeta meta_;
    std::string path_;
    uint64_t file_bytes_ = 0, weight_bytes_ = 0, device_bytes_ = 0;

    // device memory
    uint8_t* arena_ = nullptr;     // weights
    size_t arena_size_ = 0;
    uint8_t* rt_ = nullptr;        // runtime buffers (KV cache, activations, scratch)
    size_t rt_size_ = 0;
    std::vector<LayerWeights> layers_;
    DevMatrix embd_, output_;
    // lm_head rows this rank computes: all of them, or under tensor parallelism (vocab a
    // multiple of the rank count) rows [head_row0_, head_row0_ + head_rows_)
    int head_row0_ = 0, head_rows_ = 0;
    uint32_t tp_wait_polls_ = 0;  // bound of the tensor-parallel waits (0: the default)
    float* out_norm_ = nullptr;
    uint8_t* kv_ = nullptr;  // [L][2][n_kv_local][max_seq][hd], fp16 or f32
    bool kv_f32_ = false;
    size_t kv_elem_bytes() const { return kv_f32_ ? 4 : 2; }
    int max_seq_ = 0;
    int n_heads_l_ = 0, n_kv_l_ = 0;  // per-rank heads (TP)
    float* rope_cos_ = nullptr;
    float* rope_sin_ = nullptr;
    float* x_ = nullptr;        // residual stream [dim]
    float* x2_ = nullptr;       // its second buffer under tensor parallelism (gather target)
    float* qbuf_ = nullptr;     // [n_heads_l * hd] q before RoPE
    float* qrot_ = nullptr;     // [n_heads_l * hd] q after RoPE (written by attention, for traces)
    float* kraw_ = nullptr;     // [n_kv_l * hd] this step's k before RoPE
    float* attn_ = nullptr;     // [n_heads_l * hd]
    float* h_ = nullptr;        // [2 * ffn_l]: gate rows then up rows; MoE: the selected experts' and the shared expert's products
    float* moe_logits_ = nullptr;  // [n_expert] router logits
    int* moe_sel_ = nullptr;       // [n_expert_used] selected experts, ascending
    float* moe_w_ = nullptr;       // [n_expert_used] their routing weights
    float* moe_acc_ = nullptr;     // [dim] weighted sum of the experts' outputs
    int* moe_count_ = nullptr;     // routing kernel's ticket (kept at zero between launches)
    float* logits_ = nullptr;   // [vocab]
    uint32_t* tok_in_ = nullptr;
    uint32_t* tok_out_ = nullptr;
    uint32_t* history_ = nullptr;  // [max_seq]
    int* pos_ = nullptr;
    int* err_ = nullptr;
    int* step_ = nullptr;  // decode steps so far (tensor-parallel reduction epochs)
    uint8_t* act_ = nullptr;  // prepared GEMV activation (gemv_launch)
    int* chain_bar_ = nullptr;     // [L + 1][kChainMaxPhases] chain arrival counters
    int* sample_counts_ = nullptr;     // [vocab] context token counts (repeat penalty)
    float* sample_scratch_ = nullptr;  // [vocab]
    unsigned char* sample_work_ = nullptr;  // kSampleWorkBytes (the sampling kernels' histograms and partials)
    int* sample_step_ = nullptr;       // draws so far in this inference
    float* best_val_ = nullptr;    // [2 * SMs] per-CTA argmax partials of the lm_head chain
    int* best_idx_ = nullptr;
    float* attn_partial_ = nullptr;
    int* attn_counters_ = nullptr;
    int attn_splits_ = 1;
    // batched prefill: buffers allocated on demand for the chunk size (tokens)
    static constexpr int kPrefillChunk = 8192;
    int prefill_gemm_min_ = 16;
    int prefill_fused_ = TPTC_FUSED_AUTO;
    uint8_t* pf_ = nullptr;
    size_t pf_size_ = 0;
    int pf_chunk_ = 0;
    uint32_t* pf_ids_ = nullptr;  // [T] token ids
    float* pf_x_ = nullptr;       // [T][dim] residual stream
    __half* pf_xn_ = nullptr;     // [T][dim] normed activations (GEMM A operand)
    float* pf_qkv_ = nullptr;     // [T][(n_heads + 2 n_kv) hd] projection output
    __half* pf_q_ = nullptr;      // [T][n_heads hd] rotated queries
    __half* pf_o_ = nullptr;      // [T][n_heads hd] attention output
    __half* pf_h_ = nullptr;      // [T][ffn] silu(gate) * up
    __half* pf_w_ = nullptr;      // one layer matrix as dense fp16 (GEMM B operand)
    float* pf_part_ = nullptr;    // [T][dim] row-parallel partial sums (tensor parallel)
    // mixture of experts: the chunk's routing ([T][n_used] experts, ascending, and weights),
    // the chosen (token, expert) rows grouped by expert: token of each row, row of each
    // choice, gathered activations, gate|up products and down outputs; the shared expert's
    int* pf_rsel_ = nullptr;
    float* pf_rw_ = nullptr;
    int* pf_gidx_ = nullptr;
    int* pf_rowof_ = nullptr;
    __half* pf_ga_ = nullptr;
    __half* pf_gh_ = nullptr;
    float* pf_gy_ = nullptr;
    __half* pf_sh_h_ = nullptr;
    float* pf_sh_y_ = nullptr;

    // pinned host staging
    uint32_t* h_tok_ = nullptr;
    int* h_pos_ = nullptr;
    int* h_err_ = nullptr;

    cudaGraphExec_t graph_plain_ = nullptr, graph_chained_ = nullptr;
    cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
    std::vector<uint32_t> cached_tokens_;  // KvCache::cached_tokens (wgpu_kvcache.rs:21-23)
    std::unique_ptr<Tp> tp_;
};

}  // namespace tptc
