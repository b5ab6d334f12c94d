/*
 * tptc.h -- C ABI of the B200 (sm_100a) engine for tpt-spark's GGUF Llama/Mistral path.
 *
 * The engine replaces the reference's wgpu engine (src-tauri/src/engine/wgpu_engine.rs,
 * wgpu_loader.rs, wgpu_kvcache.rs, wgpu_ops.rs and the WGSL kernels in shaders/) behind the
 * LlmEngine trait (src-tauri/src/engine/mod.rs:62-82).  A Rust `engine/cuda_engine.rs`
 * binds these functions through `extern "C"`; Python binds them through ctypes.
 *
 * Conventions
 *   - Every function that can fail returns int: TPTC_OK (0) or a negative TPTC_ERR_*.
 *     tptc_last_error(ctx) gives the message of the last failure on that context
 *     (the anyhow::Error text the Rust side surfaces, commands.rs:59-62,291).
 *   - The caller owns every host pointer; the library owns all device memory it
 *     allocates.  Kernel-level test entry points take DEVICE pointers owned by the caller.
 *   - One host thread drives one context at a time (the reference serialises engine calls
 *     through EngineHandle = Arc<tokio::Mutex<..>>, engine/mod.rs:95).  Tensor parallelism
 *     uses one context per GPU, one thread or process per rank.
 *   - `stream` arguments are cudaStream_t passed as void* (NULL = legacy default stream).
 */
#ifndef TPTC_H
#define TPTC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(TPTC_BUILD)
#define TPTC_API __attribute__((visibility("default")))
#else
#define TPTC_API
#endif

#define TPTC_OK 0
#define TPTC_ERR_ARG (-1)         /* invalid argument / shape */
#define TPTC_ERR_CUDA (-2)        /* CUDA runtime error */
#define TPTC_ERR_IO (-3)          /* file open / read / mmap failure */
#define TPTC_ERR_FORMAT (-4)      /* malformed or truncated GGUF */
#define TPTC_ERR_UNSUPPORTED (-5) /* architecture, tensor type or shape not supported */
#define TPTC_ERR_STATE (-6)       /* call not valid in the current state (e.g. no model) */
#define TPTC_ERR_NCCL (-7)        /* NCCL failure */
#define TPTC_ERR_OOM (-8)         /* device allocation failed or over the configured cap */
#define TPTC_ERR_CANCELLED (-9)   /* the token callback asked to stop */
#define TPTC_ERR_TIMEOUT (-10)    /* a bounded device-side wait gave up */

/* GGML tensor type ids (GGUF tensor_info.type). */
#define TPTC_TYPE_F32 0
#define TPTC_TYPE_F16 1
#define TPTC_TYPE_Q4_0 2
#define TPTC_TYPE_Q4_1 3
#define TPTC_TYPE_Q5_0 6
#define TPTC_TYPE_Q5_1 7
#define TPTC_TYPE_Q8_0 8
#define TPTC_TYPE_Q2_K 10
#define TPTC_TYPE_Q3_K 11
#define TPTC_TYPE_Q4_K 12
#define TPTC_TYPE_Q5_K 13
#define TPTC_TYPE_Q6_K 14

typedef struct tptc_ctx tptc_ctx;
typedef struct tptc_matrix tptc_matrix;

/* ModelInfo (engine/mod.rs:85-92) plus the GgufMeta fields the forward pass uses
 * (engine/wgpu_loader.rs:41-67). */
typedef struct {
    char name[256];
    char path[1024];
    uint64_t size_bytes;      /* bytes of tensor data uploaded (wgpu_loader.rs total_bytes) */
    char backend[64];         /* "cuda-sm100a" or "cuda-sm100a-tpN" */
    char architecture[32];
    uint32_t context_length, n_layers, n_heads, n_kv_heads, head_dim, dim, ffn, vocab;
    float rope_freq_base, rope_scale, rms_eps;
    uint32_t tied_embeddings;
    uint32_t tp_rank, tp_size;
    uint64_t device_bytes;    /* device memory held by this context */
} tptc_model_info;

/* InferenceParams (engine/mod.rs:35-46) minus the prompt text: the caller tokenises
 * (tokenizer.json beside the .gguf, wgpu_engine.rs:892-906) and passes ids. */
typedef struct {
    uint32_t max_tokens;
    float temperature;        /* below 1e-7: greedy (LogitsProcessor::new takes it as None) */
    float top_p;              /* >= 1: no nucleus filter */
    float repeat_penalty;     /* 1: off (candle_engine.rs:87-101) */
    uint64_t seed;            /* sampling seed (the reference uses LogitsProcessor::new(42, ..)) */
    int64_t eos_token_id;     /* < 0: never stop on a token (find_eos_token, :908-913) */
} tptc_infer_params;

/* Called once per generated token with done=0, then once with done=1 (token 0), also on
 * cancellation -- the TokenEvent protocol of wgpu_engine.rs:297-300,332.  Return non-zero
 * to cancel; tptc_infer then emits done=1 and returns TPTC_ERR_CANCELLED. */
typedef int (*tptc_token_cb)(uint32_t token, int done, void* user);
/* on_progress(done, total) after each tensor upload (wgpu_loader.rs:185). */
typedef void (*tptc_progress_cb)(uint32_t done, uint32_t total, void* user);

/* ------------------------------------------------------------------ lifecycle */

/* Replaces WgpuEngine::new + GpuContext::try_init (wgpu_engine.rs:52-66,
 * wgpu_context.rs:22-97).  device: CUDA ordinal.  tp_size 1: single GPU (nccl_uid NULL).
 * tp_size > 1: nccl_uid points at the 128-byte ncclUniqueId rank 0 made with
 * tptc_nccl_unique_id and shared with the other ranks. */
TPTC_API int tptc_create(int device, int tp_rank, int tp_size, const void* nccl_uid, tptc_ctx** out);
TPTC_API int tptc_nccl_unique_id(void* out128);

/* Megatron shard of one weight for rank `rank` of `size` (host only, no device): the rows
 * [*r0, *r1) and input columns [*k0, *k1) of the full [N x K] matrix the loader keeps.
 * Column-parallel q / k / v (by heads) and gate / up (by ffn rows); row-parallel o (by the
 * heads' columns) and down (by ffn columns).  The reference has no tensor parallelism (one
 * wgpu device, wgpu_engine.rs:62-124); this is the north_star's sharding.  Returns
 * TPTC_ERR_UNSUPPORTED when the model does not split evenly (kv heads, or whole 256-blocks of
 * the row-parallel K slices). */
enum {
    TPTC_SHARD_Q = 0, TPTC_SHARD_K = 1, TPTC_SHARD_V = 2, TPTC_SHARD_O = 3,
    TPTC_SHARD_GATE = 4, TPTC_SHARD_UP = 5, TPTC_SHARD_DOWN = 6
};
TPTC_API int tptc_tp_shard(int which, int n_heads, int n_kv_heads, int head_dim, int dim, int ffn, int rank, int size,
                           int* r0, int* r1, int* k0, int* k1);
TPTC_API void tptc_destroy(tptc_ctx* ctx);
TPTC_API const char* tptc_last_error(const tptc_ctx* ctx);
/* Library version string and the number of CUDA devices (0 without a GPU). */
TPTC_API const char* tptc_version(void);
TPTC_API int tptc_device_count(void);

/* Element type of the KV cache, set before tptc_load_gguf: TPTC_TYPE_F16 (default: half the
 * bytes per decode step) or TPTC_TYPE_F32 (the precision of the reference's candle path,
 * wgpu_kvcache.rs:37 also stores f32). */
TPTC_API int tptc_set_kv_dtype(tptc_ctx* ctx, int ggml_type);
/* Prefill path selection (no counterpart in the reference, which prefills token by token on
 * the GPU, wgpu_engine.rs:252-261, and in one batched forward on the CPU,
 * candle_engine.rs:272-281).  Prompts of at least min_tokens tokens run batched: dense fp16
 * weights per layer on the tcgen05 GEMM and causal tensor-core attention, activations in fp16
 * (logits within fp16 rounding of the integer-dot path).  Shorter prompts, every prompt when
 * min_tokens <= 0, and every prompt with an f32 KV cache go token by token through the decode
 * step (bit-identical to decoding them).  Default 16; may be changed at any time. */
TPTC_API int tptc_set_prefill_gemm_min(tptc_ctx* ctx, int min_tokens);
/* How the batched prefill contracts Q4_K / Q6_K / Q8_0 weights: with the fused-dequant GEMM
 * (blocks expanded to fp16 in shared memory, tptc_gemm_q) or by expanding the matrix to fp16
 * in HBM first and running the fp16 GEMM.  TPTC_FUSED_AUTO (default) picks per matrix and
 * chunk with a wave model of both (the fused GEMM wins for short chunks of wide matrices);
 * NEVER and ALWAYS force one path.  The fused expansion rounds the Q4_K / Q6_K scale product
 * to fp16 before applying the code, so its weights are within one fp16 rounding of the
 * two-pass ones (Q8_0: identical). */
enum { TPTC_FUSED_NEVER = 0, TPTC_FUSED_AUTO = 1, TPTC_FUSED_ALWAYS = 2 };
TPTC_API int tptc_set_prefill_fused(tptc_ctx* ctx, int mode);
/* Tensor parallelism (no counterpart in the one-device reference): how many reads of a
 * peer's inbox word a decode kernel makes before it gives up on a rank that does not arrive
 * (the step then fails with TPTC_ERR_TIMEOUT instead of waiting for ever).  0 (default) keeps
 * the library's bound of 2^22 reads (seconds); a smaller bound makes a stalled peer show up
 * sooner.  Set before tptc_load_gguf. */
TPTC_API int tptc_set_tp_wait_polls(tptc_ctx* ctx, uint32_t polls);

/* LlmEngine::load (mod.rs:66-70) -> load_gguf_to_vram (wgpu_loader.rs:87-201): mmap the
 * file, parse GGUF v3, check bounds, stream every tensor through pinned staging with
 * cudaMemcpyAsync, repack to the device layout, build the KV cache and rope table.
 * Architectures llama, mistral, qwen2 (q / k / v biases, RoPE on head halves), phi3 (fused
 * attn_qkv and ffn_up, RoPE on head halves) and gemma (GEGLU, embeddings times sqrt(dim)); a
 * model with {arch}.expert_count > 1 has mixture-of-experts layers wherever
 * blk.N.ffn_gate_inp.weight exists (experts stacked as ffn_*_exps or one tensor each as
 * ffn_*.E, an optional shared expert ffn_*_shexp, an F32 / F16 router; one GPU only); weight
 * types F16, Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K; anything else
 * TPTC_ERR_UNSUPPORTED. */
TPTC_API int tptc_load_gguf(tptc_ctx* ctx, const char* path, tptc_progress_cb progress, void* user);
/* LlmEngine::unload / is_loaded / model_info (mod.rs:71-73, wgpu_engine.rs:126-147). */
TPTC_API int tptc_unload(tptc_ctx* ctx);
TPTC_API int tptc_is_loaded(const tptc_ctx* ctx);
TPTC_API int tptc_get_model_info(const tptc_ctx* ctx, tptc_model_info* out);

/* ------------------------------------------------------------ forward pass */

/* KvCache::reset (wgpu_kvcache.rs:55-58). */
TPTC_API int tptc_kv_reset(tptc_ctx* ctx);
/* KvCache::common_prefix_len against the token ids resident in the cache
 * (wgpu_kvcache.rs:63-69); returns the length (>= 0) or an error. */
TPTC_API int tptc_kv_prefix_len(const tptc_ctx* ctx, const uint32_t* ids, int n);
/* Keep only the first n positions of the KV cache (n <= tptc_kv_len): rewinds a turn. */
TPTC_API int tptc_kv_truncate(tptc_ctx* ctx, int n);
/* Number of positions resident in the KV cache. */
TPTC_API int tptc_kv_len(const tptc_ctx* ctx);
/* The comparison KvCache::common_prefix_len performs (wgpu_kvcache.rs:63-69), on two id
 * sequences; host-only, needs no device. */
TPTC_API int tptc_common_prefix_len(const uint32_t* cached, int n_cached, const uint32_t* ids, int n);

/* Batched prefill of ids[0..n) at positions start_pos.. (replaces the per-token prefill
 * loop of wgpu_engine.rs:252-261 and candle's forward(&input, 0), candle_engine.rs:272-281).
 * start_pos must equal tptc_kv_len().  last_logits (host, [vocab] f32) may be NULL. */
TPTC_API int tptc_prefill(tptc_ctx* ctx, const uint32_t* ids, int n, int start_pos, float* last_logits);
/* One decode step of token `id` at position `pos` (run_forward_pass, wgpu_engine.rs:339-490).
 * logits (host, [vocab] f32) and argmax (host) may each be NULL. */
TPTC_API int tptc_decode(tptc_ctx* ctx, uint32_t id, int pos, float* logits, uint32_t* argmax);
/* n greedy steps chained on the device: the argmax of each step is the next step's token,
 * starting from `id` at `pos`; out_ids (host, n entries) receives the n argmax tokens. */
TPTC_API int tptc_decode_greedy(tptc_ctx* ctx, uint32_t id, int pos, int n, uint32_t* out_ids);

/* LlmEngine::infer (mod.rs:76-81, gpu_infer wgpu_engine.rs:165-334) over token ids:
 * truncation to context_length - max_tokens, prefix reuse, batched prefill, repeat
 * penalty, greedy or temperature/top-p sampling, EOS / max_tokens / context stops, and
 * the on_token protocol above. */
TPTC_API int tptc_infer(tptc_ctx* ctx, const uint32_t* prompt, int n, const tptc_infer_params* params,
                        tptc_token_cb on_token, void* user);
/* Device time (CUDA events on the context's stream) of the last tptc_prefill or
 * tptc_decode_greedy call, in milliseconds. */
TPTC_API int tptc_last_device_ms(const tptc_ctx* ctx, double* ms);
/* Kernel launches in one decode step (the kernel nodes of the step's CUDA graph), or an error
 * code when no model is loaded. */
TPTC_API int tptc_decode_kernels(const tptc_ctx* ctx);
/* Wall-clock phases of the last tptc_infer call in milliseconds (wgpu_engine.rs:320-330). */
TPTC_API int tptc_last_timing(const tptc_ctx* ctx, double* prefill_ms, double* decode_ms, int* n_prompt,
                              int* n_generated);

/* Test hook: one decode step (as tptc_decode, outside the CUDA graph) that also copies, for
 * every layer l, q after RoPE, the attention output and the residual stream into rows 3l,
 * 3l+1, 3l+2 of trace (host, [3 * n_layers][dim] f32), for layer-by-layer parity checks. */
TPTC_API int tptc_debug_trace(tptc_ctx* ctx, uint32_t id, int pos, float* trace);

/* ------------------------------------------------ kernel-level entry points */
/* Device pointers owned by the caller.  These expose each hot-path kernel for parity tests
 * and microbenchmarks; the forward pass uses the same kernels. */

/* Dequantise n elements of raw GGUF blocks to f32 (dequant_q4k/q6k/q8/f16.wgsl and the
 * reference's Q4_0 / Q5_0 / Q5_1 / Q2_K / Q3_K / Q5_K shaders, shaders/dequant_*.wgsl): every
 * TPTC_TYPE_* above, in gguf-py's layouts and rounding (bit-exact).  n is a multiple of the
 * type's block (32 or 256 elements). */
TPTC_API int tptc_dequant(int ggml_type, const void* d_blocks, int64_t n, float* d_out, void* stream);
/* Q8_K activation blocks (292 B each: f32 d, int8 qs[256], int16 bsums[16]) of x[k]. */
TPTC_API int tptc_quant_q8k(const float* d_x, int64_t k, void* d_out, void* stream);
/* Q8_0 activation blocks (34 B each: f16 d, int8 qs[32]) of x[k]. */
TPTC_API int tptc_quant_q80(const float* d_x, int64_t k, void* d_out, void* stream);

/* A weight matrix [N out x K in] in the device layout the forward pass uses, made from raw
 * GGUF bytes (host or device pointer; `raw_on_device` says which). */
TPTC_API int tptc_matrix_create(int ggml_type, const void* raw, int raw_on_device, int N, int K,
                                tptc_matrix** out);
TPTC_API void tptc_matrix_destroy(tptc_matrix* m);
/* Bytes the matrix occupies on the device (the algorithmic bytes of one GEMV over it). */
TPTC_API int64_t tptc_matrix_bytes(const tptc_matrix* m);
/* y[N] = W . x with candle QMatMul semantics (x quantised to Q8_K / Q8_0 on the device; F16
 * in f32) -- gemm.wgsl + dequant_*.wgsl fused.  The matrix holds the scratch of its launches:
 * calls on the same matrix must not overlap on the GPU. */
TPTC_API int tptc_gemv(const tptc_matrix* m, const float* d_x, float* d_y, void* stream);
/* The matrix expanded to dense row-major fp16 [N x K] on the device (the prefill GEMM's B
 * operand): each value the GGUF dequantisation (dequant_*.wgsl semantics, gguf-py order)
 * rounded to nearest fp16. */
TPTC_API int tptc_matrix_dequant_f16(const tptc_matrix* m, void* d_out, void* stream);
/* Per (row, super-block) integer sums of the same kernel: isum = sum_j sc_j*dot_j,
 * msum = sum_j m_j*bsum_j (Q4_K, Q5_K; not written otherwise; d_msum may be NULL);
 * [N, K/256] for k-quants, [N, K/32] for Q4_0 / Q5_0 / Q8_0 (candle's per-block sumi). */
TPTC_API int tptc_block_dots(const tptc_matrix* m, const float* d_x, int32_t* d_isum, int32_t* d_msum,
                             void* stream);

/* The engine's next-token selection on the device (infer's sampling step), as kernels on
 * `stream` (their 36 KB work area is allocated and freed stream-ordered for the call):
 * logits[vocab] with the repeat penalty applied once per context occurrence (counts[vocab],
 * candle_engine.rs:87-101; the picked token's count is incremented), then argmax when
 * temperature is below 1e-7 (ties to the highest index), else softmax(x / temperature), the top-p
 * nucleus in (0, 1) (candle sample_topp's kept set, computed exactly in fixed point) and one
 * SplitMix64 draw of (seed, *step) (*step incremented).  scratch: [vocab] floats.  dbg
 * (nullable): [3] u64 = kept-set cut (fp32 bit pattern of the smallest kept exp(x - max)),
 * kept mass, total mass, both in units of 2^-40.  counts and step may be null. */
TPTC_API int tptc_sample(const float* d_logits, int vocab, int* d_counts, float penalty, float temperature,
                         float top_p, uint64_t seed, int* d_step, float* d_scratch, uint32_t* d_out_tok,
                         uint64_t* d_dbg, void* stream);
/* Prefill GEMM on the tensor cores: C[M x N] (f32, row-major) = A[M x K] . B[N x K]^T with A
 * and B row-major fp16 (16-byte aligned), K a multiple of 64 -- the prompt-wide replacement of
 * gemm.wgsl's per-token M = 1 products. */
TPTC_API int tptc_gemm_f16(const void* d_a, const void* d_b, float* d_c, int M, int N, int K, void* stream);
/* The prefill GEMM with the weight dequantisation fused in: C[M x N] (f32) = A[M x K] . W^T
 * with A row-major fp16 (16-byte aligned) and W a Q4_K / Q6_K / Q8_0 matrix (tptc_matrix,
 * N x K): the quantised blocks reach shared memory by TMA and are expanded there to fp16. */
TPTC_API int tptc_gemm_q(const tptc_matrix* m, const void* d_a, float* d_c, int M, void* stream);

/* Causal GQA attention of a prompt chunk on the tensor cores (the prefill replacement of
 * attention.wgsl's per-token passes, :31-170, run once per prompt token by
 * wgpu_engine.rs:254-261).  Query rows t = 0..T-1 sit at positions start + t and attend to
 * cache positions 0 .. start + t (the chunk's own keys already in the cache); head h reads kv
 * head h / (n_heads / n_kv); scale 1/sqrt(head_dim).  All fp16, device pointers:
 *   d_q [T][n_heads][head_dim] (rotated), d_kcache / d_vcache [n_kv][max_seq][head_dim],
 *   d_out [T][n_heads][head_dim].
 * head_dim 64, 96 or 128; start + T <= max_seq. */
TPTC_API int tptc_attn_prefill(const void* d_q, const void* d_kcache, const void* d_vcache, void* d_out, int T,
                               int start, int n_heads, int n_kv, int head_dim, int max_seq, void* stream);

/* GQA attention of one query position, the decode step of attention.wgsl's three passes
 * (scores :31-58, softmax :73-135, P.V :152-170; dispatched from wgpu_engine.rs:666-726).
 *   d_q [n_heads * head_dim], d_kraw [n_kv * head_dim]: q and this position's key before RoPE;
 *     both are rotated (candle rope_i) with d_rope_cos / d_rope_sin [max_seq][head_dim / 2].
 *   d_kcache, d_vcache [n_kv][max_seq][head_dim] of kv_type (TPTC_TYPE_F16 or TPTC_TYPE_F32):
 *     the rotated key is written to d_kcache at position *d_pos; V at *d_pos must be present.
 *   d_pos: device int p, 0 <= p < max_seq; keys and values 0..p are attended.
 *   d_out [n_heads * head_dim] = softmax(q.k / sqrt(head_dim)) . V, query head h reading kv
 *     head h / (n_heads / n_kv).
 * Limits: n_heads a multiple of n_kv with at most 8 query heads per kv head; head_dim 64,
 * 96 or 128.  d_workspace holds tptc_attn_decode_workspace_bytes() bytes
 * (for the current device) and must be zero before its first use; each call leaves it ready
 * for the next (its split counters return to zero, the partial results are overwritten).  Its
 * first int receives a nonzero TPTC_ERR_* code if the kernel found p outside [0, max_seq)
 * (nothing is written then) or a copy wait timed out.  Calls that may overlap on the GPU need
 * separate workspaces. */
TPTC_API int64_t tptc_attn_decode_workspace_bytes(int n_heads, int n_kv, int head_dim, int max_seq);
TPTC_API int tptc_attn_decode(const float* d_q, const float* d_kraw, void* d_kcache, const void* d_vcache,
                              int kv_type, const float* d_rope_cos, const float* d_rope_sin, const int* d_pos,
                              int n_heads, int n_kv, int head_dim, int max_seq, float* d_out, void* d_workspace,
                              int64_t workspace_bytes, void* stream);

/* No counterpart in the reference: tptc_attn_decode for callers that cannot allocate device
 * memory -- a host whose device memory is all reserved up front by its own pool or another
 * framework's caching allocator, or a decode loop that must not call cudaMalloc / cudaFree
 * because they can synchronise the device.  Same arguments and results, minus the
 * workspace: the scratch is a static device array of 1 MiB per device (split counters, error
 * word and split partials; the partials take splits * n_heads * (head_dim + 2) * 4 bytes).
 * Sizes whose scratch exceeds 1 MiB are rejected with TPTC_ERR_ARG and a message giving both
 * sizes.  The call makes no cudaMalloc, cudaFree or other allocating call.  Its first call on
 * a device does a one-time set-up with that device current: it looks the array's device
 * address up (cudaGetSymbolAddress) and zeroes the array on `stream`, waiting for that; make
 * this first call before any stream capture.  Every call then zeroes the error word and the
 * split counters on `stream` before its launch, so a launch that was flagged or whose bounded
 * wait gave up never affects the next call.  The array is shared by all calls on a device:
 * calls that may overlap on the GPU (different streams without ordering, several host
 * threads) race on it and give wrong results, so callers serialise them.  A position outside
 * the cache or a timed-out wait leaves d_out unwritten; tptc_attn_decode_noalloc_status
 * reports it. */
TPTC_API int tptc_attn_decode_noalloc(const float* d_q, const float* d_kraw, void* d_kcache, const void* d_vcache,
                                      int kv_type, const float* d_rope_cos, const float* d_rope_sin,
                                      const int* d_pos, int n_heads, int n_kv, int head_dim, int max_seq,
                                      float* d_out, void* stream);
/* No counterpart in the reference: the outcome of the most recent tptc_attn_decode_noalloc
 * launch on the current device.  Waits for `stream`, then sets *out_code to the launch's
 * internal error word: 0 (completed), TPTC_ERR_ARG (its position was outside [0, max_seq),
 * nothing was written) or TPTC_ERR_TIMEOUT (a bounded wait gave up, d_out is incomplete).  A
 * nonzero word also re-zeroes the whole static array.  *out_code is 0 when no call has run on
 * this device.  Allocates nothing. */
TPTC_API int tptc_attn_decode_noalloc_status(void* stream, int* out_code);

#ifdef __cplusplus
}
#endif
#endif /* TPTC_H */
