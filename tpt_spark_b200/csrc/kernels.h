// kernels.h -- host launchers of the small kernels (quant.cu, attn_decode.cu, misc.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemv.cuh"

namespace tptc {

// quant.cu
cudaError_t launch_dequant_raw(int type, const void* blocks, int64_t n, float* out, cudaStream_t st);
cudaError_t launch_quant_q8k(const float* x, int64_t k, void* out, cudaStream_t st);
cudaError_t launch_quant_q80(const float* x, int64_t k, void* out, cudaStream_t st);
// nr raw GGUF rows (device, raw_row bytes apart) -> logical rows first_row.. of `m` in the
// tiled device layout (main / dplane already allocated).
cudaError_t launch_repack(const uint8_t* raw, int64_t raw_row, int nr, int first_row, const DevMatrix& m,
                          cudaStream_t st);
// Device-layout rows [row0, row0+rows) of `m` -> dense f16 [rows, K] (prefill operand).
// Rows [row0, row0 + rows) of m as dense fp16 rows: logical rows, or with `physical` the
// device (tile) order -- for a gate|up matrix, 4 gate rows then the 4 matching up rows.
cudaError_t launch_dequant_rows_f16(const DevMatrix& m, int row0, int rows, __half* out, cudaStream_t st,
                                    bool physical = false);

// attn_decode.cu
struct AttnDecodeParams {
    const float* q;        // [n_heads * hd] before RoPE (rotated on load)
    const float* kraw;     // [n_kv * hd] this position's key before RoPE
    void* kcache;          // this layer, [n_kv][max_seq][hd], fp16 (default) or f32; the CTA
                           // owning `pos` writes the rotated key there before reading tiles
    const void* vcache;    // V at `pos` already written by the QKV GEMV
    int kv_f32;
    const float* rope_cos;  // [max_seq][hd/2]
    const float* rope_sin;
    const int* pos;        // device scalar: the query position (keys 0..pos)
    float* out;            // [n_heads * hd]
    float* q_out;          // optional [n_heads * hd]: rotated q (test trace)
    float* partial;        // scratch [n_kv][splits][group][hd + 4]: m, l, 2 pad, acc
    int* counters;         // scratch [n_kv], zero between launches
    int n_heads, n_kv, hd, max_seq;
    int splits;            // grid splits per kv head (attn_decode_splits); the kernel uses
                           // min(splits, ceil(kv_len / 128)) of them
    int stages;            // filled by launch_attn_decode
    float scale;           // 1/sqrt(hd)
    int* err;
    // optional: the output also written as the next GEMV's prepared activation (gemv.cuh
    // ActLayout, act_nb 256-blocks over all heads); requires (n_heads / n_kv) * hd % 256 == 0
    uint8_t* act_out;
    ActLayout act;
    int act_transposed, act_nb;
    int rope_neox;  // 1: RoPE pairs element i with i + hd/2 (candle rope, qwen2); 0: rope_i pairs
};
int attn_decode_splits(int n_kv, int max_seq, int sm_count);
size_t attn_decode_partial_floats(int n_heads, int n_kv, int hd, int splits);
// nullptr when the kernel supports the shape, else the reason.
const char* attn_decode_shape_error(int n_heads, int n_kv, int hd, int max_seq);
// Scratch of one launch as one buffer (kernel-level entry points): byte offsets of the
// error word (0), the counters ([n_kv] int, zero between launches) and the partials.
struct AttnScratch {
    int splits;
    size_t counters, err, partial, total;
};
AttnScratch attn_scratch_layout(int n_heads, int n_kv, int hd, int max_seq, int sm_count);
cudaError_t launch_attn_decode(const AttnDecodeParams& p, cudaStream_t st, bool pdl);

// attn_noalloc.cu: static per-device scratch of tptc_attn_decode_noalloc (allocates nothing).
constexpr size_t kAttnNoAllocScratchBytes = size_t(1) << 20;
// Address of `device`'s static scratch (the current device); the first call per device looks
// it up and zeroes it on `st` (synchronously).
cudaError_t attn_noalloc_scratch(int device, cudaStream_t st, uint8_t** out);
// The error word the last launch on `device`'s static scratch left (0: none), read after
// `st` finishes; a nonzero word re-zeroes the whole array.
cudaError_t attn_noalloc_status(int device, cudaStream_t st, int* code);

// misc.cu
// x[dim] = dequantised row `tok` of token_embd (device layout), token read from *tok_ptr,
// times `scale` (gemma's sqrt(dim); 1 leaves the row as it is).
// `step` (optional): a counter the kernel increments once (the decode step, for TpLink epochs).
cudaError_t launch_embed_row(const DevMatrix& emb, const uint32_t* tok_ptr, float* x, cudaStream_t st, bool pdl,
                             int* step = nullptr, float scale = 1.f);
// argmax over logits[n] (ties -> highest index, candle sample_argmax); writes *out_tok;
// when next_tok/pos are non-null also stores the token as the next step's input and
// increments *pos (device-chained greedy decode).
cudaError_t launch_argmax(const float* logits, int n, uint32_t* out_tok, uint32_t* next_tok, int* pos,
                          uint32_t* history, cudaStream_t st, bool pdl);
// The same over a vocab-parallel lm_head: logits[n] are this rank's rows [row0, row0 + n);
// the ranks exchange their best (value, index) over the TpLink inboxes and all pick the same
// token (a peer that never arrives: TPTC_ERR_TIMEOUT in *err after link->wait_polls reads).
cudaError_t launch_argmax_tp(const float* logits, int n, int row0, const TpLink* link, int* err, uint32_t* out_tok,
                             uint32_t* next_tok, int* pos, uint32_t* history, cudaStream_t st, bool pdl);

// sample.cu: the next token from logits[vocab] on the device (one CTA): repeat penalty over
// the context counts, then argmax (temperature below 1e-7) or softmax(x / T), top-p and one seeded draw.
struct SampleParams {
    const float* logits;
    int vocab;
    int* counts;        // [vocab] occurrences of each token in the context (penalty); the
                        // sampled token's count is incremented; may be null (no penalty)
    float penalty;      // 1 = off
    float temperature;  // below 1e-7 (candle: no temperature): argmax, ties to the highest index
    float top_p;        // in (0, 1): nucleus; otherwise every token
    unsigned long long seed;
    int* step;          // draw counter (read, then incremented); null = draw 0
    float* scratch;     // [vocab]
    uint32_t* out_tok;
    uint32_t* next_tok;  // optional chaining, as argmax: next decode input, ++pos, history[pos]
    int* pos;
    uint32_t* history;
    unsigned long long* dbg;  // optional [3]: cut pattern, kept mass, total mass (2^-40 units)
    unsigned char* work;      // kSampleWorkBytes of device memory (histograms, per-CTA partials)
};
constexpr size_t kSampleWorkBytes = 36 * 1024;
// Vocabularies up to 262144 tokens (256 CTAs of 1024).
cudaError_t launch_sample(const SampleParams& p, cudaStream_t st, bool pdl);

cudaError_t kernels_init_device();

}  // namespace tptc
