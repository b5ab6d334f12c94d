// cuda_ffi.rs -- Rust declarations of libtptc's C ABI (include/tptc.h), for
// src-tauri/src/engine/cuda_ffi.rs in tpt-spark.
//
// Not compiled here: there is no cargo or rustc on the machines this repository is built and
// tested on.  tests/test_rust_ffi.py checks this file against include/tptc.h on every CPU
// test run: the same functions, the same parameter counts and the same struct fields, in the
// same order.
//
// Every function returns an int status (0 = ok, < 0 = one of the TPTC_ERR_* codes) unless it
// says otherwise; tptc_last_error(ctx) gives the message.  Device pointers are plain
// pointers (`*const c_void` / `*mut f32` ...); `stream` is a cudaStream_t or null (the legacy
// default stream).
#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_int, c_void};

pub const TPTC_OK: c_int = 0;
pub const TPTC_ERR_ARG: c_int = -1;
pub const TPTC_ERR_CUDA: c_int = -2;
pub const TPTC_ERR_IO: c_int = -3;
pub const TPTC_ERR_FORMAT: c_int = -4;
pub const TPTC_ERR_UNSUPPORTED: c_int = -5;
pub const TPTC_ERR_STATE: c_int = -6;
pub const TPTC_ERR_NCCL: c_int = -7;
pub const TPTC_ERR_OOM: c_int = -8;
pub const TPTC_ERR_CANCELLED: c_int = -9;
pub const TPTC_ERR_TIMEOUT: c_int = -10;

pub const TPTC_TYPE_F32: c_int = 0;
pub const TPTC_TYPE_F16: c_int = 1;
pub const TPTC_TYPE_Q4_0: c_int = 2;
pub const TPTC_TYPE_Q4_1: c_int = 3;
pub const TPTC_TYPE_Q5_0: c_int = 6;
pub const TPTC_TYPE_Q5_1: c_int = 7;
pub const TPTC_TYPE_Q8_0: c_int = 8;
pub const TPTC_TYPE_Q2_K: c_int = 10;
pub const TPTC_TYPE_Q3_K: c_int = 11;
pub const TPTC_TYPE_Q4_K: c_int = 12;
pub const TPTC_TYPE_Q5_K: c_int = 13;
pub const TPTC_TYPE_Q6_K: c_int = 14;

pub const TPTC_SHARD_Q: c_int = 0;
pub const TPTC_SHARD_K: c_int = 1;
pub const TPTC_SHARD_V: c_int = 2;
pub const TPTC_SHARD_O: c_int = 3;
pub const TPTC_SHARD_GATE: c_int = 4;
pub const TPTC_SHARD_UP: c_int = 5;
pub const TPTC_SHARD_DOWN: c_int = 6;

pub const TPTC_FUSED_NEVER: c_int = 0;
pub const TPTC_FUSED_AUTO: c_int = 1;
pub const TPTC_FUSED_ALWAYS: c_int = 2;

/// Opaque engine context (one per GPU; one host thread at a time).
#[repr(C)]
pub struct tptc_ctx {
    _private: [u8; 0],
}

/// Opaque weight matrix in the engine's device layout (kernel-level entry points).
#[repr(C)]
pub struct tptc_matrix {
    _private: [u8; 0],
}

/// ModelInfo (engine/mod.rs:85-92) plus the GGUF metadata the forward pass uses.
#[repr(C)]
pub struct tptc_model_info {
    pub name: [c_char; 256],
    pub path: [c_char; 1024],
    pub size_bytes: u64,
    pub backend: [c_char; 64],
    pub architecture: [c_char; 32],
    pub context_length: u32,
    pub n_layers: u32,
    pub n_heads: u32,
    pub n_kv_heads: u32,
    pub head_dim: u32,
    pub dim: u32,
    pub ffn: u32,
    pub vocab: u32,
    pub rope_freq_base: f32,
    pub rope_scale: f32,
    pub rms_eps: f32,
    pub tied_embeddings: u32,
    pub tp_rank: u32,
    pub tp_size: u32,
    pub device_bytes: u64,
}

/// InferenceParams (engine/mod.rs:35-46) without the prompt text (the caller tokenises).
#[repr(C)]
pub struct tptc_infer_params {
    pub max_tokens: u32,
    pub temperature: f32,
    pub top_p: f32,
    pub repeat_penalty: f32,
    pub seed: u64,
    pub eos_token_id: i64,
}

/// Token callback: once per token with done = 0, then once with done = 1 (also on
/// cancellation); return non-zero to cancel.
pub type tptc_token_cb = extern "C" fn(token: u32, done: c_int, user: *mut c_void) -> c_int;
/// Load progress: (tensors uploaded, total tensors).
pub type tptc_progress_cb = extern "C" fn(done: u32, total: u32, user: *mut c_void);

#[link(name = "tptc")]
extern "C" {
    // ---------------------------------------------------------------- lifecycle
    pub fn tptc_create(device: c_int, tp_rank: c_int, tp_size: c_int, nccl_uid: *const c_void,
                       out: *mut *mut tptc_ctx) -> c_int;
    pub fn tptc_nccl_unique_id(out128: *mut c_void) -> c_int;
    pub fn tptc_tp_shard(which: c_int, n_heads: c_int, n_kv_heads: c_int, head_dim: c_int, dim: c_int,
                         ffn: c_int, rank: c_int, size: c_int, r0: *mut c_int, r1: *mut c_int,
                         k0: *mut c_int, k1: *mut c_int) -> c_int;
    pub fn tptc_destroy(ctx: *mut tptc_ctx);
    pub fn tptc_last_error(ctx: *const tptc_ctx) -> *const c_char;
    pub fn tptc_version() -> *const c_char;
    pub fn tptc_device_count() -> c_int;
    pub fn tptc_set_kv_dtype(ctx: *mut tptc_ctx, ggml_type: c_int) -> c_int;
    pub fn tptc_set_prefill_gemm_min(ctx: *mut tptc_ctx, min_tokens: c_int) -> c_int;
    pub fn tptc_set_prefill_fused(ctx: *mut tptc_ctx, mode: c_int) -> c_int;
    pub fn tptc_set_tp_wait_polls(ctx: *mut tptc_ctx, polls: u32) -> c_int;
    pub fn tptc_load_gguf(ctx: *mut tptc_ctx, path: *const c_char, progress: Option<tptc_progress_cb>,
                          user: *mut c_void) -> c_int;
    pub fn tptc_unload(ctx: *mut tptc_ctx) -> c_int;
    pub fn tptc_is_loaded(ctx: *const tptc_ctx) -> c_int;
    pub fn tptc_get_model_info(ctx: *const tptc_ctx, out: *mut tptc_model_info) -> c_int;

    // ------------------------------------------------------------- forward pass
    pub fn tptc_kv_reset(ctx: *mut tptc_ctx) -> c_int;
    pub fn tptc_kv_prefix_len(ctx: *const tptc_ctx, ids: *const u32, n: c_int) -> c_int;
    pub fn tptc_kv_truncate(ctx: *mut tptc_ctx, n: c_int) -> c_int;
    pub fn tptc_kv_len(ctx: *const tptc_ctx) -> c_int;
    pub fn tptc_common_prefix_len(cached: *const u32, n_cached: c_int, ids: *const u32, n: c_int) -> c_int;
    pub fn tptc_prefill(ctx: *mut tptc_ctx, ids: *const u32, n: c_int, start_pos: c_int,
                        last_logits: *mut f32) -> c_int;
    pub fn tptc_decode(ctx: *mut tptc_ctx, id: u32, pos: c_int, logits: *mut f32, argmax: *mut u32) -> c_int;
    pub fn tptc_decode_greedy(ctx: *mut tptc_ctx, id: u32, pos: c_int, n: c_int, out_ids: *mut u32) -> c_int;
    pub fn tptc_infer(ctx: *mut tptc_ctx, prompt: *const u32, n: c_int, params: *const tptc_infer_params,
                      on_token: tptc_token_cb, user: *mut c_void) -> c_int;
    pub fn tptc_last_device_ms(ctx: *const tptc_ctx, ms: *mut f64) -> c_int;
    pub fn tptc_decode_kernels(ctx: *const tptc_ctx) -> c_int;
    pub fn tptc_last_timing(ctx: *const tptc_ctx, prefill_ms: *mut f64, decode_ms: *mut f64,
                            n_prompt: *mut c_int, n_generated: *mut c_int) -> c_int;
    pub fn tptc_debug_trace(ctx: *mut tptc_ctx, id: u32, pos: c_int, trace: *mut f32) -> c_int;

    // ------------------------------------------------- kernel-level entry points
    pub fn tptc_dequant(ggml_type: c_int, d_blocks: *const c_void, n: i64, d_out: *mut f32,
                        stream: *mut c_void) -> c_int;
    pub fn tptc_quant_q8k(d_x: *const f32, k: i64, d_out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn tptc_quant_q80(d_x: *const f32, k: i64, d_out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn tptc_matrix_create(ggml_type: c_int, raw: *const c_void, raw_on_device: c_int, n: c_int, k: c_int,
                              out: *mut *mut tptc_matrix) -> c_int;
    pub fn tptc_matrix_destroy(m: *mut tptc_matrix);
    pub fn tptc_matrix_bytes(m: *const tptc_matrix) -> i64;
    pub fn tptc_gemv(m: *const tptc_matrix, d_x: *const f32, d_y: *mut f32, stream: *mut c_void) -> c_int;
    pub fn tptc_matrix_dequant_f16(m: *const tptc_matrix, d_out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn tptc_block_dots(m: *const tptc_matrix, d_x: *const f32, d_isum: *mut i32, d_msum: *mut i32,
                           stream: *mut c_void) -> c_int;
    pub fn tptc_sample(d_logits: *const f32, vocab: c_int, d_counts: *mut c_int, penalty: f32, temperature: f32,
                       top_p: f32, seed: u64, d_step: *mut c_int, d_scratch: *mut f32, d_out_tok: *mut u32,
                       d_dbg: *mut u64, stream: *mut c_void) -> c_int;
    pub fn tptc_gemm_f16(d_a: *const c_void, d_b: *const c_void, d_c: *mut f32, m: c_int, n: c_int, k: c_int,
                         stream: *mut c_void) -> c_int;
    pub fn tptc_gemm_q(m: *const tptc_matrix, d_a: *const c_void, d_c: *mut f32, rows: c_int,
                       stream: *mut c_void) -> c_int;
    pub fn tptc_attn_prefill(d_q: *const c_void, d_kcache: *const c_void, d_vcache: *const c_void,
                             d_out: *mut c_void, t: c_int, start: c_int, n_heads: c_int, n_kv: c_int,
                             head_dim: c_int, max_seq: c_int, stream: *mut c_void) -> c_int;
    pub fn tptc_attn_decode_workspace_bytes(n_heads: c_int, n_kv: c_int, head_dim: c_int, max_seq: c_int) -> i64;
    pub fn tptc_attn_decode(d_q: *const f32, d_kraw: *const f32, d_kcache: *mut c_void, d_vcache: *const c_void,
                            kv_type: c_int, d_rope_cos: *const f32, d_rope_sin: *const f32, d_pos: *const c_int,
                            n_heads: c_int, n_kv: c_int, head_dim: c_int, max_seq: c_int, d_out: *mut f32,
                            d_workspace: *mut c_void, workspace_bytes: i64, stream: *mut c_void) -> c_int;
    // No counterpart in the reference: the same attention for hosts that cannot allocate
    // device memory (static per-device scratch; see include/tptc.h), and its status query.
    pub fn tptc_attn_decode_noalloc(d_q: *const f32, d_kraw: *const f32, d_kcache: *mut c_void,
                                    d_vcache: *const c_void, kv_type: c_int, d_rope_cos: *const f32,
                                    d_rope_sin: *const f32, d_pos: *const c_int, n_heads: c_int, n_kv: c_int,
                                    head_dim: c_int, max_seq: c_int, d_out: *mut f32,
                                    stream: *mut c_void) -> c_int;
    pub fn tptc_attn_decode_noalloc_status(stream: *mut c_void, out_code: *mut c_int) -> c_int;
}
