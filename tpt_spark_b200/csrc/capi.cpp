// capi.cpp -- extern "C" boundary (include/tptc.h).  Every entry point converts C++ state
// into an int status and keeps the message for tptc_last_error.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <new>
#include <string>

#include "engine.h"
#include "kernels.h"
#include "prefill.h"
#include "tp.h"
#include "tptc.h"

using tptc::Engine;
using tptc::Status;

struct tptc_ctx {
    Engine* eng = nullptr;
    std::string err;
};

struct tptc_matrix {
    tptc::DevMatrix m;
    uint8_t* mem = nullptr;
    int* err = nullptr;
    uint8_t* act = nullptr;  // the prepared activation of this matrix's GEMV launches
    int device = 0;
};

namespace {

thread_local std::string g_err;  // errors without a context (create, kernel-level calls)

int fail(tptc_ctx* c, const Status& s) {
    if (c) c->err = s.msg;
    else g_err = s.msg;
    return s.code;
}

int fail_code(tptc_ctx* c, int code, const std::string& m) { return fail(c, Status{code, m}); }

int cuda_fail(cudaError_t e, const char* what) {
    g_err = tptc::cuda_msg(e, what);
    return TPTC_ERR_CUDA;
}

}  // namespace

extern "C" {

TPTC_API const char* tptc_version(void) { return "tptc 0.1 (sm_100a)"; }

TPTC_API int tptc_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

TPTC_API int tptc_nccl_unique_id(void* out128) {
    if (!out128) return TPTC_ERR_ARG;
    return tptc::nccl_unique_id(out128);
}

TPTC_API int tptc_create(int device, int tp_rank, int tp_size, const void* nccl_uid, tptc_ctx** out) {
    if (!out) return TPTC_ERR_ARG;
    *out = nullptr;
    tptc_ctx* c = new (std::nothrow) tptc_ctx();
    if (!c) return TPTC_ERR_OOM;
    c->eng = new (std::nothrow) Engine(device, tp_rank, tp_size);
    if (!c->eng) {
        delete c;
        return TPTC_ERR_OOM;
    }
    Status s = c->eng->init(nccl_uid);
    if (!s.ok()) {
        g_err = s.msg;
        delete c->eng;
        delete c;
        return s.code;
    }
    *out = c;
    return TPTC_OK;
}

TPTC_API void tptc_destroy(tptc_ctx* ctx) {
    if (!ctx) return;
    delete ctx->eng;
    delete ctx;
}

TPTC_API const char* tptc_last_error(const tptc_ctx* ctx) { return ctx ? ctx->err.c_str() : g_err.c_str(); }

TPTC_API int tptc_set_kv_dtype(tptc_ctx* ctx, int ggml_type) {
    if (!ctx) return TPTC_ERR_ARG;
    if (ggml_type != TPTC_TYPE_F16 && ggml_type != TPTC_TYPE_F32)
        return fail_code(ctx, TPTC_ERR_UNSUPPORTED, "KV cache type must be F16 or F32");
    Status s = ctx->eng->set_kv_f32(ggml_type == TPTC_TYPE_F32);
    return s.ok() ? TPTC_OK : fail(ctx, s);
}

TPTC_API int tptc_tp_shard(int which, int n_heads, int n_kv_heads, int head_dim, int dim, int ffn, int rank, int size,
                           int* r0, int* r1, int* k0, int* k1) {
    if (!r0 || !r1 || !k0 || !k1) return TPTC_ERR_ARG;
    int a, b, c, d;
    if (!tptc::tp_shard(which, n_heads, n_kv_heads, head_dim, dim, ffn, rank, size, a, b, c, d))
        return TPTC_ERR_UNSUPPORTED;
    *r0 = a;
    *r1 = b;
    *k0 = c;
    *k1 = d;
    return TPTC_OK;
}

TPTC_API int tptc_set_prefill_gemm_min(tptc_ctx* ctx, int min_tokens) {
    if (!ctx) return TPTC_ERR_ARG;
    ctx->eng->set_prefill_gemm_min(min_tokens);
    return TPTC_OK;
}

TPTC_API int tptc_set_prefill_fused(tptc_ctx* ctx, int mode) {
    if (!ctx) return TPTC_ERR_ARG;
    if (mode != TPTC_FUSED_NEVER && mode != TPTC_FUSED_AUTO && mode != TPTC_FUSED_ALWAYS)
        return fail_code(ctx, TPTC_ERR_ARG, "prefill fused mode must be TPTC_FUSED_NEVER, AUTO or ALWAYS");
    ctx->eng->set_prefill_fused(mode);
    return TPTC_OK;
}

TPTC_API int tptc_set_tp_wait_polls(tptc_ctx* ctx, uint32_t polls) {
    if (!ctx) return TPTC_ERR_ARG;
    tptc::Status s = ctx->eng->set_tp_wait_polls(polls);
    return s.ok() ? TPTC_OK : fail_code(ctx, s.code, s.msg);
}

TPTC_API int tptc_load_gguf(tptc_ctx* ctx, const char* path, tptc_progress_cb progress, void* user) {
    if (!ctx || !path) return fail_code(ctx, TPTC_ERR_ARG, "null argument");
    Status s = ctx->eng->load(path, progress, user);
    return s.ok() ? TPTC_OK : fail(ctx, s);
}

TPTC_API int tptc_unload(tptc_ctx* ctx) {
    if (!ctx) return TPTC_ERR_ARG;
    ctx->eng->unload();
    return TPTC_OK;
}

TPTC_API int tptc_is_loaded(const tptc_ctx* ctx) { return ctx && ctx->eng->loaded() ? 1 : 0; }

TPTC_API int tptc_get_model_info(const tptc_ctx* ctx, tptc_model_info* out) {
    if (!ctx || !out) return TPTC_ERR_ARG;
    if (!ctx->eng->loaded()) return TPTC_ERR_STATE;
    ctx->eng->info(out);
    return TPTC_OK;
}

TPTC_API int tptc_kv_reset(tptc_ctx* ctx) {
    if (!ctx) return TPTC_ERR_ARG;
    Status s = ctx->eng->kv_reset();
    return s.ok() ? TPTC_OK : fail(ctx, s);
}

TPTC_API int tptc_kv_truncate(tptc_ctx* ctx, int n) {
    if (!ctx) return TPTC_ERR_ARG;
    if (n < 0 || n > ctx->eng->kv_len()) return fail_code(ctx, TPTC_ERR_ARG, "truncate length outside the cache");
    ctx->eng->kv_truncate(n);
    return TPTC_OK;
}

TPTC_API int tptc_kv_prefix_len(const tptc_ctx* ctx, const uint32_t* ids, int n) {
    if (!ctx || (n > 0 && !ids) || n < 0) return TPTC_ERR_ARG;
    return ctx->eng->prefix_len(ids, n);
}

TPTC_API int tptc_kv_len(const tptc_ctx* ctx) { return ctx ? ctx->eng->kv_len() : TPTC_ERR_ARG; }

TPTC_API int tptc_common_prefix_len(const uint32_t* cached, int n_cached, const uint32_t* ids, int n) {
    if (n_cached < 0 || n < 0 || (n_cached > 0 && !cached) || (n > 0 && !ids)) return TPTC_ERR_ARG;
    return tptc::common_prefix_len(cached, n_cached, ids, n);
}

TPTC_API int tptc_prefill(tptc_ctx* ctx, const uint32_t* ids, int n, int start_pos, float* last_logits) {
    if (!ctx || !ids) return fail_code(ctx, TPTC_ERR_ARG, "null argument");
    Status s = ctx->eng->prefill(ids, n, start_pos, last_logits);
    return s.ok() ? TPTC_OK : fail(ctx, s);
}

TPTC_API int tptc_decode(tptc_ctx* ctx, uint32_t id, int pos, float* logits, uint32_t* argmax) {
    if (!ctx) return TPTC_ERR_ARG;
    Status s = ctx->eng->decode(id, pos, logits, argmax);
    return s.ok() ? TPTC_OK : fail(ctx, s);
}

TPTC_API int tptc_debug_trace(tptc_ctx* ctx, uint32_t id, int pos, float* trace) {
    if (!ctx || !trace) return TPTC_ERR_ARG;
    Status s = ctx->eng->debug_trace(id, pos, trace);
    return s.ok() ? TPTC_OK : fail(ctx, s);
}

TPTC_API int tptc_decode_greedy(tptc_ctx* ctx, uint32_t id, int pos, int n, uint32_t* out_ids) {
    if (!ctx) return TPTC_ERR_ARG;
    Status s = ctx->eng->decode_greedy(id, pos, n, out_ids);
    return s.ok() ? TPTC_OK : fail(ctx, s);
}

TPTC_API int tptc_infer(tptc_ctx* ctx, const uint32_t* prompt, int n, const tptc_infer_params* params,
                        tptc_token_cb on_token, void* user) {
    if (!ctx || !params || (n > 0 && !prompt)) return fail_code(ctx, TPTC_ERR_ARG, "null argument");
    Status s = ctx->eng->infer(prompt, n, *params, on_token, user);
    return s.ok() ? TPTC_OK : fail(ctx, s);
}

TPTC_API int tptc_last_device_ms(const tptc_ctx* ctx, double* ms) {
    if (!ctx || !ms) return TPTC_ERR_ARG;
    *ms = ctx->eng->last_device_ms;
    return TPTC_OK;
}

TPTC_API int tptc_decode_kernels(const tptc_ctx* ctx) {
    if (!ctx) return TPTC_ERR_ARG;
    if (!ctx->eng->loaded()) return TPTC_ERR_STATE;
    return ctx->eng->graph_kernels_;
}

TPTC_API int tptc_last_timing(const tptc_ctx* ctx, double* prefill_ms, double* decode_ms, int* n_prompt,
                              int* n_generated) {
    if (!ctx) return TPTC_ERR_ARG;
    if (prefill_ms) *prefill_ms = ctx->eng->last_prefill_ms;
    if (decode_ms) *decode_ms = ctx->eng->last_decode_ms;
    if (n_prompt) *n_prompt = ctx->eng->last_n_prompt;
    if (n_generated) *n_generated = ctx->eng->last_n_generated;
    return TPTC_OK;
}

// ---- kernel-level entry points -----------------------------------------------------------

static bool type_ok(int t) {
    return t == TPTC_TYPE_Q2_K || t == TPTC_TYPE_Q3_K || t == TPTC_TYPE_Q4_K || t == TPTC_TYPE_Q5_K ||
           t == TPTC_TYPE_Q6_K || t == TPTC_TYPE_Q4_0 || t == TPTC_TYPE_Q5_0 || t == TPTC_TYPE_Q4_1 ||
           t == TPTC_TYPE_Q5_1 || t == TPTC_TYPE_Q8_0 || t == TPTC_TYPE_F16;
}

TPTC_API int tptc_dequant(int ggml_type, const void* d_blocks, int64_t n, float* d_out, void* stream) {
    if (!d_blocks || !d_out || n < 0) return TPTC_ERR_ARG;
    int64_t be = 0;
    switch (ggml_type) {
    case TPTC_TYPE_F32: case TPTC_TYPE_F16: be = 1; break;
    case TPTC_TYPE_Q4_0: case TPTC_TYPE_Q4_1: case TPTC_TYPE_Q5_0: case TPTC_TYPE_Q5_1: case TPTC_TYPE_Q8_0: be = 32; break;
    case TPTC_TYPE_Q2_K: case TPTC_TYPE_Q3_K: case TPTC_TYPE_Q4_K: case TPTC_TYPE_Q5_K: case TPTC_TYPE_Q6_K: be = 256; break;
    }
    if (be == 0 || n % be) return TPTC_ERR_ARG;
    cudaError_t e = tptc::launch_dequant_raw(ggml_type, d_blocks, n, d_out, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "dequant");
}

TPTC_API int tptc_quant_q8k(const float* d_x, int64_t k, void* d_out, void* stream) {
    if (!d_x || !d_out || k < 0 || k % 256) return TPTC_ERR_ARG;
    cudaError_t e = tptc::launch_quant_q8k(d_x, k, d_out, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "quant_q8k");
}

TPTC_API int tptc_quant_q80(const float* d_x, int64_t k, void* d_out, void* stream) {
    if (!d_x || !d_out || k < 0 || k % 32) return TPTC_ERR_ARG;
    cudaError_t e = tptc::launch_quant_q80(d_x, k, d_out, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "quant_q80");
}

TPTC_API int tptc_matrix_create(int ggml_type, const void* raw, int raw_on_device, int N, int K, tptc_matrix** out) {
    if (!out || !raw || N <= 0 || K <= 0) return TPTC_ERR_ARG;
    *out = nullptr;
    if (!type_ok(ggml_type)) {
        g_err = "unsupported matrix type";
        return TPTC_ERR_UNSUPPORTED;
    }
    if (K % 256) {
        g_err = "K must be a multiple of 256";
        return TPTC_ERR_UNSUPPORTED;
    }
    tptc_matrix* m = new (std::nothrow) tptc_matrix();
    if (!m) return TPTC_ERR_OOM;
    cudaGetDevice(&m->device);
    cudaError_t ie = tptc::kernels_init_device();
    if (ie != cudaSuccess) {
        delete m;
        return cuda_fail(ie, "kernel setup");
    }
    tptc::DevMatrix& d = m->m;
    d = tptc::dm_geometry(ggml_type, N, K, 0);
    int64_t raw_row = d.main_row_bytes;  // Q4_K, Q5_K, F16: the device super-block is the GGUF block
    if (ggml_type == TPTC_TYPE_Q6_K) raw_row = (int64_t)K / 256 * 210;
    if (ggml_type == TPTC_TYPE_Q8_0) raw_row = (int64_t)K / 32 * 34;
    if (ggml_type == TPTC_TYPE_Q4_0) raw_row = (int64_t)K / 32 * 18;
    if (ggml_type == TPTC_TYPE_Q5_0) raw_row = (int64_t)K / 32 * 22;
    if (ggml_type == TPTC_TYPE_Q4_1) raw_row = (int64_t)K / 32 * 20;
    if (ggml_type == TPTC_TYPE_Q5_1) raw_row = (int64_t)K / 32 * 24;
    if (ggml_type == TPTC_TYPE_Q2_K) raw_row = (int64_t)K / 256 * 84;
    if (ggml_type == TPTC_TYPE_Q3_K) raw_row = (int64_t)K / 256 * 110;
    const size_t main_al = ((size_t)d.main_bytes() + 255) / 256 * 256;
    const size_t total = main_al + 256 + tptc::gemv_act_bytes_max(K);
    cudaError_t e = cudaMalloc(&m->mem, total);
    if (e != cudaSuccess) {
        delete m;
        return cuda_fail(e, "cudaMalloc(matrix)");
    }
    d.main = m->mem;
    m->err = reinterpret_cast<int*>(m->mem + main_al);
    m->act = m->mem + main_al + 256;
    const size_t raw_bytes = (size_t)raw_row * N;
    const uint8_t* src = static_cast<const uint8_t*>(raw);
    uint8_t* tmp = nullptr;
    if (!raw_on_device) {
        e = cudaMalloc(&tmp, raw_bytes);
        if (e == cudaSuccess) e = cudaMemcpy(tmp, raw, raw_bytes, cudaMemcpyHostToDevice);
        src = tmp;
    }
    if (e == cudaSuccess) e = cudaMemset(m->mem, 0, total);
    if (e == cudaSuccess) e = tptc::launch_repack(src, raw_row, N, 0, d, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
        cudaFree(m->mem);
        delete m;
        return cuda_fail(e, "matrix upload/repack");
    }
    *out = m;
    return TPTC_OK;
}

TPTC_API void tptc_matrix_destroy(tptc_matrix* m) {
    if (!m) return;
    if (m->mem) cudaFree(m->mem);
    delete m;
}

TPTC_API int64_t tptc_matrix_bytes(const tptc_matrix* m) { return m ? m->m.bytes() : -1; }

// Programmatic dependent launch for kernel-level GEMVs: TPTC_PDL=1 (the engine's switch).
static bool kernel_pdl() {
    static const bool on = [] {
        const char* e = getenv("TPTC_PDL");
        return e && e[0] == '1';
    }();
    return on;
}

static tptc::GemvParams matrix_params(const tptc_matrix* m, const float* x) {
    tptc::GemvParams p = {};
    p.nseg = 1;
    p.seg[0] = tptc::GemvSeg{m->m, 0};
    p.K = m->m.K;
    p.x = x;
    p.err = m->err;
    p.act_global = m->act;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    tptc::gemv_prepare(p, sms);
    return p;
}

TPTC_API int tptc_gemv(const tptc_matrix* m, const float* d_x, float* d_y, void* stream) {
    if (!m || !d_x || !d_y) return TPTC_ERR_ARG;
    tptc::GemvParams p = matrix_params(m, d_x);
    p.out = d_y;
    cudaError_t e = tptc::gemv_launch(p, tptc::EPI_STORE, static_cast<cudaStream_t>(stream), kernel_pdl());
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "gemv");
}

// Kernel attributes of the current device, set once per device (allocates nothing).
static int ensure_kernels(int* dev_out, int* sms_out) {
    static std::mutex mu;
    static bool done[256];
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "device query");
    if (dev < 0 || dev >= 256) return fail_code(nullptr, TPTC_ERR_UNSUPPORTED, "device ordinal above 255");
    std::lock_guard<std::mutex> lk(mu);
    if (!done[dev]) {
        e = tptc::kernels_init_device();
        if (e != cudaSuccess) return cuda_fail(e, "kernel setup");
        done[dev] = true;
    }
    *dev_out = dev;
    *sms_out = sms;
    return TPTC_OK;
}

static int attn_args(const float* q, const float* kraw, void* kc, const void* vc, int kv_type, const float* cs,
                     const float* sn, const int* pos, float* out, int n_heads, int n_kv, int hd, int max_seq) {
    if (!q || !kraw || !kc || !vc || !cs || !sn || !pos || !out)
        return fail_code(nullptr, TPTC_ERR_ARG, "attention: null pointer");
    if (kv_type != TPTC_TYPE_F16 && kv_type != TPTC_TYPE_F32)
        return fail_code(nullptr, TPTC_ERR_UNSUPPORTED, "attention: kv_type must be TPTC_TYPE_F16 or TPTC_TYPE_F32");
    if (const char* why = tptc::attn_decode_shape_error(n_heads, n_kv, hd, max_seq))
        return fail_code(nullptr, TPTC_ERR_ARG, why);
    return TPTC_OK;
}

// One attention launch over scratch `ws` laid out by attn_scratch_layout.
static int attn_launch(const float* q, const float* kraw, void* kc, const void* vc, int kv_type, const float* cs,
                       const float* sn, const int* pos, float* out, int n_heads, int n_kv, int hd, int max_seq,
                       uint8_t* ws, const tptc::AttnScratch& L, cudaStream_t st) {
    tptc::AttnDecodeParams a = {};
    a.q = q;
    a.kraw = kraw;
    a.kcache = kc;
    a.vcache = vc;
    a.kv_f32 = kv_type == TPTC_TYPE_F32;
    a.rope_cos = cs;
    a.rope_sin = sn;
    a.pos = pos;
    a.out = out;
    a.partial = reinterpret_cast<float*>(ws + L.partial);
    a.counters = reinterpret_cast<int*>(ws + L.counters);
    a.err = reinterpret_cast<int*>(ws + L.err);
    a.n_heads = n_heads;
    a.n_kv = n_kv;
    a.hd = hd;
    a.max_seq = max_seq;
    a.splits = L.splits;
    a.scale = 1.0f / sqrtf((float)hd);
    cudaError_t e = tptc::launch_attn_decode(a, st, false);
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "attn_decode");
}

TPTC_API int64_t tptc_attn_decode_workspace_bytes(int n_heads, int n_kv, int head_dim, int max_seq) {
    if (const char* why = tptc::attn_decode_shape_error(n_heads, n_kv, head_dim, max_seq))
        return fail_code(nullptr, TPTC_ERR_ARG, why);
    int dev = 0, sms = 0;
    if (int rc = ensure_kernels(&dev, &sms)) return rc;
    return (int64_t)tptc::attn_scratch_layout(n_heads, n_kv, head_dim, max_seq, sms).total;
}

TPTC_API int tptc_attn_decode(const float* d_q, const float* d_kraw, void* d_kcache, const void* d_vcache, int kv_type,
                              const float* d_rope_cos, const float* d_rope_sin, const int* d_pos, int n_heads, int n_kv,
                              int head_dim, int max_seq, float* d_out, void* d_workspace, int64_t workspace_bytes,
                              void* stream) {
    if (int rc = attn_args(d_q, d_kraw, d_kcache, d_vcache, kv_type, d_rope_cos, d_rope_sin, d_pos, d_out, n_heads,
                           n_kv, head_dim, max_seq))
        return rc;
    if (!d_workspace) return fail_code(nullptr, TPTC_ERR_ARG, "attention: null workspace");
    int dev = 0, sms = 0;
    if (int rc = ensure_kernels(&dev, &sms)) return rc;
    const tptc::AttnScratch L = tptc::attn_scratch_layout(n_heads, n_kv, head_dim, max_seq, sms);
    if (workspace_bytes < (int64_t)L.total)
        return fail_code(nullptr, TPTC_ERR_ARG,
                         "attention: workspace of " + std::to_string(workspace_bytes) + " bytes, " +
                             std::to_string(L.total) + " needed");
    return attn_launch(d_q, d_kraw, d_kcache, d_vcache, kv_type, d_rope_cos, d_rope_sin, d_pos, d_out, n_heads, n_kv,
                       head_dim, max_seq, static_cast<uint8_t*>(d_workspace), L, static_cast<cudaStream_t>(stream));
}

TPTC_API int tptc_attn_decode_noalloc(const float* d_q, const float* d_kraw, void* d_kcache, const void* d_vcache,
                                      int kv_type, const float* d_rope_cos, const float* d_rope_sin, const int* d_pos,
                                      int n_heads, int n_kv, int head_dim, int max_seq, float* d_out, void* stream) {
    if (int rc = attn_args(d_q, d_kraw, d_kcache, d_vcache, kv_type, d_rope_cos, d_rope_sin, d_pos, d_out, n_heads,
                           n_kv, head_dim, max_seq))
        return rc;
    int dev = 0, sms = 0;
    if (int rc = ensure_kernels(&dev, &sms)) return rc;
    const tptc::AttnScratch L = tptc::attn_scratch_layout(n_heads, n_kv, head_dim, max_seq, sms);
    if (L.total > tptc::kAttnNoAllocScratchBytes)
        return fail_code(nullptr, TPTC_ERR_ARG,
                         "attention (no-alloc): these sizes need " + std::to_string(L.total) +
                             " bytes of scratch, above the static maximum of " +
                             std::to_string(tptc::kAttnNoAllocScratchBytes) + " bytes");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = nullptr;
    cudaError_t e = tptc::attn_noalloc_scratch(dev, st, &ws);
    if (e != cudaSuccess) return cuda_fail(e, "attention (no-alloc) scratch set-up");
    // error word and split counters start every call at zero, whatever the last launch left
    e = cudaMemsetAsync(ws, 0, L.partial, st);
    if (e != cudaSuccess) return cuda_fail(e, "attention (no-alloc) scratch reset");
    return attn_launch(d_q, d_kraw, d_kcache, d_vcache, kv_type, d_rope_cos, d_rope_sin, d_pos, d_out, n_heads, n_kv,
                       head_dim, max_seq, ws, L, st);
}

TPTC_API int tptc_attn_decode_noalloc_status(void* stream, int* out_code) {
    if (!out_code) return fail_code(nullptr, TPTC_ERR_ARG, "attention (no-alloc) status: null out_code");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    e = tptc::attn_noalloc_status(dev, static_cast<cudaStream_t>(stream), out_code);
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "attention (no-alloc) status");
}

TPTC_API int tptc_sample(const float* d_logits, int vocab, int* d_counts, float penalty, float temperature,
                         float top_p, uint64_t seed, int* d_step, float* d_scratch, uint32_t* d_out_tok,
                         uint64_t* d_dbg, void* stream) {
    if (!d_logits || vocab <= 0 || !d_scratch || !d_out_tok) return fail_code(nullptr, TPTC_ERR_ARG, "sample: bad argument");
    tptc::SampleParams s = {};
    s.logits = d_logits;
    s.vocab = vocab;
    s.counts = d_counts;
    s.penalty = penalty;
    s.temperature = temperature;
    s.top_p = top_p;
    s.seed = seed;
    s.step = d_step;
    s.scratch = d_scratch;
    s.out_tok = d_out_tok;
    s.dbg = reinterpret_cast<unsigned long long*>(d_dbg);
    // the kernels' work area, stream-ordered (this entry takes only the caller's buffers)
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* work = nullptr;
    cudaError_t e = cudaMallocAsync(&work, tptc::kSampleWorkBytes, st);
    if (e != cudaSuccess) return cuda_fail(e, "sample");
    s.work = static_cast<unsigned char*>(work);
    e = tptc::launch_sample(s, st, false);
    const cudaError_t ef = cudaFreeAsync(work, st);
    if (e == cudaSuccess) e = ef;
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "sample");
}

TPTC_API int tptc_gemm_f16(const void* d_a, const void* d_b, float* d_c, int M, int N, int K, void* stream) {
    if (!d_a || !d_b || !d_c || M <= 0 || N <= 0 || K <= 0) return fail_code(nullptr, TPTC_ERR_ARG, "gemm: bad argument");
    if (K % 64 || (reinterpret_cast<uintptr_t>(d_a) & 15) || (reinterpret_cast<uintptr_t>(d_b) & 15))
        return fail_code(nullptr, TPTC_ERR_ARG, "gemm: K must be a multiple of 64 and A, B 16-byte aligned");
    int dev = 0, sms = 0;
    if (int rc = ensure_kernels(&dev, &sms)) return rc;
    tptc::GemmTcParams p = {};
    p.M = M;
    p.N = N;
    p.K = K;
    p.c = d_c;
    p.ldc = N;
    cudaError_t e = tptc::gemm_tc(tptc::GEMM_STORE, static_cast<const __half*>(d_a), K, static_cast<const __half*>(d_b),
                                  K, p, static_cast<cudaStream_t>(stream), false);
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "gemm_tc");
}

TPTC_API int tptc_gemm_q(const tptc_matrix* m, const void* d_a, float* d_c, int M, void* stream) {
    if (!m || !d_a || !d_c || M <= 0) return fail_code(nullptr, TPTC_ERR_ARG, "gemm_q: bad argument");
    if (!tptc::gemm_q_supported(m->m) || m->m.glu)
        return fail_code(nullptr, TPTC_ERR_UNSUPPORTED, "gemm_q: Q4_K, Q6_K or Q8_0 matrices only");
    if (reinterpret_cast<uintptr_t>(d_a) & 15) return fail_code(nullptr, TPTC_ERR_ARG, "gemm_q: A must be 16-byte aligned");
    int dev = 0, sms = 0;
    if (int rc = ensure_kernels(&dev, &sms)) return rc;
    tptc::GemmTcParams p = {};
    p.M = M;
    p.N = m->m.N;
    p.K = m->m.K;
    p.c = d_c;
    p.ldc = m->m.N;
    p.err = m->err;
    cudaError_t e = tptc::gemm_q(tptc::GEMM_STORE, static_cast<const __half*>(d_a), m->m.K, m->m, p,
                                 static_cast<cudaStream_t>(stream), false);
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "gemm_q");
}

TPTC_API int tptc_attn_prefill(const void* d_q, const void* d_kcache, const void* d_vcache, void* d_out, int T,
                               int start, int n_heads, int n_kv, int head_dim, int max_seq, void* stream) {
    if (!d_q || !d_kcache || !d_vcache || !d_out || T <= 0 || start < 0 || n_heads <= 0 || n_kv <= 0 ||
        n_heads % n_kv || max_seq <= 0 || start + T > max_seq)
        return fail_code(nullptr, TPTC_ERR_ARG, "attn_prefill: bad argument");
    if (head_dim != 64 && head_dim != 96 && head_dim != 128)
        return fail_code(nullptr, TPTC_ERR_UNSUPPORTED, "attn_prefill: head_dim must be 64, 96 or 128");
    int dev = 0, sms = 0;
    if (int rc = ensure_kernels(&dev, &sms)) return rc;
    tptc::AttnPrefillParams p = {};
    p.q = static_cast<const __half*>(d_q);
    p.kcache = static_cast<const __half*>(d_kcache);
    p.vcache = static_cast<const __half*>(d_vcache);
    p.out = static_cast<__half*>(d_out);
    p.T = T;
    p.start = start;
    p.n_heads = n_heads;
    p.n_kv = n_kv;
    p.hd = head_dim;
    p.max_seq = max_seq;
    p.scale = (float)(1.0 / sqrt((double)head_dim));
    cudaError_t e = tptc::launch_attn_prefill(p, static_cast<cudaStream_t>(stream), false);
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "attn_prefill");
}

TPTC_API int tptc_matrix_dequant_f16(const tptc_matrix* m, void* d_out, void* stream) {
    if (!m || !d_out) return fail_code(nullptr, TPTC_ERR_ARG, "matrix_dequant_f16: null argument");
    cudaError_t e = tptc::launch_dequant_rows_f16(m->m, 0, m->m.N, static_cast<__half*>(d_out),
                                                  static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "dequant_rows_f16");
}

TPTC_API int tptc_block_dots(const tptc_matrix* m, const float* d_x, int32_t* d_isum, int32_t* d_msum, void* stream) {
    if (!m || !d_x || !d_isum) return TPTC_ERR_ARG;
    if (m->m.type == TPTC_TYPE_F16) return TPTC_ERR_UNSUPPORTED;
    tptc::GemvParams p = matrix_params(m, d_x);
    p.isum = d_isum;
    p.msum = d_msum;
    cudaError_t e = tptc::gemv_launch(p, tptc::EPI_DOTS, static_cast<cudaStream_t>(stream), false);
    return e == cudaSuccess ? TPTC_OK : cuda_fail(e, "block_dots");
}

}  // extern "C"
