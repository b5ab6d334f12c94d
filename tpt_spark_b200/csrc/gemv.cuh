// gemv.cuh -- batch-1 dequant-fused GEMV (decode) for Q4_K / Q6_K / Q8_0 / F16 weights.
#pragma once

#include "common.cuh"

namespace tptc {

// Device layout of a weight matrix [N out x K in] (K a multiple of 256):
//   Q4_K  main = GGUF blocks unchanged, 144 B per 256 elements, rows contiguous
//   Q6_K  main = ql|qh|scales (208 B per 256) ; dplane = f16 d per block [N, K/256]
//   Q8_0  main = qs (32 B per 32)              ; dplane = f16 d per block [N, K/32]
//   F16   main = f16 values [N, K]
// Every main row is a multiple of 16 bytes, so any run of whole super-blocks of a row can
// be fetched with one 1-D bulk copy.
struct DevMatrix {
    int type = 0;
    int N = 0, K = 0;
    uint8_t* main = nullptr;
    uint16_t* dplane = nullptr;
    int64_t main_row_bytes = 0;  // bytes per row in `main`
    int64_t d_per_row = 0;       // f16 entries per row in `dplane`
    int64_t bytes() const { return main_row_bytes * N + d_per_row * 2 * N; }
};

// Bytes of `main` per 256-element super-block, and super-blocks per pipeline chunk.
__host__ __device__ inline int sb_bytes(int type) {
    return type == TPTC_TYPE_Q4_K ? 144 : type == TPTC_TYPE_Q6_K ? 208 : type == TPTC_TYPE_Q8_0 ? 256 : 512;
}
__host__ __device__ inline int chunk_sb(int type) { return type == TPTC_TYPE_F16 ? 8 : 16; }

enum GemvEpi : int {
    EPI_STORE = 0,  // out[row] = y
    EPI_RESID = 1,  // out[row] += y   (residual stream update)
    EPI_QKV = 2,    // RoPE on q/k rows, q -> out, k/v -> fp16 KV cache at pos
    EPI_GLU = 3,    // paired gate/up rows: out[row] = silu(gate) * up
    EPI_DOTS = 4,   // integer block sums (test hook)
};

struct GemvSeg {
    const uint8_t* main;
    const uint16_t* dplane;
    int type;
    int N;
    int64_t row_bytes;
    int64_t d_per_row;
    int cta_begin;  // first CTA of this segment (linear mapping)
};

struct GemvParams {
    GemvSeg seg[3];
    int nseg;
    int paired;  // 1: CTA b = rows 4b..4b+3 of seg0 (warps 0-3) and seg1 (warps 4-7)
    int K;
    const float* x;       // input activation [K] (f32)
    const float* norm_w;  // RMSNorm gain [K] or nullptr (no norm)
    float eps;
    float* out;
    // EPI_QKV
    void* kcache;          // this layer's K cache, layout [n_kv][max_seq][hd], fp16 or f32
    void* vcache;
    int kv_f32;            // 1: the cache holds f32 (candle's precision), 0: fp16
    const float* rope_cos;  // [max_seq][hd/2]
    const float* rope_sin;
    const int* pos;  // device scalar: position being written
    int hd;
    int max_seq;
    // EPI_DOTS
    int32_t* isum;
    int32_t* msum;
    // activation layout in shared memory (byte offsets; -1 = absent)
    int act_f32, act_q8k, act_q8k_d, act_q8k_bs, act_q80, act_q80_d;
    int act_bytes;
    int stages;
    int slot_bytes;
    int* err;
};

// Host helpers (gemv.cu).
void gemv_prepare(GemvParams& p);  // fills activation offsets, stages, slot bytes
int gemv_grid(const GemvParams& p);
size_t gemv_smem(const GemvParams& p);
cudaError_t gemv_launch(const GemvParams& p, int epi, cudaStream_t st, bool pdl);
cudaError_t gemv_init_device();  // per-device kernel attributes (call once per device)

}  // namespace tptc
