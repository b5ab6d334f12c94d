// prefill.h -- batched prompt processing (prefill) kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace tptc {

cudaError_t prefill_init_device();

// ---- tensor-core GEMM (gemm_tc.cu): C[M x N] = A[M x K] . B[N x K]^T, fp16 in, f32 accumulate
enum GemmEpi : int {
    GEMM_STORE = 0,  // c[m][n] = acc (f32)
    GEMM_RESID = 1,  // c[m][n] += acc (f32 residual stream)
    GEMM_GLU = 2,    // B rows in gate|up tile order (per 8 rows: 4 gate, 4 up): h[m][n/2 ...] =
                     // silu(gate) * up as fp16
};
struct GemmTcParams {
    int M, N, K;
    float* c;  // GEMM_STORE / GEMM_RESID, leading dimension ldc
    int ldc;
    __half* h;  // GEMM_GLU, leading dimension ldh
    int ldh;
    int* err;   // bounded waits that give up set TPTC_ERR_TIMEOUT here
    int geglu;  // GEMM_GLU: 0 silu(gate) * up, 1 GEGLU's tanh-form gelu(gate) * up
};
// A and B 16-byte aligned, lda / ldb multiples of 8 elements, K a multiple of 64.
cudaError_t gemm_tc(int epi, const __half* a, int lda, const __half* b, int ldb, const GemmTcParams& p,
                    cudaStream_t st, bool pdl);
cudaError_t gemm_tc_init_device();

// ---- the same GEMM with the weight dequantisation fused in (gemm_q.cu): B is a Q4_K / Q6_K /
// Q8_0 matrix in the device layout (its physical rows), N <= its padded rows, K = its K.
struct DevMatrix;
bool gemm_q_supported(const DevMatrix& w);
// Whether the fused GEMM is expected to beat "expand w to fp16, then gemm_tc" for an M x N
// product on `sms` SMs (a wave model of both with B200-measured step times): the fused kernel
// re-expands a weight tile for every 128-row block of M, the two-pass path expands the whole
// matrix once, so the fused one wins for short chunks of wide matrices.
bool gemm_q_preferred(const DevMatrix& w, int M, int N, int sms);
cudaError_t gemm_q(int epi, const __half* a, int lda, const DevMatrix& w, const GemmTcParams& p, cudaStream_t st,
                   bool pdl);
cudaError_t gemm_q_init_device();

// ---- causal attention over a prompt chunk (attn_prefill.cu)
struct AttnPrefillParams {
    const __half* q;       // [T][n_heads][hd], rotated
    const __half* kcache;  // this layer's caches [n_kv][max_seq][hd] (fp16), chunk rows written
    const __half* vcache;
    __half* out;           // [T][n_heads][hd]
    int T, start;          // chunk rows are positions start .. start + T - 1
    int n_heads, n_kv, hd, max_seq;
    float scale;           // 1/sqrt(hd)
    int* err;              // optional: bounded waits that give up set TPTC_ERR_TIMEOUT here
};
// head_dim 64, 96 and 128 run on tcgen05 (attn_prefill_tc_kernel; 96 in the 128-wide layout
// with zero-filled padding); `use_tc` = 0 forces the mma.sync kernel (kernel-level comparisons).
cudaError_t launch_attn_prefill(const AttnPrefillParams& p, cudaStream_t st, bool pdl, int use_tc = 1);
cudaError_t attn_prefill_init_device();

// ---- per-token elementwise steps of a chunk (prefill.cu)
struct PrefillRope {
    const float* cos;  // [max_seq][hd/2]
    const float* sin;
};

}  // namespace tptc
