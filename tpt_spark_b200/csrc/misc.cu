// misc.cu -- token embedding row, on-device argmax, per-device kernel setup.
#include <algorithm>

#include "kernels.h"
#include "moe.h"
#include "quant.cuh"

namespace tptc {

cudaError_t attn_init_device();
cudaError_t prefill_init_device();

namespace {

// candle dequantises token_embd to f32 at load and index_selects a row; here one row is
// dequantised on the fly (bit-identical values) into the residual stream x.
// Replaces the reference's whole-table dequant + row copy (wgpu_engine.rs:235-242,364-368).
__global__ void embed_row_kernel(DevMatrix emb, const uint32_t* __restrict__ tok_ptr, float* __restrict__ x,
                                 int* step, float scale) {
    pdl_wait();
    pdl_launch_dependents();
    if (step && blockIdx.x == 0 && threadIdx.x == 0) *step += 1;  // opens a decode step (TpLink epochs)
    const int row = (int)*tok_ptr;  // token_embd is never a fused gate|up matrix: phys row = row
    const int K = emb.K;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < K; i += gridDim.x * blockDim.x) {
        const float v = dm_elem(emb, row, i);
        x[i] = scale == 1.f ? v : __fmul_rn(v, scale);
    }
}

// Greedy pick, candle LogitsProcessor::sample_argmax: Iterator::max_by(f32::total_cmp)
// returns the LAST of equal maxima, so ties go to the highest index.
__device__ __forceinline__ bool better(float v, int i, float best, int bi) {
    return i >= 0 && (bi < 0 || v > best || (v == best && i > bi));
}

// Argmax of logits[0..n) over the whole CTA; the result (value, index) is valid in lane 0 of
// warp 0 (index -1 for n == 0).
__device__ __forceinline__ void block_argmax(const float* __restrict__ logits, int n, float& best, int& bi) {
    __shared__ float sv[32];
    __shared__ int si[32];
    best = -INFINITY;
    bi = -1;
    // eight independent loads in flight per thread per round
    constexpr int U = 8;
    const int step = blockDim.x * U;
    for (int base = 0; base < n; base += step) {
        float v[U];
#pragma unroll
        for (int k = 0; k < U; k++) {
            const int i = base + k * blockDim.x + threadIdx.x;
            v[k] = i < n ? logits[i] : -INFINITY;
        }
#pragma unroll
        for (int k = 0; k < U; k++) {
            const int i = base + k * blockDim.x + threadIdx.x;
            if (i < n && better(v[k], i, best, bi)) {
                best = v[k];
                bi = i;
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(v2, i2, best, bi)) {
            best = v2;
            bi = i2;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x / 32;
        best = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : -1;
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(v2, i2, best, bi)) {
                best = v2;
                bi = i2;
            }
        }
    }
}

// The picked token: the step's output, and with chaining the next step's input, history and
// position.
__device__ __forceinline__ void emit_token(int bi, uint32_t* out_tok, uint32_t* next_tok, int* pos,
                                           uint32_t* history) {
    const uint32_t t = bi < 0 ? 0u : (uint32_t)bi;
    *out_tok = t;
    if (next_tok) *next_tok = t;
    if (pos) {
        if (history) history[*pos] = t;  // token generated after position *pos
        *pos += 1;
    }
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ logits, int n, uint32_t* out_tok,
                                                      uint32_t* next_tok, int* pos, uint32_t* history) {
    pdl_wait();
    pdl_launch_dependents();
    float best;
    int bi;
    block_argmax(logits, n, best, bi);
    if (threadIdx.x == 0) emit_token(bi, out_tok, next_tok, pos, history);
}

// Vocab-parallel argmax under tensor parallelism: this rank holds logits of rows
// [row0, row0 + n).  Its best (value, global index) goes into every rank's inbox as two
// 64-bit words, each tagged with the epoch of the step's argmax use (TpLink); then the pairs
// of all ranks are read back from this rank's own inbox (a word whose epoch is not yet the
// current one is read again, bounded by wait_polls: TPTC_ERR_TIMEOUT) and reduced in rank
// order with the same tie rule, so every rank picks the same token.
__global__ void __launch_bounds__(1024) argmax_tp_kernel(const float* __restrict__ logits, int n, int row0,
                                                         const TpLink* __restrict__ link, int* err, uint32_t* out_tok,
                                                         uint32_t* next_tok, int* pos, uint32_t* history) {
    pdl_wait();
    pdl_launch_dependents();
    float best;
    int bi;
    block_argmax(logits, n, best, bi);
    if (threadIdx.x != 0) return;
    const TpLink& t = *link;
    const unsigned int e = (unsigned int)(*reinterpret_cast<volatile const int*>(t.step)) * (unsigned int)t.uses_per_step +
                           (unsigned int)(t.uses_per_step - 1) + 1u;
    const size_t off = tp_argmax_offset(t.size, t.dim);
    const unsigned long long wv = ((unsigned long long)e << 32) | __float_as_uint(best);
    const unsigned long long wi = ((unsigned long long)e << 32) | (unsigned int)(bi < 0 ? 0 : row0 + bi);
    for (int r = 0; r < t.size; r++) {
        st_volatile_u64(t.inbox[r] + off + 2 * t.rank, wv);
        st_volatile_u64(t.inbox[r] + off + 2 * t.rank + 1, wi);
    }
    const unsigned long long* in = t.inbox[t.rank] + off;
    float gb = -INFINITY;
    int gi = -1;
    for (int r = 0; r < t.size; r++) {
        unsigned long long v = ld_volatile_u64(in + 2 * r), i = ld_volatile_u64(in + 2 * r + 1);
        uint32_t polls = 0;
        while ((unsigned int)(v >> 32) != e || (unsigned int)(i >> 32) != e) {
            if (++polls > t.wait_polls || ((polls & 255) == 0 && err && *reinterpret_cast<volatile int*>(err))) {
                if (err) atomicExch(err, TPTC_ERR_TIMEOUT);
                break;
            }
            if (polls > 64) __nanosleep(32);
            v = ld_volatile_u64(in + 2 * r);
            i = ld_volatile_u64(in + 2 * r + 1);
        }
        if ((unsigned int)(v >> 32) != e || (unsigned int)(i >> 32) != e) continue;
        const float fv = __uint_as_float((unsigned int)(v & 0xffffffffu));
        const int fi = (int)(i & 0xffffffffu);
        if (better(fv, fi, gb, gi)) {
            gb = fv;
            gi = fi;
        }
    }
    emit_token(gi, out_tok, next_tok, pos, history);
}

}  // namespace

cudaError_t launch_embed_row(const DevMatrix& emb, const uint32_t* tok_ptr, float* x, cudaStream_t st, bool pdl,
                             int* step, float scale) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::max(1, std::min(16, emb.K / 256)));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, embed_row_kernel, emb, tok_ptr, x, step, scale);
}

cudaError_t launch_argmax(const float* logits, int n, uint32_t* out_tok, uint32_t* next_tok, int* pos,
                          uint32_t* history, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1024);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, argmax_kernel, logits, n, out_tok, next_tok, pos, history);
}

cudaError_t launch_argmax_tp(const float* logits, int n, int row0, const TpLink* link, int* err, uint32_t* out_tok,
                             uint32_t* next_tok, int* pos, uint32_t* history, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1024);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, argmax_tp_kernel, logits, n, row0, link, err, out_tok, next_tok, pos, history);
}

cudaError_t kernels_init_device() {
    cudaError_t e = gemv_init_device();
    if (e != cudaSuccess) return e;
    e = moe_init_device();
    if (e != cudaSuccess) return e;
    e = attn_init_device();
    if (e != cudaSuccess) return e;
    return prefill_init_device();
}

}  // namespace tptc
