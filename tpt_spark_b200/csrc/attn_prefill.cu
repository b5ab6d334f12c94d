// attn_prefill.cu -- causal GQA attention for a prompt chunk (prefill) on the tensor cores.
//
// Replaces the reference's per-token attention passes during its prefill loop
// (attention.wgsl:31-170 once per prompt token, wgpu_engine.rs:254-261) with one kernel over
// the chunk: query rows t (absolute position start + t) attend to keys 0 .. start + t of the
// KV cache (the chunk's own keys already written there), score = q.k / sqrt(hd), softmax,
// P.V; head h reads kv head h / (n_heads / n_kv).
//
// A CTA of 4 warps owns 64 query rows of one head (16 per warp) and streams the key/value
// positions in 64-row tiles through a double-buffered shared-memory ring (cp.async): scores
// S = Q K^T and the update O += P V run on mma.sync m16n8k16 (fp16 inputs, f32 accumulate),
// with an online softmax in base 2 in registers (flash-attention, one pass).  Q and the
// probabilities enter the tensor cores as fp16; the KV cache is fp16.
#include "prefill.h"

namespace tptc {

namespace {

constexpr int BQ = 64, BKV = 64, kThreads = 128;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int HD>
__global__ void __launch_bounds__(kThreads) attn_prefill_kernel(const __grid_constant__ AttnPrefillParams p) {
    constexpr int LD = HD + 8;  // padded row (halves): conflict-free ldmatrix
    constexpr int KS = HD / 16, NB = HD / 8;
    extern __shared__ __align__(16) uint8_t smem[];
    __half* sq = reinterpret_cast<__half*>(smem);  // [BQ][LD]
    __half* skv = sq + BQ * LD;                    // [2][K|V][BKV][LD]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int h = blockIdx.y, q0 = blockIdx.x * BQ, G = p.n_heads / p.n_kv, kvh = h / G;
    const int rows = min(BQ, p.T - q0);
    const __half* kc = p.kcache + (size_t)kvh * p.max_seq * HD;
    const __half* vc = p.vcache + (size_t)kvh * p.max_seq * HD;
    const int last = p.start + q0 + rows - 1;   // last key any row of the block attends to
    const int ntiles = last / BKV + 1;

    pdl_wait();
    pdl_launch_dependents();

    // Q tile (rows past the chunk are zero) and the first K/V tile
    constexpr int CH = HD / 8;  // 16-byte chunks per row
    for (int i = tid; i < BQ * CH; i += kThreads) {
        const int r = i / CH, c = i % CH;
        __half* dst = sq + r * LD + c * 8;
        if (r < rows) cp_async16(dst, p.q + ((size_t)(q0 + r) * p.n_heads + h) * HD + c * 8);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    auto load_kv = [&](int tile, int buf) {
        __half* dk = skv + buf * 2 * BKV * LD;
        __half* dv = dk + BKV * LD;
        const int p0 = tile * BKV;
        for (int i = tid; i < BKV * CH; i += kThreads) {
            const int r = i / CH, c = i % CH;
            if (p0 + r <= last) {
                cp_async16(dk + r * LD + c * 8, kc + (size_t)(p0 + r) * HD + c * 8);
                cp_async16(dv + r * LD + c * 8, vc + (size_t)(p0 + r) * HD + c * 8);
            } else {
                *reinterpret_cast<uint4*>(dk + r * LD + c * 8) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(dv + r * LD + c * 8) = make_uint4(0, 0, 0, 0);
            }
        }
    };
    load_kv(0, 0);
    cp_async_commit();

    const int g = lane >> 2, t4 = lane & 3;
    const float sl2 = p.scale * 1.4426950408889634f;
    // this thread's two rows: warp * 16 + g and + 8 (absolute positions)
    const int pos_a = p.start + q0 + warp * 16 + g, pos_b = pos_a + 8;
    float o[NB][4];
#pragma unroll
    for (int j = 0; j < NB; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    uint32_t qf[KS][4];

    for (int tile = 0; tile < ntiles; tile++) {
        const int buf = tile & 1;
        if (tile + 1 < ntiles) load_kv(tile + 1, buf ^ 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (tile == 0) {
#pragma unroll
            for (int k = 0; k < KS; k++)
                ldsm_x4(qf[k], sq + (warp * 16 + (lane & 15)) * LD + k * 16 + (lane >> 4) * 8);
        }
        const __half* tk = skv + buf * 2 * BKV * LD;
        const __half* tv = tk + BKV * LD;
        // S = Q K^T for this warp's 16 rows x 64 positions
        float s[BKV / 8][4];
#pragma unroll
        for (int j = 0; j < BKV / 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int j = 0; j < BKV / 8; j += 2) {
#pragma unroll
            for (int k = 0; k < KS; k++) {
                uint32_t b[4];
                ldsm_x4(b, tk + (j * 8 + (lane & 7) + 8 * (lane >> 4)) * LD + k * 16 + 8 * ((lane >> 3) & 1));
                mma16816(s[j], qf[k], b[0], b[1]);
                mma16816(s[j + 1], qf[k], b[2], b[3]);
            }
        }
        // causal mask (only the last tiles reach past a row's position) and the online softmax
        const int p0 = tile * BKV;
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int j = 0; j < BKV / 8; j++) {
            const int c0 = p0 + j * 8 + 2 * t4;
            s[j][0] = c0 <= pos_a ? s[j][0] * sl2 : -INFINITY;
            s[j][1] = c0 + 1 <= pos_a ? s[j][1] * sl2 : -INFINITY;
            s[j][2] = c0 <= pos_b ? s[j][2] * sl2 : -INFINITY;
            s[j][3] = c0 + 1 <= pos_b ? s[j][3] * sl2 : -INFINITY;
            mx_a = fmaxf(mx_a, fmaxf(s[j][0], s[j][1]));
            mx_b = fmaxf(mx_b, fmaxf(s[j][2], s[j][3]));
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        const float mu_a = mn_a == -INFINITY ? 0.f : mn_a, mu_b = mn_b == -INFINITY ? 0.f : mn_b;
        const float al_a = fast_exp2(m_a - mu_a), al_b = fast_exp2(m_b - mu_b);
        m_a = mn_a;
        m_b = mn_b;
        float ls_a = 0.f, ls_b = 0.f;
#pragma unroll
        for (int j = 0; j < BKV / 8; j++) {
            s[j][0] = fast_exp2(s[j][0] - mu_a);
            s[j][1] = fast_exp2(s[j][1] - mu_a);
            s[j][2] = fast_exp2(s[j][2] - mu_b);
            s[j][3] = fast_exp2(s[j][3] - mu_b);
            ls_a += s[j][0] + s[j][1];
            ls_b += s[j][2] + s[j][3];
        }
        l_a = l_a * al_a + ls_a;  // quad partials: reduced across the 4 lanes at the end
        l_b = l_b * al_b + ls_b;
#pragma unroll
        for (int j = 0; j < NB; j++) {
            o[j][0] *= al_a;
            o[j][1] *= al_a;
            o[j][2] *= al_b;
            o[j][3] *= al_b;
        }
        // O += P V: P (fp16) from the score fragments, V through ldmatrix.trans
#pragma unroll
        for (int kk = 0; kk < BKV / 16; kk++) {
            uint32_t a[4];
            a[0] = pack_half2(s[2 * kk][0], s[2 * kk][1]);
            a[1] = pack_half2(s[2 * kk][2], s[2 * kk][3]);
            a[2] = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            a[3] = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int j = 0; j < NB; j += 2) {
                uint32_t b[4];
                ldsm_x4_t(b, tv + (kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * LD + j * 8 + 8 * (lane >> 4));
                mma16816(o[j], a, b[0], b[1]);
                mma16816(o[j + 1], a, b[2], b[3]);
            }
        }
        __syncthreads();  // the buffer is refilled by the next iteration's loads
    }
    cp_async_wait<0>();

    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    const float ia = 1.f / l_a, ib = 1.f / l_b;
    const int ra = warp * 16 + g, rb = ra + 8;
#pragma unroll
    for (int j = 0; j < NB; j++) {
        const int col = j * 8 + 2 * t4;
        if (ra < rows)
            *reinterpret_cast<uint32_t*>(p.out + ((size_t)(q0 + ra) * p.n_heads + h) * HD + col) =
                pack_half2(o[j][0] * ia, o[j][1] * ia);
        if (rb < rows)
            *reinterpret_cast<uint32_t*>(p.out + ((size_t)(q0 + rb) * p.n_heads + h) * HD + col) =
                pack_half2(o[j][2] * ib, o[j][3] * ib);
    }
}

template <int HD>
size_t attn_prefill_smem() {
    return (size_t)(BQ + 4 * BKV) * (HD + 8) * sizeof(__half);
}

}  // namespace

cudaError_t attn_prefill_init_device() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(attn_prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)attn_prefill_smem<64>())))
        return e;
    if ((e = cudaFuncSetAttribute(attn_prefill_kernel<96>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)attn_prefill_smem<96>())))
        return e;
    return cudaFuncSetAttribute(attn_prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)attn_prefill_smem<128>());
}

cudaError_t launch_attn_prefill(const AttnPrefillParams& p, cudaStream_t st, bool pdl) {
    if (p.T <= 0 || p.n_kv <= 0 || p.n_heads % p.n_kv || p.start < 0 || p.start + p.T > p.max_seq)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p.T + BQ - 1) / BQ, p.n_heads);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (p.hd) {
    case 64: cfg.dynamicSmemBytes = attn_prefill_smem<64>(); return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<64>, p);
    case 96: cfg.dynamicSmemBytes = attn_prefill_smem<96>(); return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<96>, p);
    case 128:
        cfg.dynamicSmemBytes = attn_prefill_smem<128>();
        return cudaLaunchKernelEx(&cfg, attn_prefill_kernel<128>, p);
    }
    return cudaErrorInvalidValue;
}

}  // namespace tptc
