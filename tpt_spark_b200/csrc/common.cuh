// common.cuh -- shared device/host helpers of libtptc (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "tptc.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libtptc is written for sm_100a (B200) only"
#endif

namespace tptc {

constexpr int QK_K = 256;
constexpr int QK8_0 = 32;
constexpr int Q4K_BYTES = 144;   // d f16 | dmin f16 | scales[12] | qs[128]
constexpr int Q6K_BYTES = 210;   // ql[128] | qh[64] | scales[16] int8 | d f16 (GGUF layout)
constexpr int Q6K_MAIN = 208;    // device layout: ql | qh | scales, d in a separate plane
constexpr int Q80_BYTES = 34;    // d f16 | qs[32] (GGUF layout); device: qs plane + d plane
constexpr int Q40_BYTES = 18;    // d f16 | qs[16] (element l < 16: low nibble of qs[l], l + 16: high)
constexpr int Q41_BYTES = 20;    // d f16 | m f16 | qs[16]
constexpr int Q50_BYTES = 22;    // d f16 | qh u32 (bit l: 5th bit of element l) | qs[16]
constexpr int Q51_BYTES = 24;    // d f16 | m f16 | qh u32 | qs[16]
constexpr int Q2K_BYTES = 84;    // scales[16] (sc | m << 4) | qs[64] (2-bit) | d f16 | dmin f16
constexpr int Q3K_BYTES = 110;   // hmask[32] | qs[64] (2-bit) | scales[12] (6-bit) | d f16
constexpr int Q5K_BYTES = 176;   // d f16 | dmin f16 | scales[12] | qh[32] | qs[128]

// block_q8_K: the activation format candle pairs with Q4_K / Q6_K weights (292 bytes).
struct BlockQ8K {
    float d;
    int8_t qs[QK_K];
    int16_t bsums[QK_K / 16];
};
static_assert(sizeof(BlockQ8K) == 292, "block_q8_K layout");

// Status helpers -------------------------------------------------------------------------

struct Status {
    int code = TPTC_OK;
    std::string msg;
    bool ok() const { return code == TPTC_OK; }
};

std::string cuda_msg(cudaError_t e, const char* what);

#define TPTC_CUDA_RET(call)                                                                  \
    do {                                                                                     \
        cudaError_t _e = (call);                                                             \
        if (_e != cudaSuccess) return ::tptc::Status{TPTC_ERR_CUDA, ::tptc::cuda_msg(_e, #call)}; \
    } while (0)

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Device-side primitives -------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait: every mbarrier wait in this library gives up after `limit` polls (each
// poll is a hardware try_wait with its own time slice), records TPTC_ERR_TIMEOUT in
// *err and returns false, so that a lost transfer can never hang the GPU.
constexpr uint32_t kWaitPolls = 1u << 22;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
    for (uint32_t i = 0; i < kWaitPolls; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicExch(err, TPTC_ERR_TIMEOUT);
    return false;
}

// Bounded wait that yields the issue slot between polls (nanosleep): for a warp whose wait
// is not on the critical path (a producer waiting for a free ring slot), so that it does not
// take issue cycles from the warps doing the arithmetic.  Gives up after kWaitPolls polls
// (at least 4 s of sleep), like mbar_wait_bounded.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, int* err) {
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        __nanosleep(64);
    }
    if (err) atomicExch(err, TPTC_ERR_TIMEOUT);
    return false;
}

// 1-D bulk copy global -> shared (TMA engine, no tensor map), completion on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: wait for the producing grid / let the next grid start.
// GEGLU's gate activation times up: gelu(g) = g * 0.5 * (1 + tanh(0.7978845608 * (g + 0.044715 g^3))),
// the tanh form and operation order of the reference's shaders/geglu.wgsl:24-25, unfused.
__device__ __forceinline__ float gelu_tanh_mul(float g, float u) {
    const float g3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, g), g), g);
    const float t = tanhf(__fmul_rn(0.7978845608f, __fadd_rn(g, g3)));
    return __fmul_rn(__fmul_rn(__fmul_rn(g, 0.5f), __fadd_rn(1.f, t)), u);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Volatile (relaxed, system-visible) 64-bit accesses: single-copy atomic for aligned words.
__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ld_volatile_u64x2(const unsigned long long* p, unsigned long long& a,
                                                  unsigned long long& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Q4_K 6-bit scale and min of sub-block j (gguf/quants.py Q4_K.get_scale_min).
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

}  // namespace tptc
