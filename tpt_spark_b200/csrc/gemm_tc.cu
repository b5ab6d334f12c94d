// gemm_tc.cu -- prefill GEMM on the 5th-generation tensor cores: C[M x N] = A[M x K] . B[N x K]^T
// with A the prompt's activations (fp16, one row per token) and B a weight matrix (fp16,
// dequantised from its GGUF blocks), f32 accumulation in tensor memory.
//
// Replaces the per-token matmuls of the reference's prefill loop (wgpu_engine.rs:254-261,
// gemm.wgsl with M = 1 once per token) for a whole prompt.
//
// A persistent kernel (one CTA per SM, 192 KB of shared memory) walks 128 x 256 tiles of C,
// M fastest so that concurrent CTAs share the B tiles and the whole A operand stays in L2:
//   - warp 0 (one lane): TMA producer.  Both operands are 2-D tensor maps with 128-byte
//     swizzle; a pipeline stage holds a 128 x 64 tile of A and a 256 x 64 tile of B (16 + 32
//     KB, K-major, the canonical SWIZZLE_128B operand layout of tcgen05.mma), completion
//     counted on the stage's "full" mbarrier;
//   - warp 1: allocates all 512 TMEM columns (two 256-column f32 accumulators); one lane
//     issues tcgen05.mma (M = 128, N = 256, K = 16: four per stage, the descriptor start
//     address advancing 32 bytes within the swizzle atom), commits each stage to its "empty"
//     mbarrier so the producer refills it as soon as the tensor core has read it, and each
//     finished accumulator to "tfull";
//   - warps 2-5: epilogue.  Warp w reads TMEM lanes 32 (w % 4) .. +31 (= rows of the tile)
//     with tcgen05.ld, 32 columns at a time, hands the accumulator back ("tempty") after its
//     last read and writes C (f32 store, residual add, or the fused gate|up SiLU product in
//     fp16) while the tensor core already fills the other accumulator.
// Every mbarrier wait is bounded: a wait that gives up sets the error word and the CTA's abort
// flag, the other roles stop at their next wait, the producer waits (bounded) for its copies
// in flight, the MMA lane for its MMAs, and the CTA frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "gemm_epi.cuh"
#include "prefill.h"
#include "tcgen05.cuh"

namespace tptc {

namespace {

constexpr int BM = 128, BN = 256, BK = 64, kStages = 4;
constexpr int kABytes = BM * BK * 2;  // A tile of a stage (16 KB)
constexpr int kBBytes = BN * BK * 2;  // B tile of a stage (32 KB)
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr int kAccCols = BN;             // f32 accumulator columns of one tile
constexpr int kTmemCols = 2 * kAccCols;  // double-buffered: all 512 columns

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const __grid_constant__ GemmTcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[kStages], empty[kStages], tfull[2], tempty[2], drain;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (p.M + BM - 1) / BM, num_n = (p.N + BN - 1) / BN, tiles = num_m * num_n, nk = p.K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
        }
        mbar_init(&drain, 1);
        fence_mbar_init();
        abort_flag = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                const int m0 = (t % num_m) * BM, n0 = (t / num_m) * BN;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % kStages;
                    if (it >= kStages && !wait_or_abort(&empty[s], ((it / kStages) - 1) & 1, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * kStageBytes;
                    mbar_expect_tx(&full[s], kStageBytes);
                    tma_load_2d(st, &ta, kb * BK, m0, &full[s]);
                    tma_load_2d(st + kABytes, &tb, kb * BK, n0, &full[s]);
                }
            }
            // the copies still in flight land before the CTA exits
            for (uint32_t j = it > (uint32_t)kStages ? it - kStages : 0; j < it; j++)
                mbar_wait_bounded(&full[j % kStages], (j / kStages) & 1, p.err);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            const uint32_t idesc = mma_idesc(BM, BN);
            uint32_t it = 0, tc = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, tc++) {
                const uint32_t acc = tc & 1, d = tmem + acc * kAccCols;
                if (tc >= 2 && !wait_or_abort(&tempty[acc], ((tc >> 1) - 1) & 1, p.err, &abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % kStages;
                    if (!wait_or_abort(&full[s], (it / kStages) & 1, p.err, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(smem + s * kStageBytes), b = a + kABytes;
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        mma_f16(d, sw128_desc(a + 32 * k), sw128_desc(b + 32 * k), idesc, (kb | k) != 0);
                    mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
                }
                if (ok) mma_commit(&tfull[acc]);
            }
            // every MMA issued has completed before TMEM is freed
            mma_commit(&drain);
            mbar_wait_bounded(&drain, 0, p.err);
        }
    } else {  // epilogue warps 2..5
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        uint32_t tc = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, tc++) {
            const uint32_t acc = tc & 1;
            if (!wait_or_abort(&tfull[acc], (tc >> 1) & 1, p.err, &abort_flag)) break;
            tc_fence_after();
            const int m0 = (t % num_m) * BM, n0 = (t / num_m) * BN;
            const int row = m0 + 32 * q + lane;
            const uint32_t base = tmem + acc * kAccCols + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(base + (uint32_t)c0, r);
                if (c0 + 32 == BN) {  // accumulator read out: hand it back to the MMA lane
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[acc]);
                }
                store_cols<EPI>(p, row, n0 + c0, r);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024;
// more than half of an SM's shared memory: one CTA per SM, so the 512-column TMEM allocation
// never waits for another CTA
static_assert(kSmem > 116 * 1024, "gemm_tc relies on one resident CTA per SM");

int g_sms[64];

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!g_sms[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_sms[dev] = n;
    }
    return g_sms[dev];
}

}  // namespace

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_encode_mu;

cudaError_t get_encode() {
    std::lock_guard<std::mutex> lk(g_encode_mu);
    if (g_encode) return cudaSuccess;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return cudaSuccess;
}
}  // namespace

cudaError_t make_tmap_f16(CUtensorMap* map, const __half* ptr, int64_t rows, int64_t cols, int64_t ld,
                          int box_rows) {
    cudaError_t e = get_encode();
    if (e != cudaSuccess) return e;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(ptr), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t gemm_tc_init_device() {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemm_tc_kernel<GEMM_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem)))
        return e;
    if ((e = cudaFuncSetAttribute(gemm_tc_kernel<GEMM_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem)))
        return e;
    return cudaFuncSetAttribute(gemm_tc_kernel<GEMM_GLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
}

cudaError_t gemm_tc(int epi, const __half* a, int lda, const __half* b, int ldb, const GemmTcParams& p_in,
                    cudaStream_t st, bool pdl) {
    if (p_in.M <= 0 || p_in.N <= 0 || p_in.K <= 0 || p_in.K % BK || lda % 8 || ldb % 8 ||
        (reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15))
        return cudaErrorInvalidValue;
    if (epi == GEMM_GLU && p_in.N % 8) return cudaErrorInvalidValue;
    CUtensorMap ma, mb;
    cudaError_t e = make_tmap_f16(&ma, a, p_in.M, p_in.K, lda, BM);
    if (e == cudaSuccess) e = make_tmap_f16(&mb, b, p_in.N, p_in.K, ldb, BN);
    if (e != cudaSuccess) return e;
    const long tiles = (long)((p_in.M + BM - 1) / BM) * ((p_in.N + BN - 1) / BN);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min<long>(tiles, sm_count()));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (epi) {
    case GEMM_STORE: return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<GEMM_STORE>, ma, mb, p_in);
    case GEMM_RESID: return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<GEMM_RESID>, ma, mb, p_in);
    case GEMM_GLU: return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<GEMM_GLU>, ma, mb, p_in);
    }
    return cudaErrorInvalidValue;
}

}  // namespace tptc
