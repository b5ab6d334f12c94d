// tp.h -- Megatron tensor parallelism: one context per GPU, column-parallel q/k/v/gate/up,
// row-parallel o/down.  The decode step reduces the row-parallel outputs over NVLink peer
// memory (TpLink, gemv.cuh); the batched prefill sum-allreduces them with NCCL.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv.cuh"

namespace tptc {

struct Tp {
    int rank = 0, size = 1;
    void* comm = nullptr;  // ncclComm_t
    ~Tp();
    Status init(int rank, int size, const void* uid, cudaStream_t st);
    // x[n] += sum over ranks of part[n] (every rank ends with the same x).
    Status allreduce_add(float* part, float* x, size_t n, cudaStream_t st);
    // Sum-allreduce in place.
    Status allreduce(float* buf, size_t n, cudaStream_t st);
    // In-place all-gather: rank r's `count` floats at buf + r * count, every rank's after.
    Status allgather(float* buf, size_t count, cudaStream_t st);
    // Peer-memory reduction of the decode step's row-parallel projections and the argmax
    // exchange (gemv.cuh TpLink); wait_polls 0 keeps the library's default wait bound.
    Status init_p2p(int dim, int n_layers, const int* step, uint32_t wait_polls, cudaStream_t st);
    void* p2p_mem = nullptr;                 // own inbox
    void* peer_base[kTpMaxRanks] = {};       // peers' allocations mapped here
    TpLink* link_dev = nullptr;              // device copy the kernels read
};

int nccl_unique_id(void* out128);

// The rows [r0, r1) and input columns [k0, k1) of weight `which` (TPTC_SHARD_*) that rank
// `rank` of `size` keeps; false when the model does not split evenly.
bool tp_shard(int which, int n_heads, int n_kv_heads, int head_dim, int dim, int ffn, int rank, int size, int& r0,
              int& r1, int& k0, int& k1);

}  // namespace tptc
