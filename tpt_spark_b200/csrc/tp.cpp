// tp.cpp -- NCCL communicator for tensor parallelism (the reference is single-device:
// wgpu_context.rs:38-45 picks one adapter; this is new).
//
// NCCL is loaded at run time with dlopen, not linked: a process that also uses PyTorch
// carries PyTorch's own libnccl.so.2, and the first copy loaded wins the symbol names.
// If a libnccl.so.2 is already resident it is reused; TPTC_NCCL_LIB names another file.
#include "tp.h"
#include "tptc.h"

#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "kernels.h"

namespace tptc {

namespace {

struct NcclApi {
    bool ok = false;
    std::string err;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = nullptr;
        const char* env = getenv("TPTC_NCCL_LIB");
        if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.err = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.GetErrorString &&
                 api.AllGather;
        if (!api.ok) api.err = "libnccl.so.2 lacks an expected symbol";
    });
    return api;
}

std::string nccl_msg(const char* what, ncclResult_t r) {
    return std::string(what) + ": " + (nccl().GetErrorString ? nccl().GetErrorString(r) : "error");
}

__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, size_t n) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] += y[i];
}

}  // namespace

int nccl_unique_id(void* out128) {
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    if (!nccl().ok) return TPTC_ERR_NCCL;
    ncclUniqueId id;
    if (nccl().GetUniqueId(&id) != ncclSuccess) return TPTC_ERR_NCCL;
    memcpy(out128, &id, sizeof(id));
    return TPTC_OK;
}

Tp::~Tp() {
    for (int r = 0; r < kTpMaxRanks; r++)
        if (peer_base[r]) cudaIpcCloseMemHandle(peer_base[r]);
    if (link_dev) cudaFree(link_dev);
    if (p2p_mem) cudaFree(p2p_mem);
    if (comm && nccl().ok) nccl().CommDestroy(static_cast<ncclComm_t>(comm));
}

// Own inbox allocation, its CUDA IPC handle exchanged with every rank over NCCL, the peers'
// allocations mapped into this process (peer access over NVLink), and the TpLink the
// kernels read.  Every rank calls it with the same dim and layer count.
Status Tp::init_p2p(int dim, int n_layers, const int* step, uint32_t wait_polls, cudaStream_t st) {
    if (size > kTpMaxRanks) return Status{TPTC_ERR_UNSUPPORTED, "peer-memory reduction supports up to 8 ranks"};
    const size_t bytes = tp_inbox_words(size, dim) * sizeof(unsigned long long);
    TPTC_CUDA_RET(cudaMalloc(&p2p_mem, bytes));
    TPTC_CUDA_RET(cudaMemsetAsync(p2p_mem, 0, bytes, st));  // epoch 0: no use has that tag
    cudaIpcMemHandle_t mine;
    TPTC_CUDA_RET(cudaIpcGetMemHandle(&mine, p2p_mem));
    void* d_handles = nullptr;
    TPTC_CUDA_RET(cudaMalloc(&d_handles, sizeof(cudaIpcMemHandle_t) * (size + 1)));
    uint8_t* d_all = static_cast<uint8_t*>(d_handles) + sizeof(cudaIpcMemHandle_t);
    TPTC_CUDA_RET(cudaMemcpyAsync(d_handles, &mine, sizeof(mine), cudaMemcpyHostToDevice, st));
    ncclResult_t nr = nccl().AllGather(d_handles, d_all, sizeof(mine), ncclUint8, static_cast<ncclComm_t>(comm), st);
    if (nr != ncclSuccess) {
        cudaFree(d_handles);
        return Status{TPTC_ERR_NCCL, nccl_msg("ncclAllGather", nr)};
    }
    std::vector<cudaIpcMemHandle_t> all(size);
    cudaError_t ce = cudaMemcpyAsync(all.data(), d_all, sizeof(mine) * size, cudaMemcpyDeviceToHost, st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
    cudaFree(d_handles);
    TPTC_CUDA_RET(ce);
    TpLink link = {};
    link.rank = rank;
    link.size = size;
    link.dim = dim;
    link.uses_per_step = 2 * n_layers + 1;  // o and down of every layer, then the argmax
    link.step = step;
    link.wait_polls = wait_polls ? wait_polls : kWaitPolls;
    for (int r = 0; r < size; r++) {
        void* base = p2p_mem;
        if (r != rank) {
            TPTC_CUDA_RET(cudaIpcOpenMemHandle(&base, all[r], cudaIpcMemLazyEnablePeerAccess));
            peer_base[r] = base;
        }
        link.inbox[r] = static_cast<unsigned long long*>(base);
    }
    TPTC_CUDA_RET(cudaMalloc(&link_dev, sizeof(TpLink)));
    TPTC_CUDA_RET(cudaMemcpyAsync(link_dev, &link, sizeof(link), cudaMemcpyHostToDevice, st));
    TPTC_CUDA_RET(cudaStreamSynchronize(st));
    return {};
}

Status Tp::init(int r, int s, const void* uid, cudaStream_t st) {
    (void)st;
    rank = r;
    size = s;
    if (!nccl().ok) return Status{TPTC_ERR_NCCL, nccl().err};
    if (!uid) return Status{TPTC_ERR_ARG, "tensor parallel context needs the ncclUniqueId of rank 0"};
    ncclUniqueId id;
    memcpy(&id, uid, sizeof(id));
    ncclComm_t c;
    ncclResult_t nr = nccl().CommInitRank(&c, s, id, r);
    if (nr != ncclSuccess) return Status{TPTC_ERR_NCCL, nccl_msg("ncclCommInitRank", nr)};
    comm = c;
    return {};
}

bool tp_shard(int which, int n_heads, int n_kv_heads, int head_dim, int dim, int ffn, int rank, int size, int& r0,
              int& r1, int& k0, int& k1) {
    if (size < 1 || rank < 0 || rank >= size || n_kv_heads <= 0 || n_heads % n_kv_heads) return false;
    // every rank keeps whole kv heads with their query group, and whole 256-blocks of ffn
    if (n_kv_heads % size || ffn % (256 * size)) return false;
    const int qd = n_heads / size * head_dim, kvd = n_kv_heads / size * head_dim, fl = ffn / size;
    if (size > 1 && qd % 256) return false;  // the o projection's K slice: whole quant blocks
    r0 = 0;
    k0 = 0;
    switch (which) {
    case TPTC_SHARD_Q: r0 = rank * qd; r1 = r0 + qd; k1 = dim; return true;
    case TPTC_SHARD_K:
    case TPTC_SHARD_V: r0 = rank * kvd; r1 = r0 + kvd; k1 = dim; return true;
    case TPTC_SHARD_O: r1 = dim; k0 = rank * qd; k1 = k0 + qd; return true;
    case TPTC_SHARD_GATE:
    case TPTC_SHARD_UP: r0 = rank * fl; r1 = r0 + fl; k1 = dim; return true;
    case TPTC_SHARD_DOWN: r1 = dim; k0 = rank * fl; k1 = k0 + fl; return true;
    }
    return false;
}

Status Tp::allreduce(float* b, size_t n, cudaStream_t st) {
    ncclResult_t nr = nccl().AllReduce(b, b, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st);
    if (nr != ncclSuccess) return Status{TPTC_ERR_NCCL, nccl_msg("ncclAllReduce", nr)};
    return {};
}

Status Tp::allgather(float* b, size_t count, cudaStream_t st) {
    ncclResult_t nr = nccl().AllGather(b + (size_t)rank * count, b, count, ncclFloat32, static_cast<ncclComm_t>(comm), st);
    if (nr != ncclSuccess) return Status{TPTC_ERR_NCCL, nccl_msg("ncclAllGather", nr)};
    return {};
}

Status Tp::allreduce_add(float* part, float* x, size_t n, cudaStream_t st) {
    Status s = allreduce(part, n, st);
    if (!s.ok()) return s;
    add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, part, n);
    TPTC_CUDA_RET(cudaGetLastError());
    return {};
}

}  // namespace tptc
