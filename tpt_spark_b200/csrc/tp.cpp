// tp.cpp -- NCCL communicator for tensor parallelism (the reference is single-device:
// wgpu_context.rs:38-45 picks one adapter; this is new).
//
// NCCL is loaded at run time with dlopen, not linked: a process that also uses PyTorch
// carries PyTorch's own libnccl.so.2, and the first copy loaded wins the symbol names.
// If a libnccl.so.2 is already resident it is reused; TPTC_NCCL_LIB names another file.
#include "tp.h"

#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

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
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.GetErrorString;
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
    if (comm && nccl().ok) nccl().CommDestroy(static_cast<ncclComm_t>(comm));
    if (buf) cudaFree(buf);
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

float* Tp::partial(size_t n) {
    if (n > buf_elems) {
        if (buf) cudaFree(buf);
        buf = nullptr;
        buf_elems = 0;
        if (cudaMalloc(&buf, n * sizeof(float)) != cudaSuccess) return nullptr;
        buf_elems = n;
    }
    return buf;
}

Status Tp::allreduce(float* b, size_t n, cudaStream_t st) {
    ncclResult_t nr = nccl().AllReduce(b, b, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), st);
    if (nr != ncclSuccess) return Status{TPTC_ERR_NCCL, nccl_msg("ncclAllReduce", nr)};
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
