// attn_noalloc.cu -- scratch for tptc_attn_decode_noalloc, the decode-attention entry point
// for callers that cannot allocate device memory (a host whose device memory is reserved up
// front by its own pool or another framework's allocator, or a decode loop that must not call
// cudaMalloc / cudaFree because they can synchronise the device).  It has no counterpart in
// the reference.
//
// The attention kernel needs scratch for its split partials and per-kv-head split counters
// (attn_scratch_layout: error word, counters, partials).  Here that scratch is one static
// device array of kAttnNoAllocScratchBytes (1 MiB) per device, so no cudaMalloc, cudaFree or
// allocating library routine is called on this path.
//
// What must start at zero: the split counters (the last CTA of each kv head resets its own
// counter, so a completed launch leaves them zero again, but a launch whose bounded wait gave
// up may not) and the error word.  Set-up, done by the first call on a device with that
// device current, looks the array's address up and zeroes the whole array, ordered on the
// caller's stream and waited for, before the first launch there; that first call belongs
// before any stream capture.  After that every call zeroes the error word and the counters
// (the array's head, up to the partials) on its stream before its launch, so a call never
// inherits a flagged or interrupted launch's state; the partials are always overwritten
// before they are read.  attn_noalloc_status reads the error word the last launch left.
//
// The array is shared by every call on a device.  Calls that may overlap on the GPU (launched
// on different streams without ordering between them, or from several host threads) race on
// it and produce wrong results; callers must serialise them.
#include <mutex>

#include "kernels.h"

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[tptc::kAttnNoAllocScratchBytes];

namespace tptc {

namespace {
constexpr int kMaxDevices = 256;
std::mutex g_mu;
uint8_t* g_scratch_ptr[kMaxDevices];  // set-up done when non-null
}  // namespace

cudaError_t attn_noalloc_scratch(int device, cudaStream_t st, uint8_t** out) {
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[device]) {
        // once per device, with that device current (the caller's current device)
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess) return e;
        e = cudaMemsetAsync(p, 0, kAttnNoAllocScratchBytes, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[device] = static_cast<uint8_t*>(p);
    }
    *out = g_scratch_ptr[device];
    return cudaSuccess;
}

cudaError_t attn_noalloc_status(int device, cudaStream_t st, int* code) {
    *code = 0;
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    uint8_t* p = g_scratch_ptr[device];
    if (!p) return cudaSuccess;  // no call on this device yet: nothing was flagged
    int word = 0;
    // the error word sits at offset 0 of the scratch (attn_scratch_layout); a 4-byte copy
    // into this stack variable, ordered after the stream's last launch
    cudaError_t e = cudaMemcpyAsync(&word, p, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return e;
    *code = word;
    if (word != 0) {  // a flagged launch: start the next one from a zeroed array
        e = cudaMemsetAsync(p, 0, kAttnNoAllocScratchBytes, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    }
    return e;
}

}  // namespace tptc
