// prefill.h -- batched prompt processing (prefill) kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tptc {

cudaError_t prefill_init_device();

}  // namespace tptc
