// prefill.cu -- prompt processing.
#include <vector>

#include "engine.h"
#include "prefill.h"

namespace tptc {

cudaError_t prefill_init_device() { return gemm_tc_init_device(); }

// Prompt positions one at a time through the decode graph (the reference's prefill loop,
// wgpu_engine.rs:254-261); the last step's logits are returned.
Status Engine::run_prefill_batched(const uint32_t* ids, int n, int start_pos, float* last_logits) {
    for (int i = 0; i < n; i++) {
        uint32_t am;
        Status s = decode(ids[i], start_pos + i, i + 1 == n ? last_logits : nullptr, &am);
        if (!s.ok()) return s;
    }
    return {};
}

}  // namespace tptc
