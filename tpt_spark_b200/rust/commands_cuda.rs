// commands_cuda.rs -- what tpt-spark's Tauri commands need to know about the CUDA engine
// (the API-integration row: run_benchmark / Crucible export and get_system_info).
//
// Not compiled here: there is no cargo or rustc on the machines this repository is built and
// tested on.
//
// Where each function is used in src-tauri/src/commands.rs:
//   * is_gpu_backend: the Crucible record's GPU test (commands.rs:455-459) classifies a result
//     as GPU by substrings of the engine's backend string; the CUDA engine reports
//     "cuda-sm100a" or "cuda-sm100a-tpN" (ModelInfo.backend), which the test must accept:
//     `let gpu_name = if commands_cuda::is_gpu_backend(&result.backend) { ... }`.
//   * system_backend: get_system_info's cfg ladder (commands.rs:649-655) names the compiled
//     engine; with the engine-cuda feature it reports "cuda" ahead of the wgpu / candle arms:
//     `backend: commands_cuda::system_backend(),`.
// run_benchmark itself (commands.rs:487-597) needs no change: it drives LlmEngine::infer with
// greedy parameters, which tptc_infer serves on the device.

/// Whether an engine backend string names a GPU engine: the substrings the reference already
/// tests ("wgpu", "tpt-gpu"), plus "cuda".
pub fn is_gpu_backend(backend: &str) -> bool {
    ["wgpu", "tpt-gpu", "cuda"].iter().any(|k| backend.contains(k))
}

/// The engine family compiled in, most capable first (get_system_info).
pub fn system_backend() -> String {
    if cfg!(feature = "engine-cuda") {
        "cuda".to_string()
    } else if cfg!(feature = "engine-wgpu") {
        "wgpu".to_string()
    } else if cfg!(feature = "engine-candle") {
        "candle-cpu".to_string()
    } else {
        "stub".to_string()
    }
}
