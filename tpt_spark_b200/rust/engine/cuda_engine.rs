// cuda_engine.rs -- the B200 engine behind tpt-spark's LlmEngine trait, for
// src-tauri/src/engine/cuda_engine.rs (beside wgpu_engine.rs and candle_engine.rs).
//
// Not compiled here: there is no cargo or rustc on the machines this repository is built and
// tested on.  The library side it calls (libtptc, include/tptc.h) is built and tested here;
// tests/test_rust_ffi.py checks cuda_ffi.rs against include/tptc.h.
//
// The trait (engine/mod.rs:62-82): load / unload / is_loaded / model_info / infer.  All the
// numeric work happens in libtptc: tptc_infer runs the reference's gpu_infer protocol
// (wgpu_engine.rs:165-334) -- truncation, prefix reuse against the resident KV cache,
// batched prefill, repeat penalty, greedy or temperature / top-p selection on the device,
// EOS / max_tokens / context stops, and exactly one done event, cancellation included.  This
// file only tokenises, converts the parameters and forwards token events.
//
// Registration: `#[cfg(feature = "engine-cuda")] pub mod cuda_engine; pub mod cuda_ffi;` in
// engine/mod.rs, and in default_engine() (mod.rs:97-127), before the wgpu branch:
//
//     #[cfg(feature = "engine-cuda")]
//     if let Some(h) = cuda_engine::default_handle() { return h; }
//
// Cargo.toml (features, :80-91): `engine-cuda = ["dep:tokenizers"]`; build.rs calls
// build_cuda::compile_libtptc() under that feature (build_cuda.rs).

use std::ffi::{CStr, CString};
use std::os::raw::{c_char, c_int, c_void};
use std::path::{Path, PathBuf};
use std::sync::{Arc, Mutex};

use anyhow::{anyhow, bail, Result};
use tokenizers::Tokenizer;

use super::cuda_ffi::*;
use super::{EngineHandle, InferenceParams, LlmEngine, ModelInfo, TokenEvent};

/// The context pointer, owned; libtptc wants one host thread per context at a time, which the
/// Mutex below gives (the caller's EngineHandle mutex, mod.rs:95, already serialises calls).
struct Ctx(*mut tptc_ctx);
unsafe impl Send for Ctx {}

impl Drop for Ctx {
    fn drop(&mut self) {
        if !self.0.is_null() {
            unsafe { tptc_destroy(self.0) };
        }
    }
}

pub struct CudaEngine {
    ctx: Mutex<Ctx>,
    info: Option<ModelInfo>,
    tokenizer: Option<Tokenizer>,
    eos: Option<u32>,
}

/// Some(handle) when a CUDA device is present and a context could be made on it.
pub fn default_handle() -> Option<EngineHandle> {
    if unsafe { tptc_device_count() } <= 0 {
        return None;
    }
    let e = CudaEngine::new(0).ok()?;
    Some(Arc::new(tokio::sync::Mutex::new(Box::new(e) as Box<dyn LlmEngine>)))
}

fn status(rc: c_int, ctx: *const tptc_ctx) -> Result<()> {
    if rc >= 0 {
        return Ok(());
    }
    let msg = unsafe {
        let p = tptc_last_error(ctx);
        if p.is_null() { String::new() } else { CStr::from_ptr(p).to_string_lossy().into_owned() }
    };
    bail!("cuda engine error {rc}: {msg}")
}

fn c_string(buf: &[c_char]) -> String {
    let bytes: Vec<u8> = buf.iter().take_while(|&&c| c != 0).map(|&c| c as u8).collect();
    String::from_utf8_lossy(&bytes).into_owned()
}

/// tokenizer.json beside the model file, or in a directory named after it -- the two places
/// the wgpu engine looks (wgpu_engine.rs:892-906).
fn tokenizer_for(model: &Path) -> Result<Tokenizer> {
    let dir = model.parent().unwrap_or_else(|| Path::new("."));
    let stem = model.file_stem().and_then(|s| s.to_str()).unwrap_or("model");
    let candidates: [PathBuf; 2] = [dir.join("tokenizer.json"), dir.join(stem).join("tokenizer.json")];
    match candidates.iter().find(|p| p.exists()) {
        Some(p) => Tokenizer::from_file(p).map_err(|e| anyhow!("tokenizer load failed: {e}")),
        None => bail!("tokenizer.json not found next to {}", model.display()),
    }
}

/// The end-of-sequence id: the first of the usual end markers the vocabulary knows, else 2
/// (the same choice as the wgpu engine, wgpu_engine.rs:908-913).
fn eos_id(tok: &Tokenizer) -> u32 {
    ["<|eot_id|>", "<|end_of_text|>", "</s>", "<eos>", "[EOS]"]
        .iter()
        .find_map(|t| tok.token_to_id(t))
        .unwrap_or(2)
}

impl CudaEngine {
    pub fn new(device: c_int) -> Result<Self> {
        let mut ctx = std::ptr::null_mut();
        status(unsafe { tptc_create(device, 0, 1, std::ptr::null(), &mut ctx) }, ctx)?;
        Ok(Self { ctx: Mutex::new(Ctx(ctx)), info: None, tokenizer: None, eos: None })
    }

    fn raw(&self) -> *mut tptc_ctx {
        self.ctx.lock().expect("engine context poisoned").0
    }
}

impl LlmEngine for CudaEngine {
    fn load(&mut self, model_path: &str, on_progress: Option<&(dyn Fn(u32, u32) + Send + Sync)>) -> Result<ModelInfo> {
        extern "C" fn progress(done: u32, total: u32, user: *mut c_void) {
            let f = unsafe { &*(user as *const &(dyn Fn(u32, u32) + Send + Sync)) };
            f(done, total);
        }
        let ctx = self.raw();
        let path = CString::new(model_path)?;
        let rc = match on_progress {
            Some(ref f) => unsafe {
                tptc_load_gguf(ctx, path.as_ptr(), Some(progress), f as *const _ as *mut c_void)
            },
            None => unsafe { tptc_load_gguf(ctx, path.as_ptr(), None, std::ptr::null_mut()) },
        };
        status(rc, ctx)?;
        let mut mi: tptc_model_info = unsafe { std::mem::zeroed() };
        status(unsafe { tptc_get_model_info(ctx, &mut mi) }, ctx)?;
        let tok = tokenizer_for(Path::new(model_path))?;
        self.eos = Some(eos_id(&tok));
        self.tokenizer = Some(tok);
        let info = ModelInfo {
            name: c_string(&mi.name),
            path: model_path.to_string(),
            size_bytes: mi.size_bytes,
            backend: c_string(&mi.backend), // "cuda-sm100a" (or "cuda-sm100a-tpN")
        };
        self.info = Some(info.clone());
        Ok(info)
    }

    fn unload(&mut self) -> Result<()> {
        let ctx = self.raw();
        self.info = None;
        self.tokenizer = None;
        status(unsafe { tptc_unload(ctx) }, ctx)
    }

    fn is_loaded(&self) -> bool {
        unsafe { tptc_is_loaded(self.raw()) == 1 }
    }

    fn model_info(&self) -> Option<&ModelInfo> {
        self.info.as_ref()
    }

    fn infer(&self, params: &InferenceParams, on_token: &mut dyn FnMut(TokenEvent) -> Result<()>) -> Result<()> {
        let ctx = self.raw();
        let tok = self.tokenizer.as_ref().ok_or_else(|| anyhow!("no model loaded"))?;
        let text = match &params.system_prompt {
            Some(sys) => format!("{sys}\n{}", params.prompt),
            None => params.prompt.clone(),
        };
        let ids: Vec<u32> = tok.encode(text, true).map_err(|e| anyhow!("{e}"))?.get_ids().to_vec();
        let cp = tptc_infer_params {
            max_tokens: params.max_tokens,
            temperature: params.temperature,
            top_p: params.top_p,
            repeat_penalty: params.repeat_penalty,
            seed: 42, // the reference's LogitsProcessor::new(42, ..)
            eos_token_id: self.eos.map(|e| e as i64).unwrap_or(-1),
        };

        struct Sink<'a> {
            tok: &'a Tokenizer,
            on_token: &'a mut dyn FnMut(TokenEvent) -> Result<()>,
            error: Option<anyhow::Error>,
        }
        extern "C" fn forward_token(id: u32, done: c_int, user: *mut c_void) -> c_int {
            let sink = unsafe { &mut *(user as *mut Sink) };
            let token = if done != 0 { String::new() } else { sink.tok.decode(&[id], true).unwrap_or_default() };
            match (sink.on_token)(TokenEvent { token, done: done != 0 }) {
                Ok(()) => 0,
                Err(e) => {
                    // cancellation: libtptc still sends done = 1, then returns CANCELLED
                    if sink.error.is_none() {
                        sink.error = Some(e);
                    }
                    1
                }
            }
        }
        let mut sink = Sink { tok, on_token, error: None };
        let rc = unsafe {
            tptc_infer(ctx, ids.as_ptr(), ids.len() as c_int, &cp, forward_token, &mut sink as *mut Sink as *mut c_void)
        };
        if let Some(e) = sink.error {
            return Err(e); // the callback's error, after done (wgpu_engine.rs:297-300)
        }
        status(rc, ctx)
    }
}
