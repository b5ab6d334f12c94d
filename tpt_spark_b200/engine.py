"""CudaEngine -- the Python mirror of tpt-spark's LlmEngine trait over libtptc.

Reference interface (src-tauri/src/engine/mod.rs):
    TokenEvent {token, done}                        :27-32
    InferenceParams {prompt, system_prompt, max_tokens, temperature, top_p,
                     repeat_penalty}, defaults 512 / 0.7 / 0.9 / 1.1  :35-59
    LlmEngine::{load, unload, is_loaded, model_info, infer}          :62-82
    ModelInfo {name, path, size_bytes, backend}     :85-92
The Rust host binds the same C ABI (tpt_spark_b200/rust/engine/cuda_ffi.rs); this module is
what the tests and the benchmark drive.  Prompts are token ids (the reference tokenises with tokenizer.json,
which is not on the numeric path); a string prompt is accepted when a tokenizer is given.
Errors raise EngineError (the reference returns anyhow::Error).
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import Callable, List, Optional, Sequence, Tuple, Union

import numpy as np

from . import _lib
from ._lib import EngineError, check, lib


@dataclasses.dataclass
class TokenEvent:
    token: str
    done: bool
    token_id: int = 0


@dataclasses.dataclass
class InferenceParams:
    prompt: Union[str, Sequence[int]] = ()
    system_prompt: Optional[str] = None
    max_tokens: int = 512
    temperature: float = 0.7
    top_p: float = 0.9
    repeat_penalty: float = 1.1
    seed: int = 42
    eos_token_id: Optional[int] = None


@dataclasses.dataclass
class ModelInfo:
    name: str
    path: str
    size_bytes: int
    backend: str
    architecture: str = "llama"
    context_length: int = 0
    n_layers: int = 0
    n_heads: int = 0
    n_kv_heads: int = 0
    head_dim: int = 0
    dim: int = 0
    ffn: int = 0
    vocab: int = 0
    rope_freq_base: float = 0.0
    rms_eps: float = 0.0
    tied_embeddings: bool = False
    tp_rank: int = 0
    tp_size: int = 1
    device_bytes: int = 0


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(lib().tptc_nccl_unique_id(buf))
    return buf.raw


SHARD_NAMES = ("q", "k", "v", "o", "gate", "up", "down")


def tp_shard(which: str, n_heads: int, n_kv_heads: int, head_dim: int, dim: int, ffn: int, rank: int,
             size: int) -> Tuple[int, int, int, int]:
    """(r0, r1, k0, k1): the rows and input columns of weight `which` that TP rank `rank` of
    `size` keeps (the loader's plan, tptc_tp_shard).  Host only."""
    v = [ctypes.c_int() for _ in range(4)]
    check(lib().tptc_tp_shard(SHARD_NAMES.index(which), n_heads, n_kv_heads, head_dim, dim, ffn, rank, size,
                              *[ctypes.byref(x) for x in v]))
    return tuple(x.value for x in v)


def device_count() -> int:
    return lib().tptc_device_count()


class CudaEngine:
    """engine/cuda_engine: the B200 engine behind the LlmEngine API."""

    def __init__(self, device: int = 0, tp_rank: int = 0, tp_size: int = 1, nccl_uid: Optional[bytes] = None,
                 tokenizer=None, kv_dtype: str = "f16"):
        """kv_dtype: "f16" (default, half the KV bytes per step) or "f32" (candle's precision)."""
        self._ctx = ctypes.c_void_p()
        uid = ctypes.create_string_buffer(nccl_uid, 128) if nccl_uid is not None else None
        check(lib().tptc_create(device, tp_rank, tp_size, uid, ctypes.byref(self._ctx)))
        if kv_dtype not in ("f16", "f32"):
            raise ValueError("kv_dtype must be 'f16' or 'f32'")
        self._check(lib().tptc_set_kv_dtype(self._ctx, 0 if kv_dtype == "f32" else 1))
        self.kv_dtype = kv_dtype
        self.device = device
        self.tokenizer = tokenizer
        self._info: Optional[ModelInfo] = None

    def set_tp_wait_polls(self, polls: int) -> None:
        """Tensor parallelism: reads of a peer's word before a decode step gives up on a rank
        that does not arrive (TPTC_ERR_TIMEOUT); 0 = the library default.  Before load."""
        self._check(lib().tptc_set_tp_wait_polls(self._ctx, int(polls)))

    def set_prefill_gemm_min(self, min_tokens: int) -> None:
        """Prompts of at least min_tokens run the batched tensor-core prefill (fp16 KV only);
        shorter ones, or all when min_tokens <= 0, go token by token (exact decode numerics)."""
        self._check(lib().tptc_set_prefill_gemm_min(self._ctx, int(min_tokens)))

    FUSED_MODES = {"never": 0, "auto": 1, "always": 2}

    def set_prefill_fused(self, mode: str) -> None:
        """How the batched prefill contracts quantised weights: "auto" (default: the
        fused-dequant GEMM where a wave model expects it to be faster), "always" or "never"
        (expand each matrix to fp16 first)."""
        if mode not in self.FUSED_MODES:
            raise ValueError(f"prefill fused mode must be one of {sorted(self.FUSED_MODES)}")
        self._check(lib().tptc_set_prefill_fused(self._ctx, self.FUSED_MODES[mode]))

    # -- lifecycle ---------------------------------------------------------------------------
    def close(self):
        if self._ctx:
            lib().tptc_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _check(self, rc: int) -> int:
        return check(rc, self._ctx)

    # -- LlmEngine ---------------------------------------------------------------------------
    def load(self, model_path: str, on_progress: Optional[Callable[[int, int], None]] = None) -> ModelInfo:
        cb = _lib.PROGRESS_CB((lambda d, t, u: on_progress(d, t)) if on_progress else (lambda d, t, u: None))
        self._check(lib().tptc_load_gguf(self._ctx, model_path.encode(), cb, None))
        self._info = self._read_info()
        return self._info

    def unload(self) -> None:
        self._check(lib().tptc_unload(self._ctx))
        self._info = None

    def is_loaded(self) -> bool:
        return bool(lib().tptc_is_loaded(self._ctx))

    def model_info(self) -> Optional[ModelInfo]:
        return self._info

    def _read_info(self) -> ModelInfo:
        c = _lib.ModelInfoC()
        self._check(lib().tptc_get_model_info(self._ctx, ctypes.byref(c)))
        return ModelInfo(c.name.decode(), c.path.decode(), c.size_bytes, c.backend.decode(), c.architecture.decode(),
                         c.context_length, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.dim, c.ffn, c.vocab,
                         c.rope_freq_base, c.rms_eps, bool(c.tied_embeddings), c.tp_rank, c.tp_size, c.device_bytes)

    def infer(self, params: InferenceParams, on_token: Callable[[TokenEvent], None]) -> None:
        """LlmEngine::infer. on_token may raise to cancel (the reference's Err from on_token):
        the engine then emits done=True and this call raises EngineError(CANCELLED)."""
        ids = self._encode(params)
        p = _lib.InferParamsC(params.max_tokens, params.temperature, params.top_p, params.repeat_penalty,
                              params.seed & (2**64 - 1), -1 if params.eos_token_id is None else params.eos_token_id)
        raised: List[BaseException] = []

        def cb(tok, done, user):
            ev = TokenEvent("" if done else self._decode_token(tok), bool(done), int(tok))
            try:
                on_token(ev)
            except BaseException as e:  # cancellation
                if not done:
                    raised.append(e)
                    return 1
            return 0

        arr = (ctypes.c_uint32 * len(ids))(*ids)
        ccb = _lib.TOKEN_CB(cb)
        rc = lib().tptc_infer(self._ctx, arr, len(ids), ctypes.byref(p), ccb, None)
        if rc < 0 and raised and rc == -9:
            raise EngineError(rc, f"cancelled: {raised[0]!r}")
        self._check(rc)

    def last_timing(self) -> Tuple[float, float, int, int]:
        a, b, c, d = ctypes.c_double(), ctypes.c_double(), ctypes.c_int(), ctypes.c_int()
        self._check(lib().tptc_last_timing(self._ctx, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c),
                                           ctypes.byref(d)))
        return a.value, b.value, c.value, d.value

    def decode_kernels(self) -> int:
        """Kernel launches in one decode step (kernel nodes of the step's CUDA graph)."""
        return self._check(lib().tptc_decode_kernels(self._ctx))

    def last_device_ms(self) -> float:
        """CUDA-event time of the last prefill / decode_greedy on the engine's stream."""
        v = ctypes.c_double()
        self._check(lib().tptc_last_device_ms(self._ctx, ctypes.byref(v)))
        return v.value

    # -- lower-level forward API -------------------------------------------------------------
    def kv_reset(self) -> None:
        self._check(lib().tptc_kv_reset(self._ctx))

    def kv_truncate(self, n: int) -> None:
        self._check(lib().tptc_kv_truncate(self._ctx, n))

    def kv_len(self) -> int:
        return self._check(lib().tptc_kv_len(self._ctx))

    def kv_prefix_len(self, ids: Sequence[int]) -> int:
        arr = np.ascontiguousarray(np.asarray(ids, np.uint32))
        return self._check(lib().tptc_kv_prefix_len(self._ctx, arr.ctypes.data, arr.size))

    def _need_model(self):
        if self._info is None:
            raise EngineError(-6, "no model loaded")

    def prefill(self, ids: Sequence[int], start_pos: Optional[int] = None, want_logits: bool = True):
        self._need_model()
        arr = np.ascontiguousarray(np.asarray(ids, np.uint32))
        start = self.kv_len() if start_pos is None else start_pos
        out = np.empty(self._info.vocab, np.float32) if want_logits else None
        self._check(lib().tptc_prefill(self._ctx, arr.ctypes.data, arr.size, start,
                                       out.ctypes.data if out is not None else None))
        return out

    def decode(self, token: int, pos: int, want_logits: bool = True):
        self._need_model()
        out = np.empty(self._info.vocab, np.float32) if want_logits else None
        am = ctypes.c_uint32()
        self._check(lib().tptc_decode(self._ctx, token, pos, out.ctypes.data if out is not None else None,
                                      ctypes.byref(am)))
        return (out, am.value) if want_logits else am.value

    def debug_trace(self, token: int, pos: int) -> np.ndarray:
        """Per-layer trace of one decode step: [3 * n_layers, dim] (q, attention, residual)."""
        self._need_model()
        tr = np.zeros((3 * self._info.n_layers, self._info.dim), np.float32)
        self._check(lib().tptc_debug_trace(self._ctx, token, pos, tr.ctypes.data))
        return tr

    def decode_greedy(self, token: int, pos: int, n: int) -> List[int]:
        out = np.empty(n, np.uint32)
        self._check(lib().tptc_decode_greedy(self._ctx, token, pos, n, out.ctypes.data))
        return out.tolist()

    # -- tokens ------------------------------------------------------------------------------
    def _encode(self, params: InferenceParams) -> List[int]:
        if isinstance(params.prompt, str):
            if self.tokenizer is None:
                raise EngineError(-1, "a string prompt needs a tokenizer (tokenizer.json beside the .gguf)")
            text = params.prompt if not params.system_prompt else params.system_prompt + "\n" + params.prompt
            return list(self.tokenizer.encode(text).ids)
        return [int(t) for t in params.prompt]

    def _decode_token(self, tok: int) -> str:
        if self.tokenizer is not None:
            return self.tokenizer.decode([tok])
        return str(tok)
