"""ctypes declarations of libtptc.so (include/tptc.h).

The product path is the compiled library: if ``lib/libtptc.so`` is missing this module
raises instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os

from ._build import lib_path

c_int, c_u32, c_i64, c_u64, c_f, c_d, c_vp = (ctypes.c_int, ctypes.c_uint32, ctypes.c_int64, ctypes.c_uint64,
                                             ctypes.c_float, ctypes.c_double, ctypes.c_void_p)

OK = 0
ERR_NAMES = {-1: "ARG", -2: "CUDA", -3: "IO", -4: "FORMAT", -5: "UNSUPPORTED", -6: "STATE", -7: "NCCL", -8: "OOM",
             -9: "CANCELLED", -10: "TIMEOUT"}


class ModelInfoC(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("path", ctypes.c_char * 1024), ("size_bytes", c_u64),
                ("backend", ctypes.c_char * 64), ("architecture", ctypes.c_char * 32),
                ("context_length", c_u32), ("n_layers", c_u32), ("n_heads", c_u32), ("n_kv_heads", c_u32),
                ("head_dim", c_u32), ("dim", c_u32), ("ffn", c_u32), ("vocab", c_u32),
                ("rope_freq_base", c_f), ("rope_scale", c_f), ("rms_eps", c_f), ("tied_embeddings", c_u32),
                ("tp_rank", c_u32), ("tp_size", c_u32), ("device_bytes", c_u64)]


class InferParamsC(ctypes.Structure):
    _fields_ = [("max_tokens", c_u32), ("temperature", c_f), ("top_p", c_f), ("repeat_penalty", c_f),
                ("seed", c_u64), ("eos_token_id", c_i64)]


TOKEN_CB = ctypes.CFUNCTYPE(c_int, c_u32, c_int, c_vp)
PROGRESS_CB = ctypes.CFUNCTYPE(None, c_u32, c_u32, c_vp)

# name -> (restype, argtypes); every symbol include/tptc.h declares.
SIGNATURES = {
    "tptc_create": (c_int, [c_int, c_int, c_int, c_vp, ctypes.POINTER(c_vp)]),
    "tptc_nccl_unique_id": (c_int, [c_vp]),
    "tptc_destroy": (None, [c_vp]),
    "tptc_last_error": (ctypes.c_char_p, [c_vp]),
    "tptc_version": (ctypes.c_char_p, []),
    "tptc_device_count": (c_int, []),
    "tptc_set_kv_dtype": (c_int, [c_vp, c_int]),
    "tptc_set_prefill_gemm_min": (c_int, [c_vp, c_int]),
    "tptc_set_prefill_fused": (c_int, [c_vp, c_int]),
    "tptc_set_tp_wait_polls": (c_int, [c_vp, ctypes.c_uint32]),
    "tptc_tp_shard": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp, c_vp]),
    "tptc_load_gguf": (c_int, [c_vp, ctypes.c_char_p, PROGRESS_CB, c_vp]),
    "tptc_unload": (c_int, [c_vp]),
    "tptc_is_loaded": (c_int, [c_vp]),
    "tptc_get_model_info": (c_int, [c_vp, ctypes.POINTER(ModelInfoC)]),
    "tptc_kv_reset": (c_int, [c_vp]),
    "tptc_kv_prefix_len": (c_int, [c_vp, c_vp, c_int]),
    "tptc_kv_len": (c_int, [c_vp]),
    "tptc_kv_truncate": (c_int, [c_vp, c_int]),
    "tptc_common_prefix_len": (c_int, [c_vp, c_int, c_vp, c_int]),
    "tptc_prefill": (c_int, [c_vp, c_vp, c_int, c_int, c_vp]),
    "tptc_decode": (c_int, [c_vp, c_u32, c_int, c_vp, c_vp]),
    "tptc_debug_trace": (c_int, [c_vp, c_u32, c_int, c_vp]),
    "tptc_decode_greedy": (c_int, [c_vp, c_u32, c_int, c_int, c_vp]),
    "tptc_infer": (c_int, [c_vp, c_vp, c_int, ctypes.POINTER(InferParamsC), TOKEN_CB, c_vp]),
    "tptc_last_device_ms": (c_int, [c_vp, ctypes.POINTER(c_d)]),
    "tptc_decode_kernels": (c_int, [c_vp]),
    "tptc_last_timing": (c_int, [c_vp, ctypes.POINTER(c_d), ctypes.POINTER(c_d), ctypes.POINTER(c_int),
                                 ctypes.POINTER(c_int)]),
    "tptc_dequant": (c_int, [c_int, c_vp, c_i64, c_vp, c_vp]),
    "tptc_quant_q8k": (c_int, [c_vp, c_i64, c_vp, c_vp]),
    "tptc_quant_q80": (c_int, [c_vp, c_i64, c_vp, c_vp]),
    "tptc_matrix_create": (c_int, [c_int, c_vp, c_int, c_int, c_int, ctypes.POINTER(c_vp)]),
    "tptc_matrix_destroy": (None, [c_vp]),
    "tptc_matrix_bytes": (c_i64, [c_vp]),
    "tptc_gemv": (c_int, [c_vp, c_vp, c_vp, c_vp]),
    "tptc_matrix_dequant_f16": (c_int, [c_vp, c_vp, c_vp]),
    "tptc_block_dots": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp]),
    "tptc_sample": (c_int, [c_vp, c_int, c_vp, c_f, c_f, c_f, c_u64, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "tptc_gemm_f16": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp]),
    "tptc_gemm_q": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp]),
    "tptc_attn_prefill": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_vp]),
    "tptc_attn_decode_workspace_bytes": (c_i64, [c_int, c_int, c_int, c_int]),
    "tptc_attn_decode": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp,
                                 c_vp, c_i64, c_vp]),
    "tptc_attn_decode_noalloc": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int,
                                         c_vp, c_vp]),
    "tptc_attn_decode_noalloc_status": (c_int, [c_vp, ctypes.POINTER(c_int)]),
}

_L = None


def lib() -> ctypes.CDLL:
    global _L
    if _L is None:
        path = lib_path("libtptc.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with tpt_spark_b200._build.build() "
                               "(the engine has no non-CUDA fallback)")
        L = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _L = L
    return _L


class EngineError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{ERR_NAMES.get(code, code)}] {msg}")
        self.code = code


def check(rc: int, ctx=None) -> int:
    if rc < 0:
        msg = lib().tptc_last_error(ctx)
        raise EngineError(rc, msg.decode(errors="replace") if msg else "")
    return rc
