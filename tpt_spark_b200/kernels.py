"""Kernel-level entry points of libtptc over device memory.

Device buffers are passed as raw pointers; tests and the benchmark allocate them with
torch (plumbing only -- the arithmetic runs in libtptc's kernels).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from ._lib import check, lib

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q5_K = 2, 3, 6, 7, 10, 11, 13


def _ptr(t) -> int:
    return t if isinstance(t, int) else t.data_ptr()


def dequant(ggml_type: int, d_blocks, n: int, d_out, stream: Optional[int] = None) -> None:
    check(lib().tptc_dequant(ggml_type, _ptr(d_blocks), n, _ptr(d_out), stream))


def quant_q8k(d_x, k: int, d_out, stream: Optional[int] = None) -> None:
    check(lib().tptc_quant_q8k(_ptr(d_x), k, _ptr(d_out), stream))


def quant_q80(d_x, k: int, d_out, stream: Optional[int] = None) -> None:
    check(lib().tptc_quant_q80(_ptr(d_x), k, _ptr(d_out), stream))


class Matrix:
    """A weight matrix [N x K] in the engine's device layout, made from raw GGUF bytes."""

    def __init__(self, ggml_type: int, raw: np.ndarray, N: int, K: int):
        raw = np.ascontiguousarray(raw).view(np.uint8)
        self._h = ctypes.c_void_p()
        check(lib().tptc_matrix_create(ggml_type, raw.ctypes.data, 0, N, K, ctypes.byref(self._h)))
        self.type, self.N, self.K = ggml_type, N, K

    @property
    def nbytes(self) -> int:
        return lib().tptc_matrix_bytes(self._h)

    def gemv(self, d_x, d_y, stream: Optional[int] = None) -> None:
        check(lib().tptc_gemv(self._h, _ptr(d_x), _ptr(d_y), stream))

    def gemm(self, d_a, d_c, M: int, stream: Optional[int] = None) -> None:
        """C[M x N] (f32) = A[M x K] (fp16) . W^T with the dequantisation fused (tptc_gemm_q)."""
        check(lib().tptc_gemm_q(self._h, _ptr(d_a), _ptr(d_c), M, stream))

    def dequant_f16(self, d_out, stream: Optional[int] = None) -> None:
        """The matrix as dense row-major fp16 [N x K] (the prefill GEMM operand)."""
        check(lib().tptc_matrix_dequant_f16(self._h, _ptr(d_out), stream))

    def block_dots(self, d_x, d_isum, d_msum=None, stream: Optional[int] = None) -> None:
        check(lib().tptc_block_dots(self._h, _ptr(d_x), _ptr(d_isum), _ptr(d_msum) if d_msum is not None else None,
                                    stream))

    def close(self):
        if self._h:
            lib().tptc_matrix_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def attn_decode_workspace_bytes(n_heads: int, n_kv: int, head_dim: int, max_seq: int) -> int:
    return check(lib().tptc_attn_decode_workspace_bytes(n_heads, n_kv, head_dim, max_seq))


def attn_decode(d_q, d_kraw, d_kcache, d_vcache, kv_type: int, d_rope_cos, d_rope_sin, d_pos, n_heads: int,
                n_kv: int, head_dim: int, max_seq: int, d_out, d_workspace, workspace_bytes: int,
                stream: Optional[int] = None) -> None:
    """One decode-step attention (tptc_attn_decode); every buffer a device pointer or tensor."""
    check(lib().tptc_attn_decode(_ptr(d_q), _ptr(d_kraw), _ptr(d_kcache), _ptr(d_vcache), kv_type, _ptr(d_rope_cos),
                                 _ptr(d_rope_sin), _ptr(d_pos), n_heads, n_kv, head_dim, max_seq, _ptr(d_out),
                                 _ptr(d_workspace), workspace_bytes, stream))


def attn_decode_noalloc(d_q, d_kraw, d_kcache, d_vcache, kv_type: int, d_rope_cos, d_rope_sin, d_pos, n_heads: int,
                        n_kv: int, head_dim: int, max_seq: int, d_out, stream: Optional[int] = None) -> None:
    """tptc_attn_decode_noalloc: as attn_decode, with the library's static scratch (no allocation)."""
    check(lib().tptc_attn_decode_noalloc(_ptr(d_q), _ptr(d_kraw), _ptr(d_kcache), _ptr(d_vcache), kv_type,
                                         _ptr(d_rope_cos), _ptr(d_rope_sin), _ptr(d_pos), n_heads, n_kv, head_dim,
                                         max_seq, _ptr(d_out), stream))


def attn_decode_noalloc_status(stream: Optional[int] = None) -> int:
    """tptc_attn_decode_noalloc_status: the error word of the last no-alloc attention launch on
    the current device (0, or a negative TPTC_ERR_* code), after `stream` finishes."""
    code = ctypes.c_int()
    check(lib().tptc_attn_decode_noalloc_status(stream, ctypes.byref(code)))
    return code.value


def sample(d_logits, vocab: int, d_counts, penalty: float, temperature: float, top_p: float, seed: int, d_step,
           d_scratch, d_out, d_dbg=None, stream: Optional[int] = None) -> None:
    """The engine's device next-token selection (tptc_sample): repeat penalty over d_counts,
    argmax or softmax(x / T) + top-p + one seeded draw; the token lands in d_out[0]."""
    check(lib().tptc_sample(_ptr(d_logits), vocab, _ptr(d_counts) if d_counts is not None else None, penalty,
                            temperature, top_p, seed, _ptr(d_step) if d_step is not None else None, _ptr(d_scratch),
                            _ptr(d_out), _ptr(d_dbg) if d_dbg is not None else None, stream))


def gemm_f16(d_a, d_b, d_c, M: int, N: int, K: int, stream: Optional[int] = None) -> None:
    """C[M x N] (f32) = A[M x K] . B[N x K]^T on the tensor cores (fp16 row-major A and B)."""
    check(lib().tptc_gemm_f16(_ptr(d_a), _ptr(d_b), _ptr(d_c), M, N, K, stream))


def attn_prefill(d_q, d_kcache, d_vcache, d_out, T: int, start: int, n_heads: int, n_kv: int, head_dim: int,
                 max_seq: int, stream: Optional[int] = None) -> None:
    """Causal GQA attention of T prompt rows at positions start.. over an fp16 KV cache."""
    check(lib().tptc_attn_prefill(_ptr(d_q), _ptr(d_kcache), _ptr(d_vcache), _ptr(d_out), T, start, n_heads, n_kv,
                                  head_dim, max_seq, stream))
