"""ctypes binding of the CPU oracle (oracle/oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the checker and
by bench.py's CPU-baseline legs.  The product package never imports this module.

GGUF files are read here through gguf-py's GGUFReader (installed gguf 0.19), not through
the product's own parser, so the two read paths check each other.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q5_K = 2, 3, 6, 7, 10, 11, 13
Q8K_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (256,)), ("bsums", "<i2", (16,))])
assert Q8K_DTYPE.itemsize == 292


def build() -> str:
    src = os.path.join(HERE, "oracle.c")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


class _Desc(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("dim", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn", ctypes.c_int),
                ("vocab", ctypes.c_int), ("max_seq", ctypes.c_int), ("rope_base", ctypes.c_float),
                ("rms_eps", ctypes.c_float), ("rope_scale", ctypes.c_float),
                ("tensors", ctypes.POINTER(ctypes.c_void_p)), ("types", ctypes.POINTER(ctypes.c_int)),
                ("biases", ctypes.POINTER(ctypes.c_void_p)), ("rope_neox", ctypes.c_int),
                ("ffn_geglu", ctypes.c_int), ("embd_scale", ctypes.c_float),
                ("n_expert", ctypes.c_int), ("n_expert_used", ctypes.c_int), ("expert_ffn", ctypes.c_int),
                ("shared_ffn", ctypes.c_int), ("moe", ctypes.POINTER(ctypes.c_void_p)),
                ("moe_types", ctypes.POINTER(ctypes.c_int))]


_L = None


def lib():
    global _L
    if _L is None:
        L = ctypes.CDLL(build())
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.or_h2f.restype = ctypes.c_float
        L.or_h2f.argtypes = [ctypes.c_uint16]
        L.or_f2h.restype = ctypes.c_uint16
        L.or_f2h.argtypes = [ctypes.c_float]
        L.or_dequant.restype = i32
        L.or_dequant.argtypes = [i32, vp, i64, vp]
        L.or_quant_q8k.restype = None
        L.or_quant_q8k.argtypes = [vp, i64, vp]
        L.or_quant_q80.restype = None
        L.or_quant_q80.argtypes = [vp, i64, vp]
        L.or_block_dots.restype = i32
        L.or_block_dots.argtypes = [i32, vp, vp, i32, vp, vp]
        L.or_matmul.restype = i32
        L.or_matmul.argtypes = [i32, vp, i32, i32, vp, i32, vp]
        L.or_model_create.restype = vp
        L.or_model_create.argtypes = [ctypes.POINTER(_Desc)]
        L.or_model_destroy.restype = None
        L.or_model_destroy.argtypes = [vp]
        L.or_forward.restype = i32
        L.or_forward.argtypes = [vp, vp, i32, i32, vp, vp]
        L.or_argmax.restype = ctypes.c_uint32
        L.or_argmax.argtypes = [vp, i32]
        L.or_repeat_penalty.restype = None
        L.or_repeat_penalty.argtypes = [vp, i32, vp, i32, ctypes.c_float]
        L.or_set_trace.restype = None
        L.or_set_trace.argtypes = [vp]
        L.or_set_route_trace.restype = None
        L.or_set_route_trace.argtypes = [vp]
        L.or_set_threads.restype = None
        L.or_set_threads.argtypes = [i32]
        L.or_set_norm_lanes.restype = None
        L.or_set_norm_lanes.argtypes = [i32]
        L.or_set_simd.restype = None
        L.or_set_simd.argtypes = [i32]
        L.or_rope_table.restype = None
        L.or_rope_table.argtypes = [i32, i32, ctypes.c_float, ctypes.c_float, vp, vp]
        L.or_set_threads(os.cpu_count() or 1)
        _L = L
    return _L


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def set_simd(on: bool) -> None:
    """AVX2 quantised dots (default) or the scalar reference loops; both give the same bits."""
    lib().or_set_simd(1 if on else 0)


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def set_norm_lanes(n: int) -> None:
    """RMSNorm sum-of-squares order: 1 = candle's sequential sum (default); n > 1 = n
    interleaved partial sums added in order (an equally valid f32 evaluation)."""
    lib().or_set_norm_lanes(int(n))


def dequant(t: int, raw: np.ndarray, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw).view(np.uint8)
    y = np.empty(n, np.float32)
    assert lib().or_dequant(t, _p(raw), n, _p(y)) == 0
    return y


def quant_q8k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(x.size // 256, Q8K_DTYPE)
    lib().or_quant_q8k(_p(x), x.size, _p(out))
    return out


def quant_q80(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(x.size // 32 * 34, np.uint8)
    lib().or_quant_q80(_p(x), x.size, _p(out))
    return out


def quant_for(t: int, x: np.ndarray) -> np.ndarray:
    """Activation quantisation candle applies before the dot with a `t` weight."""
    return quant_q8k(x) if t in (Q2_K, Q3_K, Q4_K, Q5_K, Q6_K) else quant_q80(x)


def block_dots(t: int, wrow: np.ndarray, xq: np.ndarray, nb: int):
    wrow = np.ascontiguousarray(wrow).view(np.uint8)
    isum = np.zeros(nb, np.int32)
    msum = np.zeros(nb, np.int32)
    assert lib().or_block_dots(t, _p(wrow), _p(np.ascontiguousarray(xq)), nb, _p(isum), _p(msum)) == 0
    return isum, msum


def matmul(t: int, W: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    """y[m, N] = x[m, K] . W^T with candle QMatMul semantics."""
    W = np.ascontiguousarray(W)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, K)
    y = np.empty((x.shape[0], N), np.float32)
    assert lib().or_matmul(t, _p(W), N, K, _p(x), x.shape[0], _p(y)) == 0
    return y


def rope_table(max_seq: int, hd: int, base: float, scale: float = 1.0):
    c = np.empty((max_seq, hd // 2), np.float32)
    s = np.empty((max_seq, hd // 2), np.float32)
    lib().or_rope_table(max_seq, hd, base, scale, _p(c), _p(s))
    return c, s


def argmax(logits: np.ndarray) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().or_argmax(_p(logits), logits.size))


def repeat_penalty(logits: np.ndarray, seen: Sequence[int], penalty: float) -> np.ndarray:
    out = np.array(logits, np.float32, copy=True)
    s = np.ascontiguousarray(np.asarray(seen, np.uint32))
    lib().or_repeat_penalty(_p(out), out.size, _p(s), s.size, penalty)
    return out


class Model:
    """candle quantized_llama (architectures llama / mistral, with its mixture-of-experts block
    when the file has experts), quantized_qwen2 (qwen2: q / k / v biases, RoPE on head halves) or
    quantized_phi3 (phi3: fused attn_qkv and ffn_up, RoPE on head halves), or gemma (GEGLU,
    embeddings times sqrt(dim), RoPE on head halves) restated on CPU over a GGUF file (read with
    gguf-py)."""

    def __init__(self, path: str, max_seq: Optional[int] = None):
        import gguf

        self.reader = r = gguf.GGUFReader(path)

        def field(k, default=None):
            f = r.fields.get(k)
            if f is None:
                return default
            v = f.parts[f.data[0]]
            if f.types[0] == gguf.GGUFValueType.STRING:
                return bytes(v).decode()
            return v[0].item()

        arch = field("general.architecture", "llama")
        self.dim = field(f"{arch}.embedding_length")
        self.n_layers = field(f"{arch}.block_count")
        self.n_heads = field(f"{arch}.attention.head_count")
        self.n_kv_heads = field(f"{arch}.attention.head_count_kv", self.n_heads)
        self.head_dim = self.dim // self.n_heads
        self.ffn = field(f"{arch}.feed_forward_length")
        self.rope_base = field(f"{arch}.rope.freq_base", 10000.0)
        self.rms_eps = field(f"{arch}.attention.layer_norm_rms_epsilon", 1e-5)
        self.context_length = field(f"{arch}.context_length", 4096)
        tensors = {t.name: t for t in r.tensors}
        emb = tensors["token_embd.weight"]
        self.vocab = int(emb.shape[1])
        order = ["token_embd.weight", "output_norm.weight",
                 "output.weight" if "output.weight" in tensors else "token_embd.weight"]
        for i in range(self.n_layers):
            order += [f"blk.{i}.{n}.weight" for n in ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                                       "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")]
        # phi3 (candle quantized_phi3): attn_qkv rows are q | k | v and ffn_up rows gate | up; the
        # fused matmul is row by row the separate ones, so the row blocks stand in for them
        hd = self.dim // self.n_heads
        nq, nkv = self.n_heads * hd, self.n_kv_heads * hd
        blocks = {}
        for i in range(self.n_layers):
            p = f"blk.{i}."
            if p + "attn_qkv.weight" in tensors:
                t = tensors[p + "attn_qkv.weight"]
                for n, (r0, r1) in (("attn_q", (0, nq)), ("attn_k", (nq, nq + nkv)), ("attn_v", (nq + nkv, nq + 2 * nkv))):
                    blocks[p + n + ".weight"] = (np.ascontiguousarray(t.data[r0:r1]), int(t.tensor_type))
            if p + "ffn_gate.weight" not in tensors and p + "ffn_up.weight" in tensors:
                t = tensors[p + "ffn_up.weight"]
                blocks[p + "ffn_gate.weight"] = (np.ascontiguousarray(t.data[:self.ffn]), int(t.tensor_type))
                blocks[p + "ffn_up.weight"] = (np.ascontiguousarray(t.data[self.ffn:]), int(t.tensor_type))

        # mixture of experts: layers with a router; experts stacked (ffn_*_exps, [E][rows][K]) or
        # one tensor each (ffn_*.E); an optional shared expert (ffn_*_shexp)
        n_exp = field(f"{arch}.expert_count", 0) or 0
        self.n_expert = n_exp if n_exp > 1 else 0
        self.n_expert_used = (field(f"{arch}.expert_used_count", 2) or 0) if self.n_expert else 0
        self.expert_ffn = field(f"{arch}.expert_feed_forward_length", self.ffn) if self.n_expert else 0
        self.shared_ffn = 0
        moe_arrays, moe_types = [], []
        if self.n_expert:
            E = self.n_expert
            for i in range(self.n_layers):
                p = f"blk.{i}."
                if p + "ffn_gate_inp.weight" not in tensors:
                    moe_arrays += [None] * (4 + 3 * E)
                    moe_types += [0] * (4 + 3 * E)
                    continue
                rt = tensors[p + "ffn_gate_inp.weight"]
                moe_arrays.append(np.ascontiguousarray(rt.data))
                moe_types.append(int(rt.tensor_type))
                for e in range(E):
                    for stem in ("ffn_gate", "ffn_up", "ffn_down"):
                        if p + stem + "_exps.weight" in tensors:
                            t = tensors[p + stem + "_exps.weight"]
                            moe_arrays.append(np.ascontiguousarray(t.data[e]))
                        else:
                            t = tensors[f"{p}{stem}.{e}.weight"]
                            moe_arrays.append(np.ascontiguousarray(t.data))
                        moe_types.append(int(t.tensor_type))
                for stem in ("ffn_gate", "ffn_up", "ffn_down"):
                    n = p + stem + "_shexp.weight"
                    if n in tensors:
                        moe_arrays.append(np.ascontiguousarray(tensors[n].data))
                        moe_types.append(int(tensors[n].tensor_type))
                        if stem == "ffn_gate":
                            self.shared_ffn = int(tensors[n].shape[1])
                    else:
                        moe_arrays.append(None)
                        moe_types.append(0)
                # a MoE layer has no dense ffn tensors; its dense slots hold the router, unread
                router = moe_arrays[-(4 + 3 * E)], moe_types[-(4 + 3 * E)]
                for stem in ("ffn_gate", "ffn_up", "ffn_down"):
                    blocks.setdefault(p + stem + ".weight", router)

        def get(n):
            return blocks[n] if n in blocks else (np.ascontiguousarray(tensors[n].data), int(tensors[n].tensor_type))

        self._arrays = [get(n)[0] for n in order]
        self._types = [get(n)[1] for n in order]
        self.types = dict(zip(order, self._types))
        ptrs = (ctypes.c_void_p * len(order))(*[a.ctypes.data for a in self._arrays])
        tys = (ctypes.c_int * len(order))(*self._types)
        self.max_seq = max_seq or self.context_length
        self.arch = arch
        bnames = [f"blk.{i}.attn_{w}.bias" for i in range(self.n_layers) for w in ("q", "k", "v")]
        self._biases = [np.ascontiguousarray(tensors[n].data, np.float32) if n in tensors else None for n in bnames]
        barr = None
        if any(b is not None for b in self._biases):
            barr = (ctypes.c_void_p * len(bnames))(*[b.ctypes.data if b is not None else None for b in self._biases])
        d = _Desc(self.n_layers, self.dim, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn, self.vocab,
                  self.max_seq, self.rope_base, self.rms_eps, 1.0, ptrs, tys,
                  ctypes.cast(barr, ctypes.POINTER(ctypes.c_void_p)) if barr is not None else None,
                  1 if arch in ("qwen2", "phi3", "gemma") else 0)
        d.ffn_geglu = 1 if arch == "gemma" else 0
        d.embd_scale = float(np.float32(np.sqrt(np.float32(self.dim)))) if arch == "gemma" else 1.0
        marr = mtys = None
        if self.n_expert:
            self._moe = moe_arrays
            self._moe_types = moe_types
            marr = (ctypes.c_void_p * len(moe_arrays))(*[a.ctypes.data if a is not None else None for a in moe_arrays])
            mtys = (ctypes.c_int * len(moe_types))(*moe_types)
            d.n_expert, d.n_expert_used = self.n_expert, self.n_expert_used
            d.expert_ffn, d.shared_ffn = self.expert_ffn, self.shared_ffn
            d.moe = ctypes.cast(marr, ctypes.POINTER(ctypes.c_void_p))
            d.moe_types = ctypes.cast(mtys, ctypes.POINTER(ctypes.c_int))
        self._keep = (ptrs, tys, barr, marr, mtys)
        self.h = lib().or_model_create(ctypes.byref(d))

    def forward(self, tokens: Sequence[int], pos: int, want_hidden: bool = False):
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        logits = np.empty(self.vocab, np.float32)
        hid = np.empty(self.dim, np.float32) if want_hidden else None
        rc = lib().or_forward(self.h, _p(t), t.size, pos, _p(logits), _p(hid) if hid is not None else None)
        if rc != 0:
            raise ValueError("oracle forward rejected the input")
        return (logits, hid) if want_hidden else logits

    def forward_route(self, tokens: Sequence[int], pos: int):
        """forward() that also returns, per layer, the last position's routing margin: the
        router-logit gap between the last chosen expert and the best one left out (NaN for
        dense layers).  A small margin is a routing near-tie: evaluations that differ in the
        last bits may choose different experts there."""
        gaps = np.full(self.n_layers, np.nan, np.float32)
        lib().or_set_route_trace(_p(gaps))
        try:
            logits = self.forward(tokens, pos)
        finally:
            lib().or_set_route_trace(None)
        return logits, gaps

    def forward_trace(self, tokens: Sequence[int], pos: int):
        """forward() that also returns the per-layer trace [3 * n_layers, dim] of the last
        position: q after RoPE, attention output, residual stream after the layer."""
        tr = np.zeros((3 * self.n_layers, self.dim), np.float32)
        lib().or_set_trace(_p(tr))
        try:
            logits = self.forward(tokens, pos)
        finally:
            lib().or_set_trace(None)
        return logits, tr

    def greedy(self, prompt: Sequence[int], n_new: int) -> List[int]:
        logits = self.forward(prompt, 0)
        out, pos = [], len(prompt)
        for _ in range(n_new):
            tok = argmax(logits)
            out.append(tok)
            logits = self.forward([tok], pos)
            pos += 1
        return out

    def close(self):
        if self.h:
            lib().or_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
