"""Synthetic GGUF models for tests and benchmarks.

The benchmark configurations are random-init Llama-architecture decoders: linear weights
drawn N(0, 0.02) from a seed, RMSNorm gains 1.0, quantised to GGUF Q4_K / Q5_K / Q6_K / Q4_0 /
Q5_0 / Q8_0 or stored as F16.  There is no network and no checkpoint, so the files are generated here.

The GGUF v3 container written by :func:`write_gguf` carries the metadata keys that the
reference reads: ``general.architecture`` and the ``llama.*`` keys of
src-tauri/src/engine/wgpu_loader.rs:305-406 (context_length, block_count, head_count,
head_count_kv, embedding_length, vocab_size, rope.freq_base, feed_forward_length,
layer_norm_rms_epsilon) plus ``llama.rope.dimension_count``, which candle's
quantized_llama requires.  Tensor names follow llama.cpp (token_embd, blk.N.attn_q, ...),
dims are stored innermost first ([K, N] for an N x K weight).  Block encoding and the
random draw run in C (``csrc/synth.c`` -> ``lib/libtptsynth.so``).
"""
from __future__ import annotations

import ctypes
import dataclasses
import os
import struct
from typing import Callable, Dict, List, Optional, Tuple

import numpy as np

from ._build import lib_path

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
Q4_0, Q5_0, Q5_K, Q2_K, Q3_K, Q4_1, Q5_1 = 2, 6, 13, 10, 11, 3, 7
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q4_0: (32, 18),
         Q5_0: (32, 22), Q5_K: (256, 176), Q2_K: (256, 84), Q3_K: (256, 110), Q4_1: (32, 20), Q5_1: (32, 24)}
TYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", Q4_0: "Q4_0", Q5_0: "Q5_0",
              Q5_K: "Q5_K", Q2_K: "Q2_K", Q3_K: "Q3_K", Q4_1: "Q4_1", Q5_1: "Q5_1"}
ALIGN = 32


def type_bytes(t: int, n: int) -> int:
    be, bb = BLOCK[t]
    assert n % be == 0, (t, n)
    return n // be * bb


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    """Shape and storage types of a synthetic Llama-architecture model."""

    name: str
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    vocab: int
    rope_base: float
    context_length: int
    rms_eps: float = 1e-5
    tied: bool = False
    default_type: int = Q4_K
    overrides: Tuple[Tuple[str, int], ...] = ()  # (tensor-kind, type), kinds below
    embd_type: Optional[int] = None
    output_type: Optional[int] = None
    norm_std: float = 0.0  # 0: gains exactly 1.0 (the configs); >0: 1 + N(0, norm_std)
    weight_std: float = 0.02
    arch: str = "llama"     # general.architecture; "qwen2" / "phi3" rotate head halves (NEOX);
                            # "phi3" stores attn_qkv (rows q | k | v) and ffn_up (rows gate | up) fused
    qkv_bias: bool = False  # f32 attn_q / attn_k / attn_v biases, N(0, bias_std)
    bias_std: float = 0.1
    # mixture of experts: n_expert > 1 makes the layers in moe_layers (None: all) MoE layers
    # with a router (ffn_gate_inp, router_type) and n_expert experts of expert_ffn rows, stored
    # stacked (ffn_*_exps, llama.cpp) or one tensor each (ffn_*.E, candle's names), plus a
    # shared expert of shared_ffn rows when > 0
    n_expert: int = 0
    n_expert_used: int = 0
    expert_ffn: int = 0
    moe_layers: Optional[Tuple[int, ...]] = None
    stacked_experts: bool = True
    shared_ffn: int = 0
    router_type: int = F32
    router_std: float = 0.02

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    def is_moe_layer(self, i: int) -> bool:
        return self.n_expert > 1 and (self.moe_layers is None or i in self.moe_layers)

    def type_of(self, kind: str) -> int:
        if kind.endswith("norm") or kind == "bias":
            return F32
        if kind == "ffn_gate_inp":
            return self.router_type
        kind = kind.replace("_exps", "").replace("_shexp", "")  # experts take the dense kinds' types
        if kind == "token_embd":
            return self.embd_type if self.embd_type is not None else self.default_type
        if kind == "output":
            return self.output_type if self.output_type is not None else self.default_type
        return dict(self.overrides).get(kind, self.default_type)

    def tensors(self) -> List[Tuple[str, str, List[int]]]:
        """(name, kind, ne) in file order; ne innermost first."""
        d, hd = self.dim, self.head_dim
        out = [("token_embd.weight", "token_embd", [d, self.vocab])]
        for i in range(self.n_layers):
            p = f"blk.{i}."
            out += [(p + "attn_norm.weight", "attn_norm", [d])]
            if self.arch == "phi3":
                out += [(p + "attn_qkv.weight", "attn_qkv", [d, (self.n_heads + 2 * self.n_kv_heads) * hd])]
            else:
                out += [
                    (p + "attn_q.weight", "attn_q", [d, self.n_heads * hd]),
                    (p + "attn_k.weight", "attn_k", [d, self.n_kv_heads * hd]),
                    (p + "attn_v.weight", "attn_v", [d, self.n_kv_heads * hd]),
                ]
            if self.qkv_bias:
                out += [(p + "attn_q.bias", "bias", [self.n_heads * hd]),
                        (p + "attn_k.bias", "bias", [self.n_kv_heads * hd]),
                        (p + "attn_v.bias", "bias", [self.n_kv_heads * hd])]
            out += [(p + "attn_output.weight", "attn_output", [self.n_heads * hd, d]),
                    (p + "ffn_norm.weight", "ffn_norm", [d])]
            if self.is_moe_layer(i):
                E, ef = self.n_expert, self.expert_ffn
                out += [(p + "ffn_gate_inp.weight", "ffn_gate_inp", [d, E])]
                if self.stacked_experts:
                    out += [(p + "ffn_gate_exps.weight", "ffn_gate_exps", [d, ef, E]),
                            (p + "ffn_up_exps.weight", "ffn_up_exps", [d, ef, E]),
                            (p + "ffn_down_exps.weight", "ffn_down_exps", [ef, d, E])]
                else:
                    for e in range(E):
                        out += [(p + f"ffn_gate.{e}.weight", "ffn_gate", [d, ef]),
                                (p + f"ffn_up.{e}.weight", "ffn_up", [d, ef]),
                                (p + f"ffn_down.{e}.weight", "ffn_down", [ef, d])]
                if self.shared_ffn:
                    sf = self.shared_ffn
                    out += [(p + "ffn_gate_shexp.weight", "ffn_gate_shexp", [d, sf]),
                            (p + "ffn_up_shexp.weight", "ffn_up_shexp", [d, sf]),
                            (p + "ffn_down_shexp.weight", "ffn_down_shexp", [sf, d])]
            elif self.arch == "phi3":
                out += [(p + "ffn_up.weight", "ffn_up", [d, 2 * self.ffn])]
            else:
                out += [(p + "ffn_gate.weight", "ffn_gate", [d, self.ffn]),
                        (p + "ffn_up.weight", "ffn_up", [d, self.ffn])]
            if not self.is_moe_layer(i):
                out += [(p + "ffn_down.weight", "ffn_down", [self.ffn, d])]
        out.append(("output_norm.weight", "output_norm", [d]))
        if not self.tied:
            out.append(("output.weight", "output", [d, self.vocab]))
        return out


Q4_K_M = (("attn_v", Q6_K), ("ffn_down", Q6_K))

# The five benchmark configurations (C1 is a single matrix, see GEMV_C1).
CONFIGS: Dict[str, ModelConfig] = {
    "c2_llama1b_q4km": ModelConfig(
        "c2_llama1b_q4km", dim=2048, n_layers=16, n_heads=32, n_kv_heads=8, ffn=8192,
        vocab=128256, rope_base=500000.0, context_length=2048, tied=True,
        overrides=Q4_K_M, embd_type=Q6_K),
    "c3_mistral7b_q8_0": ModelConfig(
        "c3_mistral7b_q8_0", dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn=14336,
        vocab=32000, rope_base=10000.0, context_length=4096, default_type=Q8_0),
    "c4_phi3mini_f16": ModelConfig(
        "c4_phi3mini_f16", dim=3072, n_layers=32, n_heads=32, n_kv_heads=32, ffn=8192,
        vocab=32064, rope_base=10000.0, context_length=4096, default_type=F16),
    "c5_llama8b_q4km": ModelConfig(
        "c5_llama8b_q4km", dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn=14336,
        vocab=128256, rope_base=500000.0, context_length=9216, overrides=Q4_K_M,
        embd_type=Q4_K, output_type=Q6_K),
}

# Further bench workloads (bench.py --workload): Mixtral 8x7B's layer shape for the
# mixture-of-experts decode path, 4 of its 32 layers (8 experts of 14336 rows, 2 per token,
# llama.cpp's stacked expert tensors, Q4_K_M mix, f32 router).
WORKLOADS: Dict[str, ModelConfig] = {
    "mixtral8x7b_l4_q4km": ModelConfig(
        "mixtral8x7b_l4_q4km", dim=4096, n_layers=4, n_heads=32, n_kv_heads=8, ffn=14336, vocab=32000,
        rope_base=1000000.0, context_length=4096, overrides=Q4_K_M, embd_type=Q4_K, output_type=Q6_K,
        n_expert=8, n_expert_used=2, expert_ffn=14336),
}

# Small models with the same code paths, for parity tests that the CPU oracle finishes
# in seconds.
TINY: Dict[str, ModelConfig] = {
    "tiny_q4km": ModelConfig(
        "tiny_q4km", dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn=512, vocab=512,
        rope_base=10000.0, context_length=512, overrides=Q4_K_M, embd_type=Q4_K,
        output_type=Q6_K, norm_std=0.1),
    "tiny_q4km_tied": ModelConfig(
        "tiny_q4km_tied", dim=256, n_layers=2, n_heads=4, n_kv_heads=1, ffn=768, vocab=384,
        rope_base=500000.0, context_length=512, tied=True, overrides=Q4_K_M, embd_type=Q6_K),
    "tiny_q8_0": ModelConfig(
        "tiny_q8_0", dim=256, n_layers=2, n_heads=2, n_kv_heads=2, ffn=512, vocab=320,
        rope_base=10000.0, context_length=512, default_type=Q8_0, norm_std=0.1),
    "tiny_f16": ModelConfig(
        "tiny_f16", dim=768, n_layers=2, n_heads=8, n_kv_heads=8, ffn=512, vocab=320,
        rope_base=10000.0, context_length=512, default_type=F16, norm_std=0.1),
    # splits over 2 tensor-parallel ranks: 4 query heads of 64 (one 256-block of o's K) and
    # 2 kv heads per rank, 512 ffn rows per rank
    # the further formats: Q5_K_M's mix (Q5_K, with Q6_K attn_v / ffn_down / output) and a
    # Q4_0 model with Q5_0 attn_v / ffn_down / output (one q|k|v launch over both)
    "tiny_q5km": ModelConfig(
        "tiny_q5km", dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn=512, vocab=448,
        rope_base=10000.0, context_length=512, default_type=Q5_K, overrides=Q4_K_M, embd_type=Q5_K,
        output_type=Q6_K, norm_std=0.1),
    "tiny_q4_0": ModelConfig(
        "tiny_q4_0", dim=256, n_layers=2, n_heads=4, n_kv_heads=4, ffn=512, vocab=352,
        rope_base=10000.0, context_length=512, default_type=Q4_0,
        overrides=(("attn_v", Q5_0), ("ffn_down", Q5_0)), embd_type=Q4_0, output_type=Q5_0, norm_std=0.1),
    # Q2_K with Q3_K attn_v / ffn_down and a Q4_K output (the mix of llama.cpp's Q2_K files)
    "tiny_q2k": ModelConfig(
        "tiny_q2k", dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn=512, vocab=416,
        rope_base=10000.0, context_length=512, default_type=Q2_K,
        overrides=(("attn_v", Q3_K), ("ffn_down", Q3_K)), embd_type=Q2_K, output_type=Q4_K, norm_std=0.1),
    # Q4_1 with Q5_1 attn_v / ffn_down / output (candle pairs both with Q8_1 activations)
    "tiny_q4_1": ModelConfig(
        "tiny_q4_1", dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn=512, vocab=320,
        rope_base=10000.0, context_length=512, default_type=Q4_1,
        overrides=(("attn_v", Q5_1), ("ffn_down", Q5_1)), embd_type=Q4_1, output_type=Q5_1, norm_std=0.1),
    # qwen2 (candle quantized_qwen2): q / k / v biases, RoPE on head halves, tied embeddings
    "tiny_qwen2": ModelConfig(
        "tiny_qwen2", dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn=512, vocab=384,
        rope_base=1000000.0, context_length=512, tied=True, overrides=Q4_K_M, embd_type=Q4_K,
        norm_std=0.1, arch="qwen2", qkv_bias=True),
    # phi3 (candle quantized_phi3): fused attn_qkv and ffn_up, RoPE on head halves, head_dim 96
    "tiny_phi3": ModelConfig(
        "tiny_phi3", dim=768, n_layers=2, n_heads=8, n_kv_heads=8, ffn=512, vocab=352,
        rope_base=10000.0, context_length=512, default_type=Q4_K, embd_type=Q4_K, output_type=Q6_K,
        norm_std=0.1, arch="phi3"),
    # mixture of experts, candle's per-expert tensor names (ffn_gate.E): Mixtral's layout in
    # miniature (4 experts, 2 per token, Q4_K_M mix with Q6_K downs, f32 router)
    "tiny_mixtral": ModelConfig(
        "tiny_mixtral", dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn=512, vocab=384,
        rope_base=1000000.0, context_length=512, overrides=Q4_K_M, embd_type=Q4_K, output_type=Q6_K,
        norm_std=0.1, n_expert=4, n_expert_used=2, expert_ffn=512, stacked_experts=False, router_std=0.2),
    # llama.cpp's stacked experts (ffn_*_exps): 8 experts, 4 per token (two gate|up launches),
    # a shared expert, an f16 router, Q5_K weights; layer 0 dense, layer 1 MoE
    "tiny_moe": ModelConfig(
        "tiny_moe", dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn=512, vocab=352,
        rope_base=10000.0, context_length=512, default_type=Q5_K, overrides=(("ffn_down", Q6_K),),
        embd_type=Q5_K, output_type=Q6_K, norm_std=0.1, n_expert=8, n_expert_used=4, expert_ffn=256,
        moe_layers=(1,), shared_ffn=512, router_type=F16, router_std=0.2),
    # gemma: GEGLU, embeddings times sqrt(dim), RoPE on head halves, tied embeddings
    "tiny_gemma": ModelConfig(
        "tiny_gemma", dim=256, n_layers=2, n_heads=4, n_kv_heads=4, ffn=512, vocab=320,
        rope_base=10000.0, context_length=512, tied=True, overrides=Q4_K_M, embd_type=Q4_K,
        norm_std=0.1, arch="gemma"),
    "tiny_tp_q4km": ModelConfig(
        "tiny_tp_q4km", dim=512, n_layers=2, n_heads=8, n_kv_heads=4, ffn=1024, vocab=384,
        rope_base=10000.0, context_length=512, overrides=Q4_K_M, embd_type=Q4_K,
        output_type=Q6_K, norm_std=0.1),
}

# C1: one Q4_K matrix [4096 out x 4096 in], W ~ N(0, 0.02), x ~ N(0, 1).
GEMV_C1 = dict(N=4096, K=4096, type=Q4_K, w_std=0.02, x_std=1.0)


def fnv1a64(s: str) -> int:
    h = 0xCBF29CE484222325
    for ch in s.encode():
        h = ((h ^ ch) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def tensor_seed(name: str, seed: int) -> int:
    return fnv1a64(name) ^ (seed & 0xFFFFFFFFFFFFFFFF)


_lib = None


def synth_lib():
    global _lib
    if _lib is None:
        path = lib_path("libtptsynth.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run tpt_spark_b200._build.build()")
        L = ctypes.CDLL(path)
        L.sy_make_tensor.restype = ctypes.c_int64
        L.sy_make_tensor.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int64, ctypes.c_float,
                                     ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
        L.sy_encode.restype = ctypes.c_int64
        L.sy_encode.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        L.sy_fill_normal.restype = None
        L.sy_fill_normal.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                     ctypes.c_float, ctypes.c_void_p]
        _lib = L
    return _lib


def normal(seed: int, n: int, std: float = 1.0, mean: float = 0.0, start: int = 0) -> np.ndarray:
    x = np.empty(n, np.float32)
    synth_lib().sy_fill_normal(seed, start, n, mean, std, x.ctypes.data)
    return x


def encode(t: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.empty(type_bytes(t, x.size), np.uint8)
    synth_lib().sy_encode(t, x.ctypes.data, x.size, out.ctypes.data)
    return out


def make_tensor(t: int, seed: int, n: int, std: float, mean: float = 0.0) -> np.ndarray:
    out = np.empty(type_bytes(t, n), np.uint8)
    scratch = np.empty(n, np.float32)
    synth_lib().sy_make_tensor(t, seed, n, mean, std, scratch.ctypes.data, out.ctypes.data)
    return out


def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, val) -> bytes:
    out = _gguf_str(key) + struct.pack("<I", vtype)
    if vtype == 4:
        out += struct.pack("<I", val)
    elif vtype == 6:
        out += struct.pack("<f", val)
    elif vtype == 8:
        out += _gguf_str(val)
    else:
        raise ValueError(vtype)
    return out


def metadata(cfg: ModelConfig) -> List[bytes]:
    a = cfg.arch
    return [
        _kv("general.architecture", 8, a),
        _kv("general.name", 8, cfg.name),
        _kv("general.alignment", 4, ALIGN),
        _kv(f"{a}.context_length", 4, cfg.context_length),
        _kv(f"{a}.embedding_length", 4, cfg.dim),
        _kv(f"{a}.block_count", 4, cfg.n_layers),
        _kv(f"{a}.feed_forward_length", 4, cfg.ffn),
        _kv(f"{a}.attention.head_count", 4, cfg.n_heads),
        _kv(f"{a}.attention.head_count_kv", 4, cfg.n_kv_heads),
        _kv(f"{a}.rope.dimension_count", 4, cfg.head_dim),
        _kv(f"{a}.rope.freq_base", 6, cfg.rope_base),
        _kv(f"{a}.attention.layer_norm_rms_epsilon", 6, cfg.rms_eps),
        _kv(f"{a}.vocab_size", 4, cfg.vocab),
    ] + ([_kv(f"{a}.expert_count", 4, cfg.n_expert),
          _kv(f"{a}.expert_used_count", 4, cfg.n_expert_used),
          _kv(f"{a}.expert_feed_forward_length", 4, cfg.expert_ffn)] if cfg.n_expert > 1 else [])


def write_gguf(path: str, cfg: ModelConfig, seed: int = 0,
               progress: Optional[Callable[[int, int], None]] = None) -> int:
    """Write the seeded model `cfg` to `path`. Returns the file size in bytes."""
    tensors = cfg.tensors()
    infos, offsets, off = [], [], 0
    for name, kind, ne in tensors:
        t = cfg.type_of(kind)
        n = int(np.prod(ne))
        nbytes = type_bytes(t, n)
        offsets.append(off)
        infos.append(_gguf_str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
                     + struct.pack("<I", t) + struct.pack("<Q", off))
        off += (nbytes + ALIGN - 1) // ALIGN * ALIGN
    kvs = metadata(cfg)
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kvs)) + b"".join(kvs) + b"".join(infos)
    pad = (-len(head)) % ALIGN
    L = synth_lib()
    chunk = 1 << 24
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        for i, ((name, kind, ne), o) in enumerate(zip(tensors, offsets)):
            t = cfg.type_of(kind)
            n = int(np.prod(ne))
            be = BLOCK[t][0]
            row = ne[0]
            if kind.endswith("norm"):
                std, mean = cfg.norm_std, 1.0
            elif kind == "bias":
                std, mean = cfg.bias_std, 0.0
            elif kind == "ffn_gate_inp":
                std, mean = cfg.router_std, 0.0
            else:
                std, mean = cfg.weight_std, 0.0
            s = tensor_seed(name, seed)
            step = max(row, chunk // row * row)
            scratch = np.empty(min(step, n), np.float32)
            done = 0
            while done < n:
                m = min(step, n - done)
                if std == 0.0:
                    scratch[:m] = mean
                else:
                    L.sy_fill_normal(s, done, m, mean, std, scratch.ctypes.data)
                assert m % be == 0
                out = np.empty(type_bytes(t, m), np.uint8)
                L.sy_encode(t, scratch.ctypes.data, m, out.ctypes.data)
                f.write(out.tobytes())
                done += m
            nbytes = type_bytes(t, n)
            f.write(b"\0" * ((-nbytes) % ALIGN))
            if progress:
                progress(i + 1, len(tensors))
        size = f.tell()
    return size


def default_model_dir() -> str:
    """Where generated benchmark models are kept: $TPTC_MODEL_DIR, else tptc_models under the
    system temporary directory."""
    import tempfile

    return os.environ.get("TPTC_MODEL_DIR") or os.path.join(tempfile.gettempdir(), "tptc_models")


def model_file(cfg: ModelConfig, model_dir: Optional[str] = None, seed: int = 0) -> str:
    """Path of the seeded model `cfg` in `model_dir` (default_model_dir()), written first if
    absent.  The file appears under its final name only once complete (written to a
    process-private name, then renamed), so concurrent writers never read a partial file."""
    model_dir = model_dir or default_model_dir()
    os.makedirs(model_dir, exist_ok=True)
    path = os.path.join(model_dir, f"{cfg.name}_s{seed}.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_gguf(tmp, cfg, seed=seed)
        os.replace(tmp, path)
    return path


def tensor_values(cfg: ModelConfig, name: str, seed: int = 0) -> np.ndarray:
    """The f32 values drawn for tensor `name` before encoding (tests)."""
    kinds = {n: (k, ne) for n, k, ne in cfg.tensors()}
    kind, ne = kinds[name]
    n = int(np.prod(ne))
    if kind.endswith("norm"):
        return np.full(n, 1.0, np.float32) if cfg.norm_std == 0 else normal(tensor_seed(name, seed), n, cfg.norm_std, 1.0)
    return normal(tensor_seed(name, seed), n, cfg.weight_std)
