"""Generate tests/golden/blocks.npz: GGUF block fixtures pinned by gguf-py.

gguf-py 0.19 (the gguf package in this image) implements the GGUF block formats in numpy:
dequantisation of Q4_K / Q6_K / Q8_0 / F16 (gguf/quants.py :395-401, :505-522, :554-572)
and of Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q2_K / Q3_K / Q5_K (:241-251, :276-288, :314-330,
:357-375, :406-428, :433-472, :527-549), and quantisation of Q8_0 (:381-393, "bit-exact with
ggml-quants.c").  The fixtures store raw
blocks (random bytes with finite f16 scales, plus hand-made edge blocks) together with
gguf-py's outputs, so the oracle and the CUDA kernels can be checked against them without
gguf-py at test time.

Run:  python tests/golden/make_golden.py
"""
import os

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants as Q

HERE = os.path.dirname(os.path.abspath(__file__))


def finite_f16_bytes(rng, n, lo=-8.0, hi=8.0):
    v = rng.uniform(lo, hi, n).astype(np.float16)
    return v.view(np.uint8).reshape(n, 2)


def q4k_blocks(rng, nb):
    b = rng.integers(0, 256, (nb, 144), dtype=np.uint8)
    b[:, 0:2] = finite_f16_bytes(rng, nb, 1e-4, 0.1)
    b[:, 2:4] = finite_f16_bytes(rng, nb, 1e-4, 0.1)
    # edge blocks: all scale/min bits set, all zero, max nibbles
    b[0, 4:16] = 0xFF
    b[0, 16:] = 0xFF
    b[1, 4:] = 0
    b[2, 4:16] = 0x3F
    b[3, 0:2] = np.array([0], np.float16).view(np.uint8)  # d = 0
    return b


def q6k_blocks(rng, nb):
    b = rng.integers(0, 256, (nb, 210), dtype=np.uint8)
    b[:, 208:210] = finite_f16_bytes(rng, nb, -0.1, 0.1)
    b[0, 192:208] = np.array([-128] * 16, np.int8).view(np.uint8)
    b[1, 192:208] = np.array([127] * 16, np.int8).view(np.uint8)
    b[2, :192] = 0xFF
    b[3, :192] = 0
    return b


def q80_blocks(rng, nb):
    b = rng.integers(0, 256, (nb, 34), dtype=np.uint8)
    b[:, 0:2] = finite_f16_bytes(rng, nb, -0.5, 0.5)
    b[0, 2:] = np.array([-128] * 32, np.int8).view(np.uint8)
    return b


# (name, type, bytes per block, elements per block, byte offsets of f16 scale fields)
MORE_FORMATS = (
    ("q40", T.Q4_0, 18, 32, (0,)),
    ("q41", T.Q4_1, 20, 32, (0, 2)),
    ("q50", T.Q5_0, 22, 32, (0,)),
    ("q51", T.Q5_1, 24, 32, (0, 2)),
    ("q2k", T.Q2_K, 84, 256, (80, 82)),
    ("q3k", T.Q3_K, 110, 256, (108,)),
    ("q5k", T.Q5_K, 176, 256, (0, 2)),
)


def more_blocks(rng, nbytes, scale_offs, nb):
    """Random blocks with finite f16 scales; block 0 all quant bits set, block 1 all clear."""
    b = rng.integers(0, 256, (nb, nbytes), dtype=np.uint8)
    keep = np.zeros(nbytes, bool)
    for o in scale_offs:
        b[:, o:o + 2] = finite_f16_bytes(rng, nb, -0.1, 0.1)
        keep[o:o + 2] = True
    b[0, ~keep] = 0xFF
    b[1, ~keep] = 0
    return b


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    for name, qt, blocks, be in (("q4k", T.Q4_K, q4k_blocks(rng, 64), 256), ("q6k", T.Q6_K, q6k_blocks(rng, 64), 256),
                                 ("q80", T.Q8_0, q80_blocks(rng, 128), 32)):
        out[f"{name}_raw"] = blocks.ravel()
        out[f"{name}_f32"] = Q.dequantize(blocks.ravel(), qt).astype(np.float32).ravel()
        assert out[f"{name}_f32"].size == blocks.shape[0] * be
    f16 = rng.standard_normal(4096).astype(np.float16)
    f16[:4] = np.array([65504, -65504, 6e-8, -0.0], np.float16)
    out["f16_raw"] = f16.view(np.uint8)
    out["f16_f32"] = Q.dequantize(f16.view(np.uint8), T.F16).astype(np.float32).ravel()
    # Q8_0 quantisation of activations: normal values, ties, zeros, a constant block
    x = rng.standard_normal(2048).astype(np.float32) * 3
    x[32:64] = 0.0
    x[64:96] = 1.25
    x[96:128] = np.linspace(-127, 127, 32, dtype=np.float32) / 127.0 * 4.0
    out["q80_x"] = x
    out["q80_q"] = Q.quantize(x.reshape(1, -1), T.Q8_0).ravel()
    # the further formats, from their own generator so that the fixtures above stay as they were
    rng2 = np.random.default_rng(20261202)
    for name, qt, nbytes, be, offs in MORE_FORMATS:
        blocks = more_blocks(rng2, nbytes, offs, 64 if be == 256 else 256)
        out[f"{name}_raw"] = blocks.ravel()
        out[f"{name}_f32"] = Q.dequantize(blocks.ravel(), qt).astype(np.float32).ravel()
        assert out[f"{name}_f32"].size == blocks.shape[0] * be
    np.savez_compressed(os.path.join(HERE, "blocks.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
