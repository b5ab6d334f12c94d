"""tptc_gemm_q (the prefill GEMM with the weight dequantisation fused in) against torch fp32.

The kernel expands each quantised block to fp16 in shared memory with fp16 arithmetic:
  Q4_K  w = fp16(code * s + m),   s = fp16(d * sc),  m = fp16(-(dmin * mn))  (one fused rounding)
  Q6_K  w = fp16((code - 32) * s), s = fp16(d * sc)
  Q8_0  w = fp16(code * d)        (= the f32 expansion rounded to fp16)
`expand_fp16` below restates that in numpy (exact products in float64, one rounding to fp16),
so the GEMM is checked against torch's fp32 matmul of the same fp16 operands with the f32
summation-order tolerance of the plain fp16 GEMM, and bit for bit against that GEMM
(tptc_gemm_f16, the same tcgen05 instruction sequence) given the expanded matrix.  The
expansion itself is within one fp16 rounding of the reference dequantisation
(candle k_quants.rs dequantize_row_q4_k / q6_k / q8_0) -- checked on the CPU here too.
"""
import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")


def _k4_scale_min(q):
    """6-bit scales and mins of the eight Q4_K sub-blocks (get_scale_min_k4, k_quants.rs)."""
    q = q.astype(np.int32)
    sc = np.empty(q.shape[:-1] + (8,), np.int32)
    mn = np.empty_like(sc)
    for j in range(8):
        if j < 4:
            sc[..., j] = q[..., j] & 63
            mn[..., j] = q[..., j + 4] & 63
        else:
            sc[..., j] = (q[..., j + 4] & 0xF) | ((q[..., j - 4] >> 6) << 4)
            mn[..., j] = (q[..., j + 4] >> 4) | ((q[..., j] >> 6) << 4)
    return sc, mn


def expand_fp16(t, raw, N, K):
    """The fused kernel's fp16 weight values [N x K] from raw GGUF blocks (numpy)."""
    raw = np.ascontiguousarray(raw).view(np.uint8)
    if t == O.Q4_K:
        b = raw.reshape(-1, 144)
        d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
        dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)
        sc, mn = _k4_scale_min(b[:, 4:16])
        s = (d * sc.astype(np.float32)).astype(np.float16).astype(np.float64)
        m = (-(dmin * mn.astype(np.float32))).astype(np.float16).astype(np.float64)
        qs = b[:, 16:].reshape(-1, 4, 32)
        codes = np.stack([qs & 15, qs >> 4], axis=2).reshape(-1, 8, 32).astype(np.float64)
        w = (codes * s[:, :, None] + m[:, :, None]).astype(np.float16)
    elif t == O.Q6_K:
        b = raw.reshape(-1, 210)
        ql, qh = b[:, :128].astype(np.int32), b[:, 128:192].astype(np.int32)
        sc = b[:, 192:208].copy().view(np.int8).astype(np.float32)
        d = b[:, 208:210].copy().view(np.float16).astype(np.float32)
        codes = np.empty((b.shape[0], 256), np.int32)
        for h in range(2):
            lo, hi, hb = ql[:, 64 * h:64 * h + 32], ql[:, 64 * h + 32:64 * h + 64], qh[:, 32 * h:32 * h + 32]
            base = 128 * h
            codes[:, base:base + 32] = (lo & 15) | (((hb >> 0) & 3) << 4)
            codes[:, base + 32:base + 64] = (hi & 15) | (((hb >> 2) & 3) << 4)
            codes[:, base + 64:base + 96] = (lo >> 4) | (((hb >> 4) & 3) << 4)
            codes[:, base + 96:base + 128] = (hi >> 4) | (((hb >> 6) & 3) << 4)
        s = (d * sc).astype(np.float16).astype(np.float64)  # [blocks, 16]
        w = ((codes - 32).reshape(-1, 16, 16).astype(np.float64) * s[:, :, None]).astype(np.float16)
    elif t == O.Q8_0:
        b = raw.reshape(-1, 34)
        d = b[:, 0:2].copy().view(np.float16).astype(np.float64)
        x = b[:, 2:].copy().view(np.int8).astype(np.float64)
        w = (x * d).astype(np.float16)
    else:
        raise ValueError(t)
    return w.reshape(N, K)


def make(t, N, K, seed):
    from tpt_spark_b200 import synth
    from tpt_spark_b200.kernels import Matrix

    raw = synth.encode(t, synth.normal(2000 + seed, N * K, 0.02))
    return raw, Matrix(t, raw, N, K)


TYPES = [("q4k", O.Q4_K), ("q6k", O.Q6_K), ("q80", O.Q8_0)]


@pytest.mark.parametrize("name,t", TYPES)
def test_expansion_within_one_fp16_rounding_of_dequant(name, t):
    """CPU: the kernel's fp16 values are the oracle's f32 dequantisation to within one fp16
    rounding of the scale product (Q8_0: exactly the f32 value rounded to fp16)."""
    from tpt_spark_b200 import synth

    N, K = 16, 512
    raw = synth.encode(t, synth.normal(7, N * K, 0.02))
    want = O.dequant(t, raw, N * K).reshape(N, K)
    got = expand_fp16(t, raw, N, K).astype(np.float32)
    if t == O.Q8_0:
        np.testing.assert_array_equal(got, want.astype(np.float16).astype(np.float32))
    else:
        # |fp16(s) - s| <= 2^-11 |s| and one more rounding of the result
        np.testing.assert_allclose(got, want, rtol=2e-3, atol=2e-3 * np.abs(want).max())


SHAPES = [
    # M, N, K
    (128, 256, 256),    # one tile, one super-block
    (300, 512, 4352),   # ragged M; 17 super-blocks: a full chunk and a one-block last chunk
    (77, 200, 1024),    # ragged M and N (the last row group past the matrix reads zeros)
    (1, 1024, 2048),    # a single token; fewer super-blocks than a chunk
]


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "m%d_n%d_k%d" % s)
@pytest.mark.parametrize("name,t", TYPES)
def test_gemm_q_matches_torch(cuda_device, name, t, shape):
    M, N, Kd = shape
    raw, m = make(t, N, Kd, M + N)
    w = torch.from_numpy(expand_fp16(t, raw, N, Kd)).to(cuda_device)
    g = torch.Generator(device="cpu").manual_seed(M * 5 + Kd)
    a = torch.randn(M, Kd, generator=g).half().to(cuda_device)
    c = torch.full((M, N), float("nan"), device=cuda_device)
    m.gemm(a, c, M)
    torch.cuda.synchronize()
    want = a.float() @ w.float().T
    torch.testing.assert_close(c, want, rtol=1e-4, atol=1e-4 * (Kd ** 0.5) * 0.05)


@pytest.mark.gpu
@pytest.mark.parametrize("name,t", TYPES)
def test_gemm_q_bitwise_equals_gemm_of_expanded(cuda_device, name, t):
    """Same tcgen05 sequence as the fp16 GEMM (128 x 256 tiles, K 16 products in the same
    order): identical bits given the expanded matrix (1024 x 6144 x 4096 for Q4_K: more tiles
    than SMs, both accumulators cycling)."""
    from tpt_spark_b200 import kernels as K

    M, N, Kd = (1024, 6144, 4096) if t == O.Q4_K else (256, 1024, 4096)
    raw, m = make(t, N, Kd, 3)
    w = torch.from_numpy(expand_fp16(t, raw, N, Kd)).to(cuda_device)
    a = (torch.randn(M, Kd, generator=torch.Generator(device="cpu").manual_seed(11))).half().to(cuda_device)
    c = torch.full((M, N), float("nan"), device=cuda_device)
    c2 = torch.full((M, N), float("nan"), device=cuda_device)
    m.gemm(a, c, M)
    K.gemm_f16(a, w, c2, M, N, Kd)
    torch.cuda.synchronize()
    assert torch.equal(c.view(torch.int32), c2.view(torch.int32))


@pytest.mark.gpu
def test_gemm_q_rejects_f16_and_glu(cuda_device):
    from tpt_spark_b200 import synth
    from tpt_spark_b200._lib import EngineError
    from tpt_spark_b200.kernels import Matrix

    raw = synth.encode(O.F16, synth.normal(1, 64 * 256, 0.02))
    m = Matrix(O.F16, raw, 64, 256)
    a = torch.zeros(4, 256, dtype=torch.half, device=cuda_device)
    c = torch.zeros(4, 64, device=cuda_device)
    with pytest.raises(EngineError, match="Q4_K, Q6_K or Q8_0"):
        m.gemm(a, c, 4)
