"""tptc_attn_decode (one decode-step GQA attention) against a plain torch fp32 reference.

The reference follows candle quantized_llama forward_attn for one query: rope_i on q and k,
scores q.k / sqrt(hd) over keys 0..pos, softmax, P.V with kv head h / (n_heads / n_kv)
(the reference engine's attention.wgsl:31-170 computes the same for its queries).
"""
import math

import pytest

torch = pytest.importorskip("torch")

from tpt_spark_b200 import kernels as K  # noqa: E402
from tpt_spark_b200._lib import EngineError  # noqa: E402

pytestmark = pytest.mark.gpu

# fp32 arithmetic in a different summation order (split-K flash-decode vs one softmax)
RTOL, ATOL = 1e-4, 1e-5


def rope_tables(max_seq, hd, base=10000.0):
    """candle rope_i tables: theta_j = base^(-2j/hd), angle = pos * theta_j (f32)."""
    j = torch.arange(0, hd, 2, dtype=torch.float32)
    theta = 1.0 / torch.pow(torch.tensor(base, dtype=torch.float32), j / hd)
    ang = torch.arange(max_seq, dtype=torch.float32)[:, None] * theta[None, :]
    return torch.cos(ang).contiguous(), torch.sin(ang).contiguous()


def rope(x, c, s):
    """Interleaved-pair rotation: (x0*c - x1*s, x0*s + x1*c), each product rounded alone."""
    x0, x1 = x[..., 0::2], x[..., 1::2]
    r0 = x0 * c - x1 * s
    r1 = x0 * s + x1 * c
    return torch.stack([r0, r1], dim=-1).flatten(-2)


def reference(q, kraw, kc, vc, cs, sn, pos, n_heads, n_kv, hd, kv_dtype):
    krot = rope(kraw.view(n_kv, hd), cs[pos], sn[pos]).to(kv_dtype)
    keys = kc[:, : pos + 1].float().clone()
    keys[:, pos] = krot.float()
    vals = vc[:, : pos + 1].float()
    qr = rope(q.view(n_heads, hd), cs[pos], sn[pos])
    G = n_heads // n_kv
    out = torch.empty(n_heads, hd, device=q.device)
    for h in range(n_heads):
        sc = (keys[h // G] @ qr[h]) * (1.0 / math.sqrt(hd))
        p = torch.softmax(sc, dim=0)
        out[h] = p @ vals[h // G]
    return out.flatten(), krot


def make_case(n_heads, n_kv, hd, max_seq, pos, kv_type, seed, dev, base=10000.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    kv_dtype = torch.float32 if kv_type == K.F32 else torch.float16
    q = torch.randn(n_heads * hd, generator=g).to(dev)
    kraw = torch.randn(n_kv * hd, generator=g).to(dev)
    kc = torch.randn(n_kv, max_seq, hd, generator=g).to(kv_dtype).to(dev)
    vc = torch.randn(n_kv, max_seq, hd, generator=g).to(kv_dtype).to(dev)
    cs, sn = rope_tables(max_seq, hd, base)
    return q, kraw, kc, vc, cs.to(dev), sn.to(dev), kv_dtype


def run(q, kraw, kc, vc, kv_type, cs, sn, pos, n_heads, n_kv, hd, max_seq, ws=None):
    dev = q.device
    d_pos = torch.tensor([pos], dtype=torch.int32, device=dev)
    out = torch.full((n_heads * hd,), float("nan"), device=dev)
    nbytes = K.attn_decode_workspace_bytes(n_heads, n_kv, hd, max_seq)
    if ws is None:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    K.attn_decode(q, kraw, kc, vc, kv_type, cs, sn, d_pos, n_heads, n_kv, hd, max_seq, out, ws, nbytes)
    torch.cuda.synchronize()
    return out, ws


SHAPES = [
    # n_heads, n_kv, hd, max_seq, pos
    (32, 8, 128, 9216, 0),        # Llama-3-8B shape, first position
    (32, 8, 128, 9216, 4097),     # ragged last tile, several splits
    (32, 8, 128, 9216, 9215),     # last slot of the cache
    (8, 1, 128, 512, 300),        # MQA, one kv head
    (12, 4, 64, 1000, 777),       # max_seq not a multiple of the tile
    (24, 8, 96, 700, 63),         # hd 96 (Phi-3 shape), a tile boundary
    (16, 16, 64, 256, 130),       # MHA, hd 64
    (64, 8, 128, 4096, 3000),     # 8 query heads per kv head
    (16, 8, 64, 2048, 1500),      # 2 query heads per kv head
    (32, 32, 128, 8192, 7000),    # MHA at a long context: 11 key tiles per split
    (32, 32, 96, 8192, 8000),     # hd 96, 13 key tiles per split (the ring reused 4 times)
]


@pytest.mark.parametrize("kv_type", [K.F16, K.F32], ids=["f16", "f32"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "h%d_kv%d_d%d_s%d_p%d" % s)
def test_attn_decode_matches_torch(cuda_device, shape, kv_type):
    n_heads, n_kv, hd, max_seq, pos = shape
    q, kraw, kc, vc, cs, sn, kv_dtype = make_case(n_heads, n_kv, hd, max_seq, pos, kv_type, 1234 + pos, cuda_device)
    want, krot = reference(q, kraw, kc, vc, cs, sn, pos, n_heads, n_kv, hd, kv_dtype)
    out, ws = run(q, kraw, kc, vc, kv_type, cs, sn, pos, n_heads, n_kv, hd, max_seq)
    torch.testing.assert_close(out, want, rtol=RTOL, atol=ATOL)
    # the rotated key is cached exactly (each product rounded alone, as rope_i)
    assert torch.equal(kc[:, pos], krot)
    # the workspace is ready for the next call: error word and split counters zero
    assert int(ws[:4].view(torch.int32)[0]) == 0
    assert int(ws[256:256 + 4 * n_kv].view(torch.int32).abs().sum()) == 0


# The configurations' own attention shapes at their longest decode positions, with their RoPE
# bases: C2 (32/8 heads of 64, base 500000, 384 positions), C3 (32/8 of 128, base 10000, 2560),
# C4 (32/32 of 96, MHA, base 10000, 1280), C5 (32/8 of 128, base 500000, 9216).
CONFIG_SHAPES = [
    (32, 8, 64, 2048, 383, 500000.0),
    (32, 8, 128, 4096, 2559, 10000.0),
    (32, 32, 96, 4096, 1279, 10000.0),
    (32, 8, 128, 9216, 9215, 500000.0),
    (32, 8, 128, 9216, 8192, 500000.0),
]


@pytest.mark.parametrize("shape", CONFIG_SHAPES, ids=lambda s: "h%d_kv%d_d%d_s%d_p%d_base%d" % s)
def test_attn_decode_config_shapes(cuda_device, shape):
    n_heads, n_kv, hd, max_seq, pos, base = shape
    q, kraw, kc, vc, cs, sn, kv_dtype = make_case(n_heads, n_kv, hd, max_seq, pos, K.F16, 99 + pos, cuda_device, base)
    want, krot = reference(q, kraw, kc, vc, cs, sn, pos, n_heads, n_kv, hd, kv_dtype)
    out, _ = run(q, kraw, kc, vc, K.F16, cs, sn, pos, n_heads, n_kv, hd, max_seq)
    torch.testing.assert_close(out, want, rtol=RTOL, atol=ATOL)
    assert torch.equal(kc[:, pos], krot)


def test_attn_decode_repeatable(cuda_device):
    n_heads, n_kv, hd, max_seq, pos = 32, 8, 128, 9216, 5000
    q, kraw, kc, vc, cs, sn, _ = make_case(n_heads, n_kv, hd, max_seq, pos, K.F16, 7, cuda_device)
    a, ws = run(q, kraw, kc, vc, K.F16, cs, sn, pos, n_heads, n_kv, hd, max_seq)
    b, _ = run(q, kraw, kc, vc, K.F16, cs, sn, pos, n_heads, n_kv, hd, max_seq, ws=ws)
    assert torch.equal(a, b)  # the split merge runs in split order


def test_attn_decode_position_outside_cache(cuda_device):
    n_heads, n_kv, hd, max_seq = 8, 2, 64, 128
    q, kraw, kc, vc, cs, sn, _ = make_case(n_heads, n_kv, hd, max_seq, 0, K.F32, 3, cuda_device)
    kc0 = kc.clone()
    out, ws = run(q, kraw, kc, vc, K.F32, cs, sn, max_seq, n_heads, n_kv, hd, max_seq)
    assert int(ws[:4].view(torch.int32)[0]) == -1  # TPTC_ERR_ARG
    assert torch.isnan(out).all() and torch.equal(kc, kc0)


def test_attn_decode_argument_errors(cuda_device):
    n_heads, n_kv, hd, max_seq = 8, 2, 64, 128
    q, kraw, kc, vc, cs, sn, _ = make_case(n_heads, n_kv, hd, max_seq, 0, K.F32, 3, cuda_device)
    d_pos = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = torch.empty(n_heads * hd, device=cuda_device)
    nbytes = K.attn_decode_workspace_bytes(n_heads, n_kv, hd, max_seq)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(EngineError, match="workspace"):
        K.attn_decode(q, kraw, kc, vc, K.F32, cs, sn, d_pos, n_heads, n_kv, hd, max_seq, out, ws, nbytes - 1)
    with pytest.raises(EngineError, match="query heads"):
        K.attn_decode(q, kraw, kc, vc, K.F32, cs, sn, d_pos, 18, 2, hd, max_seq, out, ws, nbytes)
    with pytest.raises(EngineError, match="head_dim"):
        K.attn_decode(q, kraw, kc, vc, K.F32, cs, sn, d_pos, n_heads, n_kv, 72, max_seq, out, ws, nbytes)
    with pytest.raises(EngineError, match="kv_type"):
        K.attn_decode(q, kraw, kc, vc, K.Q8_0, cs, sn, d_pos, n_heads, n_kv, hd, max_seq, out, ws, nbytes)
