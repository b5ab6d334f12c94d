"""Batched prefill on a B200: causal tensor-core attention and the whole prompt forward.

The batched path computes every projection on the tcgen05 GEMM with fp16 operands (weights
expanded from the quantised blocks, activations rounded to fp16) and f32 accumulation, and the
attention on fp16 Q/K/V with f32 softmax.  Its numerical reference is therefore a float forward
of the same model (numpy float64 over the oracle's bit-exact dequantised weights), not candle's
integer-dot path; the final lm_head of the last token runs with candle's semantics on both
sides (Q8_K activations, oracle.matmul).  Against the candle oracle itself the difference is
candle's own 8-bit activation rounding, bounded separately.
"""
import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")

from tpt_spark_b200 import kernels as K  # noqa: E402
from tpt_spark_b200._lib import EngineError  # noqa: E402

pytestmark = pytest.mark.gpu

MODELS = ["tiny_q4km", "tiny_q4km_tied", "tiny_q8_0", "tiny_f16", "tiny_q5km", "tiny_q4_0", "tiny_q2k", "tiny_qwen2",
          "tiny_phi3", "tiny_q4_1", "tiny_gemma", "tiny_mixtral", "tiny_moe"]
BATCHED = MODELS

# fp16 operands (11-bit significands) against a float64 forward: relative error of a few
# 2^-11 per layer on the hidden state, times the logit scale of the tiny models (|logit| < 3)
LOGIT_ATOL_FLOAT_REF = 1e-2
# against candle's 8-bit activation path: that path's own rounding (Q8_K / Q8_0 of every
# projection input) dominates
LOGIT_ATOL_ORACLE = 5e-2


# ---------------------------------------------------------------- attention kernel

ATTN_SHAPES = [
    # T, start, n_heads, n_kv, hd, max_seq
    (64, 0, 32, 8, 128, 256),     # one query tile, the C5 head layout
    (200, 37, 4, 1, 64, 512),     # ragged chunk after a cached prefix, G = 4
    (1, 100, 8, 8, 96, 128),      # a single query row (MHA, hd 96: the C4 layout)
    (130, 0, 8, 8, 96, 256),      # ragged tiles from position 0
    (300, 700, 32, 32, 96, 1024),  # hd 96 after a long prefix: last head's padding out of bounds
    (512, 1000, 32, 8, 128, 2048),  # long prefix: 24 key tiles per query tile
]


def attn_reference(q, kc, vc, T, start, n_heads, n_kv, hd):
    """fp32 causal attention of query rows at positions start + t over cache rows 0..start+t."""
    G = n_heads // n_kv
    L = start + T
    qf = q.float().view(T, n_heads, hd).permute(1, 0, 2)            # [H, T, hd]
    kf = kc[:, :L].float().repeat_interleave(G, dim=0)              # [H, L, hd]
    vf = vc[:, :L].float().repeat_interleave(G, dim=0)
    s = qf @ kf.transpose(1, 2) / hd ** 0.5                         # [H, T, L]
    pos = torch.arange(start, start + T, device=q.device)[:, None]
    key = torch.arange(L, device=q.device)[None, :]
    s = s.masked_fill(key > pos, float("-inf"))
    o = torch.softmax(s, dim=-1) @ vf                               # [H, T, hd]
    return o.permute(1, 0, 2).reshape(T, n_heads * hd)


@pytest.mark.parametrize("shape", ATTN_SHAPES, ids=lambda s: "t%d_s%d_h%d_kv%d_d%d" % s[:5])
def test_attn_prefill_matches_torch(cuda_device, shape):
    T, start, H, KV, hd, max_seq = shape
    g = torch.Generator(device="cpu").manual_seed(T * 31 + start)
    q = torch.randn(T, H * hd, generator=g).half().to(cuda_device)
    kc = torch.randn(KV, max_seq, hd, generator=g).half().to(cuda_device)
    vc = torch.randn(KV, max_seq, hd, generator=g).half().to(cuda_device)
    out = torch.full((T, H * hd), float("nan"), dtype=torch.half, device=cuda_device)
    K.attn_prefill(q, kc, vc, out, T, start, H, KV, hd, max_seq)
    torch.cuda.synchronize()
    want = attn_reference(q, kc, vc, T, start, H, KV, hd)
    # probabilities enter P.V as fp16 and the output is stored as fp16 (2^-11 relative each)
    torch.testing.assert_close(out.float(), want, rtol=1e-2, atol=3e-3)


def test_attn_prefill_rejects_bad_arguments(cuda_device):
    z = torch.zeros(64 * 4 * 64, dtype=torch.half, device=cuda_device)
    with pytest.raises(EngineError, match="head_dim"):
        K.attn_prefill(z, z, z, z, 4, 0, 4, 2, 80, 64)
    with pytest.raises(EngineError, match="bad argument"):
        K.attn_prefill(z, z, z, z, 4, 62, 4, 2, 64, 64)  # runs past max_seq
    with pytest.raises(EngineError, match="bad argument"):
        K.attn_prefill(z, z, z, z, 4, 0, 4, 3, 64, 64)  # heads not a multiple of kv heads


# ---------------------------------------------------------------- float forward reference

def _weights(ref):
    arrs, tys = ref._arrays, ref._types
    D, F, hd = ref.dim, ref.ffn, ref.head_dim

    def mat(i, N, Kd):
        return O.dequant(tys[i], arrs[i], N * Kd).reshape(N, Kd).astype(np.float64)

    w = {"emb": mat(0, ref.vocab, D), "out_norm": np.asarray(arrs[1], np.float32).astype(np.float64)}
    E = getattr(ref, "n_expert", 0)
    S = 4 + 3 * E

    def moe_mat(a, t, N, Kd):
        if t in (O.F32, O.F16):  # the router: rows as stored
            return np.asarray(a).view(np.float32 if t == O.F32 else np.float16).reshape(N, Kd).astype(np.float64)
        return O.dequant(t, a, N * Kd).reshape(N, Kd).astype(np.float64)

    layers = []
    for l in range(ref.n_layers):
        b = 3 + 9 * l
        L = dict(
            attn_norm=np.asarray(arrs[b], np.float32).astype(np.float64),
            q=mat(b + 1, ref.n_heads * hd, D), k=mat(b + 2, ref.n_kv_heads * hd, D),
            v=mat(b + 3, ref.n_kv_heads * hd, D), o=mat(b + 4, D, ref.n_heads * hd),
            ffn_norm=np.asarray(arrs[b + 5], np.float32).astype(np.float64))
        moe = ref._moe[l * S: (l + 1) * S] if E else None
        if moe is not None and moe[0] is not None:  # router, experts (gate, up, down), shared expert
            mtys = ref._moe_types[l * S: (l + 1) * S]
            ef, sf = ref.expert_ffn, ref.shared_ffn
            L["router"] = moe_mat(moe[0], mtys[0], E, D)
            L["experts"] = [(moe_mat(moe[1 + 3 * e], mtys[1 + 3 * e], ef, D), moe_mat(moe[2 + 3 * e], mtys[2 + 3 * e], ef, D),
                             moe_mat(moe[3 + 3 * e], mtys[3 + 3 * e], D, ef)) for e in range(E)]
            L["shared"] = ((moe_mat(moe[1 + 3 * E], mtys[1 + 3 * E], sf, D), moe_mat(moe[2 + 3 * E], mtys[2 + 3 * E], sf, D),
                            moe_mat(moe[3 + 3 * E], mtys[3 + 3 * E], D, sf)) if moe[1 + 3 * E] is not None else None)
        else:
            L.update(gate=mat(b + 6, F, D), up=mat(b + 7, F, D), down=mat(b + 8, D, F))
        layers.append(L)
    w["layers"] = layers
    return w


def float_prefill_logits(ref, tokens):
    """Float64 forward of the prompt; the last position's final norm and lm_head with candle's
    semantics (oracle.matmul quantises the activation as candle does)."""
    w = _weights(ref)
    D, hd, H, KV = ref.dim, ref.head_dim, ref.n_heads, ref.n_kv_heads
    T, G = len(tokens), H // KV
    cos, sin = O.rope_table(T, hd, ref.rope_base)
    cos, sin = cos.astype(np.float64), sin.astype(np.float64)

    def rms(x, g):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + ref.rms_eps) * g

    arch = getattr(ref, "arch", "llama")
    neox = arch in ("qwen2", "phi3", "gemma")
    geglu = arch == "gemma"  # GEGLU and embeddings times sqrt(dim)

    def rope(x, n):  # [T, n*hd]: interleaved pairs (rope_i), or the head's two halves (qwen2)
        c, s = cos[:, None, :], sin[:, None, :]
        if neox:
            x = x.reshape(T, n, 2, hd // 2)
            r0 = x[:, :, 0] * c - x[:, :, 1] * s
            r1 = x[:, :, 0] * s + x[:, :, 1] * c
            return np.concatenate([r0, r1], -1).reshape(T, n, hd)
        x = x.reshape(T, n, hd // 2, 2)
        r0 = x[..., 0] * c - x[..., 1] * s
        r1 = x[..., 0] * s + x[..., 1] * c
        return np.stack([r0, r1], -1).reshape(T, n, hd)

    biases = getattr(ref, "_biases", None) or [None] * (3 * ref.n_layers)

    def bias(i):
        b = biases[i]
        return 0.0 if b is None else b.astype(np.float64)

    x = w["emb"][np.asarray(tokens)]
    if geglu:
        x = x * np.float64(np.float32(np.sqrt(np.float32(D))))
    mask = np.triu(np.full((T, T), -np.inf), 1)
    for li, L in enumerate(w["layers"]):
        xn = rms(x, L["attn_norm"])
        q = rope(xn @ L["q"].T + bias(3 * li), H)
        k = rope(xn @ L["k"].T + bias(3 * li + 1), KV)
        v = (xn @ L["v"].T + bias(3 * li + 2)).reshape(T, KV, hd)
        att = np.empty((T, H, hd))
        for h in range(H):
            s = q[:, h] @ k[:, h // G].T / np.sqrt(hd) + mask
            p = np.exp(s - s.max(-1, keepdims=True))
            att[:, h] = (p / p.sum(-1, keepdims=True)) @ v[:, h // G]
        x = x + att.reshape(T, H * hd) @ L["o"].T
        xn = rms(x, L["ffn_norm"])

        def mlp(z, g_, u_, d_):
            gt, up = z @ g_.T, z @ u_.T
            act = gt * 0.5 * (1 + np.tanh(0.7978845608 * (gt + 0.044715 * gt ** 3))) if geglu else gt / (1 + np.exp(-gt))
            return (act * up) @ d_.T

        if "router" in L:  # candle MlpOrMoe::MoE: softmax routing, stable top-k, renormalised
            lg = xn @ L["router"].T
            rw = np.exp(lg - lg.max(-1, keepdims=True))
            rw /= rw.sum(-1, keepdims=True)
            y = np.zeros_like(x)
            for t in range(T):
                top = np.argsort(-rw[t], kind="stable")[:ref.n_expert_used]
                for e in sorted(top.tolist()):
                    y[t] += mlp(xn[t:t + 1], *L["experts"][e])[0] * (rw[t, e] / rw[t, top].sum())
            if L["shared"] is not None:
                y += mlp(xn, *L["shared"])
            x = x + y
        else:
            x = x + mlp(xn, L["gate"], L["up"], L["down"])
    last = rms(x[-1:], w["out_norm"]).astype(np.float32)
    out_i = 2
    return O.matmul(ref._types[out_i], ref._arrays[out_i], ref.vocab, D, last)[0]


@pytest.fixture(scope="module")
def engines_f16(tiny_models, cuda_device):
    from tpt_spark_b200.engine import CudaEngine

    out = {}
    for name, path in tiny_models.items():
        e = CudaEngine(0, kv_dtype="f16")
        e.load(path)
        e.set_prefill_gemm_min(1)
        out[name] = e
    yield out
    for e in out.values():
        e.close()


def _prompt(ref, n, seed):
    return [int(t) for t in np.random.default_rng(seed).integers(0, ref.vocab, n)]


@pytest.mark.parametrize("name", BATCHED)
def test_batched_prefill_matches_float_reference(engines_f16, tiny_models, name):
    e = engines_f16[name]
    ref = O.Model(tiny_models[name])
    for n in (150, 77):
        e.kv_reset()
        prompt = _prompt(ref, n, n)
        lg = e.prefill(prompt)
        want = float_prefill_logits(ref, prompt)
        diff = float(np.abs(lg - want).max())
        print(f"{name} n={n}: max |logit - float64 reference| = {diff:.2e}")
        assert diff <= LOGIT_ATOL_FLOAT_REF


@pytest.mark.parametrize("name", MODELS)
def test_batched_prefill_then_decode_against_oracle(engines_f16, tiny_models, name):
    """Batched prefill, then 32 teacher-forced decode steps over its KV cache, against candle."""
    e = engines_f16[name]
    e.kv_reset()
    ref = O.Model(tiny_models[name])
    prompt = _prompt(ref, 100, 5)
    lg = e.prefill(prompt)
    lo = ref.forward(prompt, 0)
    worst = float(np.abs(lg - lo).max())
    pos = len(prompt)
    route_tie = False
    for step in range(32):
        tok = O.argmax(lo)
        g_logits, g_tok = e.decode(tok, pos)
        if ref.n_expert:  # routing near-ties end the comparison (tests/test_gpu_forward.py)
            lo, gaps = ref.forward_route([tok], pos)
            route_tie = route_tie or float(np.nanmin(gaps)) <= 1e-2
        else:
            lo = ref.forward([tok], pos)
        d = float(np.abs(g_logits - lo).max())
        if d > LOGIT_ATOL_ORACLE and route_tie and step >= 16:
            break
        worst = max(worst, d)
        top2 = np.sort(lo)[-2:]
        if top2[1] - top2[0] > 2 * d:
            assert g_tok == O.argmax(lo)
        pos += 1
    print(f"{name}: max |logit diff| vs oracle after batched prefill = {worst:.2e}")
    assert worst <= LOGIT_ATOL_ORACLE


@pytest.mark.parametrize("name", MODELS)
def test_prefill_in_pieces_is_bit_identical(engines_f16, tiny_models, name):
    """A prompt prefilled in two pieces (the second after a cached prefix) gives the same
    logits bit for bit: GEMM rows are independent and every query row sees the same key
    tiles in the same order whatever chunk it belongs to."""
    e = engines_f16[name]
    ref = O.Model(tiny_models[name])
    prompt = _prompt(ref, 140, 11)
    e.kv_reset()
    whole = e.prefill(prompt)
    e.kv_reset()
    e.prefill(prompt[:61])
    assert e.kv_len() == 61
    split = e.prefill(prompt[61:], start_pos=61)
    assert e.kv_len() == 140
    np.testing.assert_array_equal(split, whole)


@pytest.mark.parametrize("name", ["tiny_q4km", "tiny_q8_0"])
def test_fused_dequant_prefill_matches_float_reference(tiny_models, cuda_device, name):
    """Every quantised projection through the fused-dequant GEMM (TPTC_FUSED_ALWAYS): the same
    float-reference bound as the two-pass path, and close to the two-pass logits (the fused
    expansion differs from the two-pass one by at most one fp16 rounding of the scale
    product; Q8_0 weights are identical, so the logits are too)."""
    from tpt_spark_b200.engine import CudaEngine

    ref = O.Model(tiny_models[name])
    e = CudaEngine(0, kv_dtype="f16")
    try:
        e.load(tiny_models[name])
        e.set_prefill_gemm_min(1)
        for n in (150, 33):
            prompt = _prompt(ref, n, n + 1)
            e.set_prefill_fused("always")
            e.kv_reset()
            fused = e.prefill(prompt)
            e.set_prefill_fused("never")
            e.kv_reset()
            two_pass = e.prefill(prompt)
            want = float_prefill_logits(ref, prompt)
            diff = float(np.abs(fused - want).max())
            print(f"{name} n={n}: fused max |logit - float64 reference| = {diff:.2e}, "
                  f"vs two-pass {float(np.abs(fused - two_pass).max()):.2e}")
            assert diff <= LOGIT_ATOL_FLOAT_REF
            if name == "tiny_q8_0":
                np.testing.assert_array_equal(fused, two_pass)
            else:
                assert float(np.abs(fused - two_pass).max()) <= LOGIT_ATOL_FLOAT_REF
        with pytest.raises(ValueError):
            e.set_prefill_fused("sometimes")
    finally:
        e.close()


def test_threshold_and_f32_cache_use_the_token_path(tiny_models, cuda_device):
    """Below the threshold (and always with an f32 cache) the prompt runs token by token:
    bit-identical to decoding it."""
    from tpt_spark_b200.engine import CudaEngine

    path = tiny_models["tiny_q4km"]
    ref = O.Model(path)
    prompt = _prompt(ref, 40, 3)
    for kv, gemm_min in (("f16", 0), ("f16", 41), ("f32", 1)):
        with CudaEngine(0, kv_dtype=kv) as e:
            e.load(path)
            e.set_prefill_gemm_min(gemm_min)
            lg = e.prefill(prompt)
            e.kv_reset()
            for i, t in enumerate(prompt):
                step, _ = e.decode(t, i)
            np.testing.assert_array_equal(lg, step)
    # and at the threshold the batched path is taken (its fp16 numerics differ)
    with CudaEngine(0, kv_dtype="f16") as e:
        e.load(path)
        e.set_prefill_gemm_min(40)
        lg = e.prefill(prompt)
        e.kv_reset()
        for i, t in enumerate(prompt):
            step, _ = e.decode(t, i)
        assert not np.array_equal(lg, step)
        assert float(np.abs(lg - step).max()) <= LOGIT_ATOL_ORACLE
