"""Forward-pass parity and LlmEngine behaviour on a B200, on the small synthetic models.

North_star level 3: greedy decode gives identical token ids for 64 steps and logits within
2e-2 absolute of the oracle.  Logits are compared under teacher forcing (both sides decode the
oracle's tokens), and the oracle's top-2 margin is logged at each step so a flip can be
attributed.

Where the two paths can legitimately differ: every matmul input is rounded to 8 bits
(Q8_K / Q8_0, round half away from zero).  f32 reductions in a different order (RMSNorm's
sum of squares is sequential in candle, a tree here) move a value by an ulp, which flips the
rounding of elements sitting exactly on a .5 boundary.  Q6_K token embeddings make such exact
ties common at layer 0 (every row is integer multiples of per-sub-block scales), so the tied
Q6_K-embedding model (the C2 layout) gets a per-flip budget instead of exact identity."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-2       # north_star level 3, f32 KV cache (candle's precision)
LOGIT_ATOL_TIES = 4e-2  # tied Q6_K-embedding model: 8-bit rounding ties at layer 0 (above)
LOGIT_ATOL_F16KV = 5e-2  # fp16 KV cache: K/V rounded to 11 bits before attention
TIE_PRONE = {"tiny_q4km_tied"}
# Greedy paths that pass through near-ties of the oracle's own top two logits (measured on the
# oracle: tiny_q5km 0.046 at step 31 and 3.2e-4 at step 10, tiny_q4_0 2.3e-5 at step 60,
# tiny_q2k 9.3e-5 at step 19, tiny_qwen2 1.8e-3 at step 6, tiny_phi3 4.5e-4 at step 24,
# tiny_q4_1 3.4e-3 at step 11, tiny_mixtral 9.6e-4 at step 41, tiny_moe 3.7e-4 at step 19):
# a difference within the logit tolerance can pick the other token there, so these sequences
# may part only at such a step.
GREEDY_TIE_PRONE = TIE_PRONE | {"tiny_q5km", "tiny_q4_0", "tiny_q2k", "tiny_qwen2", "tiny_phi3", "tiny_q4_1",
                                "tiny_mixtral", "tiny_moe"}


# tiny_phi3: the oracle's own logits move by up to 0.026 over the first steps of PROMPT when
# its RMSNorm sums in 4 interleaved lanes instead of sequentially (an equally valid f32
# order, oracle.set_norm_lanes): one Q8 activation rounding flips, the floor any
# reimplementation that sums in another order meets, and the GPU lands at that floor.
FLOOR_ATOL = {"tiny_phi3": LOGIT_ATOL_TIES}


def atol_for(name):
    return LOGIT_ATOL_TIES if name in TIE_PRONE else FLOOR_ATOL.get(name, LOGIT_ATOL)


# Mixture of experts: the expert choice is discontinuous in the router logits.  Where the
# oracle's gap between the last chosen expert and the best one left out is within the two
# paths' numerical difference (the hidden states differ by about 1e-3), the GPU may choose the
# other expert and the logits jump (tiny_mixtral with a router of std 0.05: 0.098 at a gap of
# 1.2e-3; with the 0.2 router of the test models the smallest gaps on the 64-step paths are
# 9.9e-3 at step 21 and, for tiny_moe, 3.9e-4 at step 44).  Such a step ends a comparison; it is accepted only after ROUTE_MIN_STEPS strict
# steps and only where the oracle reports a gap below ROUTE_TIE at that step or before.
ROUTE_TIE = 1e-2
ROUTE_MIN_STEPS = 16


def oracle_step(ref, tokens, pos):
    """Oracle logits and its smallest routing margin over the layers (inf without experts)."""
    if not getattr(ref, "n_expert", 0):
        return ref.forward(tokens, pos), float("inf")
    lo, gaps = ref.forward_route(tokens, pos)
    return lo, float(np.nanmin(gaps))
PROMPT = [3, 141, 59, 26, 5, 358, 97, 93, 238, 46, 264, 33]


def _engines(tiny_models, kv_dtype):
    from tpt_spark_b200.engine import CudaEngine

    out = {}
    for name, path in tiny_models.items():
        e = CudaEngine(0, kv_dtype=kv_dtype)
        e.load(path)
        out[name] = e
    return out


@pytest.fixture(scope="module")
def engines(tiny_models, cuda_device):
    out = _engines(tiny_models, "f32")
    yield out
    for e in out.values():
        e.close()


@pytest.fixture(scope="module")
def engines_f16kv(tiny_models, cuda_device):
    out = _engines(tiny_models, "f16")
    yield out
    for e in out.values():
        e.close()


MODELS = ["tiny_q4km", "tiny_q4km_tied", "tiny_q8_0", "tiny_f16", "tiny_q5km", "tiny_q4_0", "tiny_q2k", "tiny_qwen2",
          "tiny_phi3", "tiny_q4_1", "tiny_mixtral", "tiny_moe", "tiny_gemma"]


@pytest.mark.parametrize("name", MODELS)
def test_model_info(engines, tiny_models, name):
    from tpt_spark_b200 import synth

    info = engines[name].model_info()
    cfg = synth.TINY[name]
    assert info.backend == "cuda-sm100a"
    assert (info.dim, info.n_layers, info.n_heads, info.n_kv_heads, info.vocab) == (
        cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.vocab)
    assert info.tied_embeddings == cfg.tied
    assert info.path == tiny_models[name] and info.size_bytes > 0


@pytest.mark.parametrize("name", MODELS)
def test_teacher_forced_logits_and_argmax(engines, tiny_models, name):
    e = engines[name]
    e.kv_reset()
    ref = O.Model(tiny_models[name])
    prompt = [t % ref.vocab for t in PROMPT]
    lg = e.prefill(prompt)
    lo = ref.forward(prompt, 0)
    atol = atol_for(name)
    np.testing.assert_allclose(lg, lo, rtol=0, atol=atol)
    pos = len(prompt)
    worst = 0.0
    route_tie = False
    for step in range(64):
        tok = O.argmax(lo)
        g_logits, g_tok = e.decode(tok, pos)
        lo, rgap = oracle_step(ref, [tok], pos)
        route_tie = route_tie or rgap <= ROUTE_TIE
        top2 = np.sort(lo)[-2:]
        margin = float(top2[1] - top2[0])  # oracle's top-2 gap for this step
        diff = float(np.abs(g_logits - lo).max())
        if diff > atol and route_tie and step >= ROUTE_MIN_STEPS:
            print(f"{name}: routing near-tie (margin {rgap:.1e}) at step {step}, diff {diff:.2e}: stop")
            break
        worst = max(worst, diff)
        assert diff <= atol, f"step {step}"
        # an argmax may only differ where the oracle's own top-2 gap is within the
        # numerical difference of the two paths
        if margin > 2 * diff:
            assert g_tok == O.argmax(lo), f"step {step} margin {margin} diff {diff}"
        pos += 1
    print(f"{name}: max |logit diff| over 64 steps = {worst:.2e}")


@pytest.mark.parametrize("name", MODELS)
def test_fp16_kv_logits_within_tolerance(engines_f16kv, tiny_models, name):
    """The default fp16 KV cache: teacher-forced logits stay within LOGIT_ATOL_F16KV."""
    e = engines_f16kv[name]
    e.kv_reset()
    ref = O.Model(tiny_models[name])
    prompt = [t % ref.vocab for t in PROMPT]
    lg = e.prefill(prompt)
    lo = ref.forward(prompt, 0)
    worst = float(np.abs(lg - lo).max())
    pos = len(prompt)
    route_tie = False
    for step in range(32):
        tok = O.argmax(lo)
        g_logits, _ = e.decode(tok, pos)
        lo, rgap = oracle_step(ref, [tok], pos)
        route_tie = route_tie or rgap <= ROUTE_TIE
        diff = float(np.abs(g_logits - lo).max())
        if diff > LOGIT_ATOL_F16KV and route_tie and step >= ROUTE_MIN_STEPS:
            break
        worst = max(worst, diff)
        pos += 1
    print(f"{name} fp16 KV: max |logit diff| over 32 steps = {worst:.2e}")
    assert worst <= LOGIT_ATOL_F16KV


@pytest.mark.parametrize("name", MODELS)
def test_greedy_64_identical(engines, tiny_models, name):
    e = engines[name]
    e.kv_reset()
    ref = O.Model(tiny_models[name])
    prompt = [t % ref.vocab for t in PROMPT]
    want = ref.greedy(prompt, 64)
    lg = e.prefill(prompt)
    first = O.argmax(lg)
    got = [first] + e.decode_greedy(first, len(prompt), 63)
    if name not in GREEDY_TIE_PRONE:
        assert got == want
        return
    # tie-prone model: the sequences may part only where the oracle itself is near a tie (of
    # its top two logits, or, with experts, of its routing at that step or before)
    if got != want:
        k = next(i for i, (a, b) in enumerate(zip(got, want)) if a != b)
        lo = ref.__class__(tiny_models[name]).forward(prompt + want[:k], 0) if k else ref.forward(prompt, 0)
        top2 = np.sort(lo)[-2:]
        if top2[1] - top2[0] > 2 * LOGIT_ATOL_TIES and getattr(ref, "n_expert", 0):
            walk = ref.__class__(tiny_models[name])
            _, gap = oracle_step(walk, prompt, 0)
            for i in range(k):
                _, g = oracle_step(walk, [want[i]], len(prompt) + i)
                gap = min(gap, g)
            assert k >= ROUTE_MIN_STEPS and gap <= ROUTE_TIE, f"diverged at step {k}, routing margin {gap}"
            return
        assert top2[1] - top2[0] <= 2 * LOGIT_ATOL_TIES, f"diverged at step {k} with margin {top2[1] - top2[0]}"


def test_infer_protocol_and_limits(engines):
    from tpt_spark_b200.engine import EngineError, InferenceParams

    e = engines["tiny_q4km"]
    e.kv_reset()
    events = []
    e.infer(InferenceParams(prompt=PROMPT, max_tokens=7, temperature=0.0, repeat_penalty=1.0), events.append)
    assert [ev.done for ev in events] == [False] * 7 + [True]
    pf, dc, n_prompt, n_gen = e.last_timing()
    assert n_gen == 7 and n_prompt == len(PROMPT)
    # EOS stop: make the first generated token the EOS id
    e.kv_reset()
    first = events[0].token_id
    ev2 = []
    e.infer(InferenceParams(prompt=PROMPT, max_tokens=7, temperature=0.0, repeat_penalty=1.0, eos_token_id=first),
            ev2.append)
    assert [ev.done for ev in ev2] == [True]
    # cancellation from the callback: done=True is still delivered
    e.kv_reset()
    ev3 = []

    def cancel_after_two(ev):
        ev3.append(ev)
        if len(ev3) == 2 and not ev.done:
            raise KeyboardInterrupt("stop")

    with pytest.raises(EngineError) as ei:
        e.infer(InferenceParams(prompt=PROMPT, max_tokens=50, temperature=0.0, repeat_penalty=1.0),
                cancel_after_two)
    assert ei.value.code == -9
    assert ev3[-1].done and len(ev3) == 3


def test_infer_greedy_matches_oracle_with_repeat_penalty(engines, tiny_models):
    from tpt_spark_b200.engine import InferenceParams

    e = engines["tiny_q8_0"]
    e.kv_reset()
    ref = O.Model(tiny_models["tiny_q8_0"])
    prompt = [t % ref.vocab for t in PROMPT]
    events = []
    e.infer(InferenceParams(prompt=prompt, max_tokens=20, temperature=0.0, repeat_penalty=1.3), events.append)
    got = [ev.token_id for ev in events if not ev.done]
    toks = list(prompt)
    lg = ref.forward(prompt, 0)
    want = []
    pos = len(prompt)
    for _ in range(20):
        nxt = O.argmax(O.repeat_penalty(lg, toks, 1.3))
        want.append(nxt)
        toks.append(nxt)
        lg = ref.forward([nxt], pos)
        pos += 1
    assert got == want


def test_prefix_reuse_and_reset(engines):
    from tpt_spark_b200.engine import InferenceParams

    e = engines["tiny_q4km"]
    e.kv_reset()
    assert e.kv_len() == 0 and e.kv_prefix_len(PROMPT) == 0  # reset_clears_tokens
    ev1 = []
    e.infer(InferenceParams(prompt=PROMPT, max_tokens=4, temperature=0.0, repeat_penalty=1.0), ev1.append)
    turn1 = PROMPT + [ev.token_id for ev in ev1 if not ev.done][:-1]
    assert e.kv_prefix_len(turn1 + [1, 2, 3]) == len(turn1)
    # second turn reuses the cached prefix and must equal a cold run
    follow = turn1 + [7, 8, 9]
    ev2 = []
    e.infer(InferenceParams(prompt=follow, max_tokens=5, temperature=0.0, repeat_penalty=1.0), ev2.append)
    e.kv_reset()
    ev3 = []
    e.infer(InferenceParams(prompt=follow, max_tokens=5, temperature=0.0, repeat_penalty=1.0), ev3.append)
    assert [x.token_id for x in ev2] == [x.token_id for x in ev3]


def test_load_errors(tmp_path, cuda_device, tiny_models):
    from tpt_spark_b200.engine import CudaEngine, EngineError

    e = CudaEngine(0)
    with pytest.raises(EngineError) as ei:
        e.load(str(tmp_path / "missing.gguf"))
    assert ei.value.code == -3
    bad = tmp_path / "trunc.gguf"
    data = open(tiny_models["tiny_q4km"], "rb").read()
    bad.write_bytes(data[: len(data) // 2])
    with pytest.raises(EngineError) as ei:
        e.load(str(bad))
    assert ei.value.code == -4
    notgguf = tmp_path / "x.gguf"
    notgguf.write_bytes(b"NOPE" + b"\0" * 64)
    with pytest.raises(EngineError) as ei:
        e.load(str(notgguf))
    assert ei.value.code == -4
    with pytest.raises(EngineError) as ei:
        e.decode(1, 0)
    assert not e.is_loaded()
    e.close()


def test_decode_argument_checks(engines):
    from tpt_spark_b200.engine import EngineError

    e = engines["tiny_q4km"]
    e.kv_reset()
    with pytest.raises(EngineError):
        e.decode(10**6, 0)  # token out of range
    with pytest.raises(EngineError):
        e.decode(1, 5)  # position != KV length


@pytest.mark.parametrize("name", MODELS)
def test_gemv_chain_decode_is_bit_identical(tiny_models, cuda_device, monkeypatch, name):
    """The GEMV-chain decode step (TPTC_DECODE_CHAIN=1: o, gate|up, down and the next q|k|v in
    one persistent launch with grid barriers, activations built in every CTA) computes the
    same bits as one launch per GEMV: same RMSNorm partition, same quantisation, same dots."""
    from tpt_spark_b200.engine import CudaEngine

    ref = O.Model(tiny_models[name])
    prompt = [t % ref.vocab for t in PROMPT]
    outs = []
    for mode in ("1", "0"):
        monkeypatch.setenv("TPTC_DECODE_CHAIN", mode)
        with CudaEngine(0, kv_dtype="f16") as e:
            e.load(tiny_models[name])
            lg = [e.prefill(prompt)]
            tok, pos = O.argmax(lg[0]), len(prompt)
            for _ in range(16):
                g, _ = e.decode(tok, pos)
                lg.append(g)
                tok, pos = O.argmax(g), pos + 1
            lg.append(np.asarray(e.decode_greedy(tok, pos, 8), np.float32))
            outs.append(lg)
    for a, b in zip(*outs):
        np.testing.assert_array_equal(a, b)
