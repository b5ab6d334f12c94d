"""Device next-token selection (tptc_sample, sample.cu) against the host rules it restates.

- repeat penalty (candle_engine.rs:87-101: divide, or multiply when negative, once per context
  occurrence) and the greedy pick (ties to the highest index): bit-exact against numpy
  float32 over the same logits;
- top-p (candle sample_topp: keep every token whose strictly larger probabilities sum below
  top_p): the kernel works on fixed-point masses m = floor(e * 2^40) of e = exp(x - max); the
  test reads back the kernel's e, applies the rule in exact integer arithmetic in numpy and
  compares the cut, the kept mass and the total; a second restatement follows candle's own
  walk (stable descending sort, running float64 sum, keep while the sum before is below
  top_p) and must give the same kept set whenever no two tokens tie at the cut (with a tie at
  the cut candle keeps only a prefix of the tied tokens in index order, the kernel all);
- a temperature below 1e-7 is greedy (candle LogitsProcessor::new);
- the draw: empirical frequencies against the kept masses (statistical bound), never a token
  outside the nucleus, and the same token for the same (seed, step);
- the engine: infer with a temperature is reproducible for a seed and stays in range.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tpt_spark_b200 import kernels as K  # noqa: E402

pytestmark = pytest.mark.gpu

FIX = 2.0 ** 40


def penalised(logits, counts, penalty):
    x = logits.astype(np.float32).copy()
    if abs(np.float32(penalty) - np.float32(1.0)) < np.float32(1.1920929e-7):
        return x
    p = np.float32(penalty)
    for i in np.nonzero(counts)[0]:
        for _ in range(int(counts[i])):
            x[i] = x[i] / p if x[i] >= 0 else x[i] * p
    return x


def argmax_last(x):
    m = x.max()
    return int(np.nonzero(x == m)[0][-1])


def run(logits, counts=None, penalty=1.0, temperature=0.0, top_p=1.0, seed=0, step=0):
    dev = "cuda"
    V = logits.size
    d_lg = torch.from_numpy(logits.astype(np.float32)).to(dev)
    d_cnt = torch.from_numpy(counts.astype(np.int32)).to(dev) if counts is not None else None
    d_step = torch.tensor([step], dtype=torch.int32, device=dev)
    d_scr = torch.empty(V, dtype=torch.float32, device=dev)
    d_out = torch.full((1,), -1, dtype=torch.int32, device=dev)
    d_dbg = torch.zeros(3, dtype=torch.int64, device=dev)
    K.sample(d_lg, V, d_cnt, penalty, temperature, top_p, seed, d_step, d_scr, d_out, d_dbg)
    torch.cuda.synchronize()
    return (int(d_out.item()), d_scr.cpu().numpy(), d_dbg.cpu().numpy().view(np.uint64),
            None if d_cnt is None else d_cnt.cpu().numpy(), int(d_step.item()))


@pytest.mark.parametrize("V", [1000, 128256])
@pytest.mark.parametrize("penalty", [1.0, 1.1, 0.9, 1.3])
def test_greedy_with_repeat_penalty_bit_exact(cuda_device, V, penalty):
    rng = np.random.default_rng(V + int(penalty * 10))
    for trial in range(4):
        lg = (rng.standard_normal(V) * 3).astype(np.float32)
        lg[rng.integers(0, V, 5)] = lg.max()  # ties at the top: the highest index wins
        hist = rng.integers(0, V, 300)
        hist = np.concatenate([hist, hist[:50], hist[:10]])  # duplicates count once each
        counts = np.bincount(hist, minlength=V).astype(np.int32)
        tok, _, _, cnt_after, step_after = run(lg, counts, penalty=penalty, temperature=0.0)
        want = argmax_last(penalised(lg, counts, penalty))
        assert tok == want
        assert cnt_after[tok] == counts[tok] + 1 and step_after == 1


def kept_rule(e, top_p):
    """candle sample_topp's kept set on fixed-point masses: keep iff the mass of strictly
    larger values is below ceil(top_p * total)."""
    m = (e.astype(np.float32) * np.float32(FIX)).astype(np.uint64)
    total = int(m.sum())
    if not (0.0 < top_p < 1.0):
        return 0, total, total
    target = int(np.ceil(np.float64(np.float32(top_p)) * np.float64(total)))
    order = np.argsort(-e, kind="stable")
    es, ms = e[order], m[order]
    # walk the distinct values from the top with the mass strictly above each
    keep_min = None
    acc = 0
    i = 0
    n = es.size
    while i < n:
        j = i
        grp = 0
        while j < n and es[j] == es[i]:
            grp += int(ms[j])
            j += 1
        if acc < target:
            keep_min = es[i]
        else:
            break
        acc += grp
        i = j
    kept = int(m[e >= keep_min].sum())
    return int(np.float32(keep_min).view(np.uint32)), kept, total


def candle_topp_kept(e, top_p):
    """candle sample_topp restated in float64: probabilities e / sum(e), indices sorted by
    descending probability (stable), a running sum; an index is kept while the sum of the
    indices before it is below top_p.  Returns (kept mask, the running sum where the walk
    stopped keeping, i.e. the boundary the decision was taken at)."""
    e64 = e.astype(np.float64)
    p = e64 / e64.sum()
    order = np.argsort(-p, kind="stable")
    before = np.cumsum(p[order]) - p[order]
    keep_sorted = before < top_p
    kept = np.zeros(e.size, bool)
    kept[order[keep_sorted]] = True
    n = int(keep_sorted.sum())
    boundary = before[n] if n < e.size else 1.0
    return kept, boundary


@pytest.mark.parametrize("V,temperature,top_p", [(1000, 1.0, 0.9), (128256, 0.7, 0.9), (128256, 0.7, 0.5),
                                                 (50000, 2.0, 0.99), (4096, 0.3, 1e-6), (4096, 1.0, 1.0)])
def test_top_p_cut_matches_rule(cuda_device, V, temperature, top_p):
    rng = np.random.default_rng(V)
    lg = (rng.standard_normal(V) * 4).astype(np.float32)
    lg[:3] = lg[3]  # a tie among the values
    tok, e, dbg, _, _ = run(lg, None, temperature=temperature, top_p=top_p, seed=5)
    x = lg / np.float32(temperature)
    assert np.isclose(e.max(), 1.0) and np.all(e >= 0)
    # e is exp(x - max) up to the GPU expf's rounding
    np.testing.assert_allclose(e, np.exp((x - x.max()).astype(np.float64)), rtol=2e-6, atol=1e-30)
    cut, kept, total = kept_rule(e, top_p)
    assert int(dbg[2]) == total
    assert int(dbg[0]) == cut
    assert int(dbg[1]) == kept
    bits = e.view(np.uint32)
    assert bits[tok] >= cut and e[tok] > 0
    if 0.0 < top_p < 1.0:
        ck, boundary = candle_topp_kept(e, top_p)
        cut_val = np.uint32(cut).view(np.float32)
        tie_at_cut = int((e == cut_val).sum()) > 1
        if not tie_at_cut and abs(boundary - top_p) > 1e-9:
            np.testing.assert_array_equal(bits >= cut, ck)


def test_tiny_temperature_is_greedy(cuda_device):
    """candle's LogitsProcessor::new takes a temperature below 1e-7 as none: argmax."""
    rng = np.random.default_rng(11)
    lg = (rng.standard_normal(128256) * 3).astype(np.float32)
    for t in (1e-9, 5e-8, 0.0, -1.0):
        assert run(lg, None, temperature=t, top_p=0.9, seed=3)[0] == argmax_last(lg)


def test_draws_follow_the_kept_masses(cuda_device):
    V, N = 40, 6000
    rng = np.random.default_rng(3)
    lg = (rng.standard_normal(V) * 1.5).astype(np.float32)
    dev = "cuda"
    d_lg = torch.from_numpy(lg).to(dev)
    d_step = torch.zeros(1, dtype=torch.int32, device=dev)
    d_scr = torch.empty(V, dtype=torch.float32, device=dev)
    d_out = torch.full((N,), -1, dtype=torch.int32, device=dev)
    for i in range(N):
        K.sample(d_lg, V, None, 1.0, 1.0, 0.8, 1234, d_step, d_scr, d_out[i:i + 1])
    torch.cuda.synchronize()
    toks = d_out.cpu().numpy()
    assert int(d_step.item()) == N
    e = d_scr.cpu().numpy()
    cut, kept, _ = kept_rule(e, 0.8)
    m = (e * np.float32(FIX)).astype(np.uint64).astype(np.float64)
    keep = e.view(np.uint32) >= cut
    p = np.where(keep, m, 0.0) / kept
    assert np.all(keep[toks]), "a token outside the nucleus was drawn"
    freq = np.bincount(toks, minlength=V) / N
    sd = np.sqrt(p * (1 - p) / N)
    assert np.all(np.abs(freq - p) <= 5 * sd + 1e-3), (freq, p)


def test_same_seed_and_step_same_token(cuda_device):
    rng = np.random.default_rng(9)
    lg = rng.standard_normal(128256).astype(np.float32)
    a = [run(lg, None, temperature=1.0, top_p=0.95, seed=77, step=s)[0] for s in range(6)]
    b = [run(lg, None, temperature=1.0, top_p=0.95, seed=77, step=s)[0] for s in range(6)]
    c = [run(lg, None, temperature=1.0, top_p=0.95, seed=78, step=s)[0] for s in range(6)]
    assert a == b
    assert a != c


def test_infer_with_temperature_is_reproducible(tiny_models, cuda_device):
    """LlmEngine::infer with the reference's default sampling (T 0.7, top-p 0.9, penalty 1.1):
    the whole selection runs on the device; the stream is reproducible for a seed."""
    from tpt_spark_b200.engine import CudaEngine, InferenceParams

    with CudaEngine(0) as e:
        e.load(tiny_models["tiny_q4km"])
        streams = []
        for seed in (7, 7, 8):
            e.kv_reset()
            ev = []
            e.infer(InferenceParams(prompt=[1, 5, 9, 13, 2, 7], max_tokens=24, seed=seed), ev.append)
            assert ev[-1].done
            streams.append([x.token_id for x in ev if not x.done])
        vocab = e.model_info().vocab
    assert streams[0] == streams[1]
    assert streams[0] != streams[2]
    assert all(0 <= t < vocab for s in streams for t in s) and len(streams[0]) == 24
