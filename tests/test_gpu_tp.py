"""Tensor-parallel engine on 2 GPUs (NCCL plus peer memory): one process per GPU, each a
CudaEngine with its Megatron shard, against the single-GPU engine on the same model and inputs.

The sharded forward differs from the single-GPU one only in the f32 summation order of the
row-parallel projections (partial sums per rank, then the reduction), which can move a
quantised activation code by one; logits are compared teacher-forced within the north_star's
2e-2.  The lm_head is vocab-parallel: every rank computes its rows, the greedy pick is
exchanged over peer memory (checked against the argmax of the gathered logits, ties to the
highest index), and the full logits are an all-gather.  A rank that stops taking steps makes
the other's next step fail with TPTC_ERR_TIMEOUT within the wait bound (and its own late step
too), and both recover.
Skipped with fewer than 2 GPUs.
"""
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-2
PROMPT = [3, 141, 59, 26, 5, 358, 97, 93, 238, 46, 264, 33]
TIMEOUT = -10  # TPTC_ERR_TIMEOUT
WAIT_POLLS = 500_000  # reads before a tensor-parallel wait gives up: a few tenths of a second


def argmax_last(x):
    return int(np.nonzero(x == x.max())[0][-1])


def _run(engine, prompt, long_prompt, steps):
    """Per-token prefill, 16 teacher-forced steps (tokens from `steps`, or greedy when None),
    chained greedy decoding from the prompt, then a batched prefill of the long prompt."""
    engine.set_prefill_gemm_min(0)
    lg = [engine.prefill(prompt)]
    toks, picks, pos = [], [], len(prompt)
    for i in range(16):
        t = argmax_last(lg[-1]) if steps is None else steps[i]
        toks.append(t)
        g, am = engine.decode(t, pos)
        lg.append(g)
        picks.append(am)
        pos += 1
    engine.kv_reset()
    first = argmax_last(engine.prefill(prompt))
    chained = [first] + engine.decode_greedy(first, len(prompt), 15)
    engine.kv_reset()
    engine.set_prefill_gemm_min(1)
    lg.append(engine.prefill(long_prompt))
    return toks, lg, picks, chained


def _spawn(target, args_for_rank, n=2, timeout=300):
    """Runs target(*args_for_rank(r), queue, event_a, event_b, barrier) in n spawned processes
    and returns {rank: payload}; a rank that reports an error fails the test."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    extra = [ctx.Event(), ctx.Event(), ctx.Barrier(n)]
    procs = [ctx.Process(target=target, args=args_for_rank(r) + (q, *extra)) for r in range(n)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in procs:
            r, status, payload = q.get(timeout=timeout)
            assert status != "error", payload
            got[r] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    return got


def _tp_rank(rank, size, uid, path, prompt, long_prompt, steps, q, ev_a, ev_b, barrier):
    from tpt_spark_b200.engine import CudaEngine

    try:
        with CudaEngine(rank, tp_rank=rank, tp_size=size, nccl_uid=uid, kv_dtype="f16") as e:
            info = e.load(path)
            _, lg, picks, chained = _run(e, prompt, long_prompt, steps)
            q.put((rank, info.backend, (lg, picks, chained)))
    except Exception as ex:  # reported to the parent
        q.put((rank, "error", repr(ex)))


def test_tp2_matches_single_gpu(tiny_models):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from tpt_spark_b200.engine import CudaEngine, nccl_unique_id

    path = tiny_models["tiny_tp_q4km"]
    long_prompt = [int(t) for t in np.random.default_rng(4).integers(0, 384, 100)]
    with CudaEngine(0, kv_dtype="f16") as e:
        e.load(path)
        steps, ref, _, _ = _run(e, PROMPT, long_prompt, None)
    uid = nccl_unique_id()
    got = _spawn(_tp_rank, lambda r: (r, 2, uid, path, PROMPT, long_prompt, steps))
    for r in range(2):
        assert got[r][0].endswith("-tp2")
    lg0, picks0, chained0 = got[0][1]
    for r in range(2):
        lg, picks, chained = got[r][1]
        # every rank holds the same gathered logits and picks the same tokens
        for a, b in zip(lg, lg0):
            np.testing.assert_array_equal(a, b)
        assert picks == picks0 and chained == chained0
    # the vocab-parallel pick is the argmax of the gathered logits (ties to the highest index)
    assert picks0 == [argmax_last(g) for g in lg0[1:17]]
    # chained greedy decoding on the device follows the step-by-step picks wherever those
    # are the greedy path of the teacher-forced tokens (the single GPU's greedy sequence)
    own = [argmax_last(lg0[0])] + picks0[:15]
    if own == list(steps):
        assert chained0 == own
    print(f"tp2 greedy {'matches' if own == list(steps) else 'leaves'} the single-GPU greedy sequence")
    worst = max(float(np.abs(a - b).max()) for a, b in zip(lg0, ref))
    print(f"tp2 vs single GPU: max |logit diff| = {worst:.2e}")
    assert worst <= LOGIT_ATOL


def _stall_rank(rank, uid, path, q, ev_stalled, ev_release, barrier):
    """Both ranks decode two steps; rank 1 then skips the third and waits (its context and
    inboxes stay alive, no kernel of it in flight).  Rank 0's third step must fail with
    TPTC_ERR_TIMEOUT within the bound.  Rank 0 does not stop at the wait that gave up: it runs
    the rest of the step (every later wait gives up within 256 reads), so its layer-1 rows
    overwrite its layer-0 rows in rank 1's inbox.  Rank 1's late third step therefore fails
    with TPTC_ERR_TIMEOUT too -- it never consumes a word of another step, because every
    word carries its (step, use) epoch -- and both step counters agree again.  A fresh prompt
    on both ranks then gives the logits of the first run.  The wait bound must exceed the skew
    between the two host processes in a step taken together (they meet at a barrier before
    each phase).  Errors are reported before the engine is destroyed: destroying an NCCL
    communicator waits for the peer's."""
    from tpt_spark_b200.engine import CudaEngine, EngineError

    def step_code(e, tok, pos):
        t0 = time.perf_counter()
        try:
            e.decode(tok, pos, want_logits=False)
            code = 0
        except EngineError as ex:
            code = ex.code
        return code, time.perf_counter() - t0

    try:
        with CudaEngine(rank, tp_rank=rank, tp_size=2, nccl_uid=uid, kv_dtype="f16") as e:
            try:
                e.set_tp_wait_polls(WAIT_POLLS)
                e.load(path)
                e.set_prefill_gemm_min(0)
                barrier.wait(120)
                first = e.prefill(PROMPT)
                pos = len(PROMPT)
                ref = []
                for t in (5, 6):
                    ref.append(e.decode(t, pos)[0])
                    pos += 1
                out = {}
                if rank == 1:
                    if not ev_stalled.wait(120):
                        raise RuntimeError("rank 0 did not report its stalled step")
                    out["code"], out["seconds"] = step_code(e, 7, pos)  # the same step counter again
                    ev_release.set()
                else:
                    out["code"], out["seconds"] = step_code(e, 7, pos)
                    ev_stalled.set()
                    if not ev_release.wait(120):
                        raise RuntimeError("rank 1 did not take its late step")
                # recovery: both ranks start over on the same prompt
                barrier.wait(120)
                e.kv_reset()
                again = e.prefill(PROMPT)
                pos = len(PROMPT)
                redo = []
                for t in (5, 6):
                    redo.append(e.decode(t, pos)[0])
                    pos += 1
                out["same"] = bool(
                    np.array_equal(again, first) and all(np.array_equal(a, b) for a, b in zip(redo, ref))
                )
                q.put((rank, "ok", out))
            except Exception as ex:
                q.put((rank, "error", repr(ex)))
                barrier.abort()  # the other rank stops waiting at its next barrier
    except Exception as ex:
        q.put((rank, "error", repr(ex)))


def test_tp2_stalled_rank_times_out_and_recovers(tiny_models, monkeypatch):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from tpt_spark_b200.engine import nccl_unique_id

    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")  # no NVLink multicast objects in a failure test
    uid = nccl_unique_id()
    path = tiny_models["tiny_tp_q4km"]
    got = _spawn(_stall_rank, lambda r: (r, uid, path))
    r0, r1 = got[0][1], got[1][1]
    print(f"rank 0's step without rank 1: code {r0['code']} after {r0['seconds']:.3f} s; "
          f"rank 1's late step: code {r1['code']} after {r1['seconds']:.3f} s")
    assert r0["code"] == TIMEOUT and r1["code"] == TIMEOUT
    assert r0["seconds"] < 10 and r1["seconds"] < 10
    assert got[0][1]["same"] and got[1][1]["same"]
