"""Tensor-parallel engine on 2 GPUs (NCCL): one process per GPU, each a CudaEngine with its
Megatron shard, against the single-GPU engine on the same model and inputs.

The sharded forward differs from the single-GPU one only in the f32 summation order of the
row-parallel projections (partial sums per rank, then the allreduce), which can move a
quantised activation code by one; logits are compared teacher-forced within the north_star's
2e-2.  Skipped with fewer than 2 GPUs.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-2
PROMPT = [3, 141, 59, 26, 5, 358, 97, 93, 238, 46, 264, 33]


def _run(engine, prompt, long_prompt, steps):
    """Per-token prefill, 16 teacher-forced steps (tokens from `steps`, or greedy when None),
    then a batched prefill of the long prompt."""
    engine.set_prefill_gemm_min(0)
    lg = [engine.prefill(prompt)]
    toks, pos = [], len(prompt)
    for i in range(16):
        t = int(np.argmax(lg[-1])) if steps is None else steps[i]
        toks.append(t)
        g, _ = engine.decode(t, pos)
        lg.append(g)
        pos += 1
    engine.kv_reset()
    engine.set_prefill_gemm_min(1)
    lg.append(engine.prefill(long_prompt))
    return toks, lg


def _tp_rank(rank, size, uid, path, prompt, long_prompt, steps, q):
    from tpt_spark_b200.engine import CudaEngine

    try:
        with CudaEngine(rank, tp_rank=rank, tp_size=size, nccl_uid=uid, kv_dtype="f16") as e:
            info = e.load(path)
            _, lg = _run(e, prompt, long_prompt, steps)
            q.put((rank, info.backend, lg))
    except Exception as ex:  # reported to the parent
        q.put((rank, "error", repr(ex)))


def test_tp2_matches_single_gpu(tiny_models):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from tpt_spark_b200.engine import CudaEngine, nccl_unique_id

    path = tiny_models["tiny_tp_q4km"]
    long_prompt = [int(t) for t in np.random.default_rng(4).integers(0, 384, 100)]
    with CudaEngine(0, kv_dtype="f16") as e:
        e.load(path)
        steps, ref = _run(e, PROMPT, long_prompt, None)
    uid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, uid, path, PROMPT, long_prompt, steps, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = {}
        for _ in procs:
            r, backend, lg = q.get(timeout=300)
            assert backend != "error", lg
            assert backend.endswith("-tp2")
            got[r] = lg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    for r in range(2):
        # every rank holds the same replicated logits
        for a, b in zip(got[r], got[0]):
            np.testing.assert_array_equal(a, b)
    worst = max(float(np.abs(a - b).max()) for a, b in zip(got[0], ref))
    print(f"tp2 vs single GPU: max |logit diff| = {worst:.2e}")
    assert worst <= LOGIT_ATOL
