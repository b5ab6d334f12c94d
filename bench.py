#!/usr/bin/env python
"""bench.py -- tpt-spark hot path on B200: batch-1 decode tok/s and prefill tok/s at the
Llama-3-8B-shape Q4_K_M configuration (the benchmark configuration "C5"), plus the Q4_K GEMV
HBM GB/s of configuration "C1" (one 4096x4096 matvec).

One JSON line on rank 0.  A "step" is one decode token (one forward pass of the whole model
at batch 1).  Inputs: a seeded random-init model of the C5 shape written as a GGUF file
(weights N(0, 0.02), norm gains 1.0 -- no checkpoint exists here) and uniform random prompt
ids.  The 4.9 GB of weights is far larger than the 126 MB L2, so no L2 flush is needed
between steps.

  value           decode tok/s, CUDA events over K chained decode graphs (device argmax feeds
                  the next step), max over ranks
  e2e             the same metric through the C ABI with host buffers (tptc_decode: token id
                  and position copied in, argmax copied out, every step)
  roofline        the dominant decode kernel, the Q4_K GEMV at the C5 ffn gate|up shape
                  (28672 x 4096, 66 MB) with its activation kernel, timed with CUDA events in
                  a graph rotating through copies larger than L2; traffic from the committed
                  ncu summary of the same kernel (profiles/)
  decode_roofline the whole decode step vs measured HBM bandwidth (weights + fp16 KV / token)
  gemv_c1         C1 Q4_K 4096x4096 GEMV, rotating through 64 weight copies (> 4x L2)
  sampled         tptc_infer (the product call) decoding 64 tokens with the reference's default
                  chat parameters (temperature 0.7, top-p 0.9, repeat penalty 1.1), the token
                  selection on the device; wall time of its decode loop, max over ranks
  prefill         prefill tok/s of the prompt (device time)
  cpu_baseline    the CPU oracle (restated candle path) on the box's host cores, bounded sample

With --gpus N > 1 (torchrun, one rank per GPU) the engine is one Megatron tensor-parallel
job over the N GPUs (column-parallel q/k/v/gate/up, row-parallel o/down; in the decode step
each row-parallel GEMV stores its partial rows into every rank's inbox over NVLink and the
next activation kernel sums them, the batched prefill all-reduces with NCCL): value is the
tok/s of the one sequence all ranks decode together ("scaling": "strong"), decode_roofline
compares against the N GPUs' aggregate HBM.

--impl reference times the CPU oracle on the same workload (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "src": "measured"}
    except Exception:
        return dict(PEAKS_FALLBACK, src="fallback")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="c5_llama8b_q4km")
    ap.add_argument("--prompt", type=int, default=None, help="prompt tokens (default: the config's)")
    ap.add_argument("--model-dir", default=None, help="generated models (default: $TPTC_MODEL_DIR or <tmp>/tptc_models)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args()


PROMPT_LEN = {"c2_llama1b_q4km": 128, "c3_mistral7b_q8_0": 2048, "c4_phi3mini_f16": 1024, "c5_llama8b_q4km": 8192,
              "mixtral8x7b_l4_q4km": 512}


def workload(name):
    """A benchmark configuration (synth.CONFIGS) or a further workload (synth.WORKLOADS)."""
    from tpt_spark_b200 import synth

    return synth.CONFIGS.get(name) or synth.WORKLOADS[name]
DECODE_LEN = {"c2_llama1b_q4km": 256, "c3_mistral7b_q8_0": 512, "c4_phi3mini_f16": 256, "c5_llama8b_q4km": 1024}


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class Dist:
    """gloo process group for the benchmark's own plumbing (barriers, max over ranks)."""

    def __init__(self):
        self.rank, self.world, self.local = dist_env()
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def model_file(cfg, model_dir, seed, dist):
    from tpt_spark_b200 import synth

    if dist.local == 0:
        synth.model_file(cfg, model_dir, seed)
    dist.barrier()
    return os.path.join(model_dir, f"{cfg.name}_s{seed}.gguf")


class Clocks:
    """SM clock, power and clock-event reasons of the benchmark's GPU, read through NVML every
    5 ms in a thread (query only) while the timed region runs: `mark(True/False)` brackets the
    region, and only samples taken inside it count.  Falls back to nvidia-smi at 200 ms when
    NVML cannot be loaded."""

    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, cuda_index, period_s=0.005):
        self.cuda_index = cuda_index
        self.period = period_s
        self.rows = []  # (in_region, sm_mhz, max_mhz, watts, reasons)
        self.inside = False
        self.stop = threading.Event()
        self.thread = None
        self.nvml = None
        self.handle = None
        self.proc = None

    def _open(self):
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            pr = torch.cuda.get_device_properties(self.cuda_index)
            try:
                bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)
            self.nvml = pynvml
        except Exception:
            self.nvml = None

    def _loop(self):
        n = self.nvml
        bits = {"hw_slowdown": n.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": n.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": n.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": n.nvmlClocksEventReasonSwPowerCap}
        mx = n.nvmlDeviceGetMaxClockInfo(self.handle, n.NVML_CLOCK_SM)
        while not self.stop.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                w = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                r = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.rows.append((self.inside, float(sm), float(mx), w, {k for k, b in bits.items() if r & b}))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        self._open()
        if self.nvml is not None:
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
        else:
            self.smi = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            try:
                self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.cuda_index), f"--query-gpu={q}",
                                              "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.smi,
                                             stderr=subprocess.DEVNULL)
            except Exception:
                self.proc = None
        return self

    def mark(self, inside):
        self.inside = inside

    def __exit__(self, *a):
        self.stop.set()
        if self.thread:
            self.thread.join(2)
        elif self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()
            for line in open(self.smi.name):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 8 and parts[1].replace(".", "").isdigit():
                    rs = {k for k, v in zip(self.NAMES, parts[4:8]) if v.lower().startswith("active")}
                    self.rows.append((True, float(parts[1]), float(parts[2]), float(parts[3] or 0), rs))

    def summary(self):
        rows = [r for r in self.rows if r[0]]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(r[1] for r in rows), "sm_max_mhz": max(r[2] for r in rows),
                "reasons": sorted(set().union(*(r[4] for r in rows))), "samples": len(rows),
                "power_w_median": round(statistics.median(r[3] for r in rows), 1),
                "source": "nvml 5 ms" if self.nvml is not None else "nvidia-smi 200 ms"}


def decode_bytes(cfg, kv_len_mean):
    """Algorithmic HBM bytes of one decode step: every weight matrix once (token_embd: one row
    unless it is also the output projection; of a mixture-of-experts layer the router and the
    n_expert_used chosen experts), norm gains, and the fp16 K and V of the kv_len positions
    attended to."""
    from tpt_spark_b200 import synth

    tot = 0
    for name, kind, ne in cfg.tensors():
        n = ne[0] * (ne[1] if len(ne) > 1 else 1)
        b = synth.type_bytes(cfg.type_of(kind), n)
        if kind == "token_embd":
            tot += b if cfg.tied else b // ne[1]
        elif kind.endswith("_exps"):  # [E][rows][K]: the chosen experts' slices
            tot += b * cfg.n_expert_used
        elif cfg.n_expert > 1 and ".ffn_" in name and name.split(".")[3].isdigit():  # blk.N.ffn_*.E.weight
            tot += b * cfg.n_expert_used // cfg.n_expert
        else:
            tot += b
    tot += int(2 * cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 2 * kv_len_mean)
    return tot


def prefill_flops(cfg, P):
    """Algorithmic FLOPs of a P-token prefill: every linear layer on every token, causal
    attention (QK^T and PV over positions 0..t for token t), lm_head on the last token."""
    d, hd, L = cfg.dim, cfg.head_dim, cfg.n_layers
    nq, nk = cfg.n_heads * hd, cfg.n_kv_heads * hd
    ffn = [3 * d * cfg.ffn] * L
    for i in range(L):  # a mixture-of-experts layer: the chosen experts, the shared one, the router
        if cfg.is_moe_layer(i):
            ffn[i] = 3 * d * (cfg.expert_ffn * cfg.n_expert_used + cfg.shared_ffn) + d * cfg.n_expert
    linear = 2.0 * P * (L * (d * (nq + 2 * nk) + nq * d) + sum(ffn))
    attn = 4.0 * L * cfg.n_heads * hd * P * (P + 1) / 2
    return linear + attn + 2.0 * d * cfg.vocab


def gemv_time(torch, gtype, N, K, w_std=0.02, seed=4242, iters=256):
    """Average device time of one GEMV launch pair (activation kernel + GEMV, as in the decode
    step) over a CUDA graph of `iters` launches rotating through weight copies totalling more
    than 4x the 126 MB L2, timed with CUDA events on the graph's stream."""
    from tpt_spark_b200 import synth
    from tpt_spark_b200.kernels import Matrix

    raw = synth.encode(gtype, synth.normal(seed, N * K, w_std))
    one = synth.type_bytes(gtype, N * K)
    copies = max(2, min(64, -(-(512 << 20) // one)))
    mats = [Matrix(gtype, raw, N, K) for _ in range(copies)]
    x = torch.randn(K, device="cuda")
    y = torch.empty(N, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for m in mats[: min(copies, 8)]:
            m.gemv(x, y, s.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(iters):
                mats[i % copies].gemv(x, y, torch.cuda.current_stream().cuda_stream)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.replay()
        e1.record(s)
        torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / iters
    algo = mats[0].nbytes + K * 4 + N * 4  # weights + x + y
    del g
    for m in mats:
        m.close()
    return algo, us


def profile_traffic(name):
    """dram bytes per launch recorded in profiles/<name>.md ("dram_bytes_per_launch: N"), or None."""
    try:
        for line in open(os.path.join(ROOT, "profiles", name + ".md")):
            if line.strip().startswith("dram_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip().replace(",", ""))
    except Exception:
        pass
    return None


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(path, cfg, decode_pos, max_decode_s=20.0, prefill_tokens=64, max_steps=60):
    """The oracle (restated candle path) on all host cores, on a bounded sample of the GPU arm's
    workload:
      prefill  one batched forward of a `prefill_tokens`-token prompt (candle_engine.rs:272-281
               prefills in one forward) -- the full 8192-token prompt would take minutes here;
      decode   greedy steps at KV positions decode_pos, decode_pos + 1, ... -- the GPU arm's
               context length -- for up to max_decode_s seconds or max_steps steps.  The cache
               positions below decode_pos hold zeros instead of a prefilled prompt (no 8192-token
               CPU prefill was run), which leaves the work of every step -- the attention over
               decode_pos + 1 keys and every weight matrix once -- the same as after a real prompt.
    Returns a dict with both rates, the cores used and a description of the sample."""
    from oracle import oracle as O

    cores = os.cpu_count() or 1
    O.set_threads(cores)
    m = O.Model(path, max_seq=max(decode_pos, prefill_tokens) + max_steps + 8)
    prompt = list(range(1, prefill_tokens + 1))
    t0 = time.perf_counter()
    lg = m.forward(prompt, 0)
    pf_s = time.perf_counter() - t0
    tok = O.argmax(lg)
    pos, n = decode_pos, 0
    t0 = time.perf_counter()
    while True:
        lg = m.forward([tok], pos)
        tok = O.argmax(lg)
        pos += 1
        n += 1
        el = time.perf_counter() - t0
        if el > max_decode_s or n >= max_steps:
            break
    m.close()
    sample = (f"{n} greedy decode steps of the full {cfg.name} model at KV lengths {decode_pos + 1}..{decode_pos + n} "
              f"(positions below {decode_pos} zero-filled, not prefilled), and one {prefill_tokens}-token prefill; "
              f"{cores} OpenMP threads on {cpu_model()}")
    return {"decode_tok_s": n / el, "steps": n, "prefill_tok_s": prefill_tokens / pf_s,
            "prefill_tokens": prefill_tokens, "cores": cores, "cpu": cpu_model(), "sample": sample}


def run_reference(args, dist):
    from tpt_spark_b200 import synth

    cfg = workload(args.workload)
    if dist.rank != 0:
        return
    path = model_file(cfg, args.model_dir, args.seed, _Solo())
    P = args.prompt if args.prompt is not None else PROMPT_LEN[cfg.name]
    cb = cpu_baseline(path, cfg, decode_pos=P + args.warmup)
    tps = cb["decode_tok_s"]
    line = {"metric": "decode tok/s (bs=1)", "value": round(tps, 4), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": cb["steps"], "warmup": 0, "ms_per_step": round(1000.0 / tps, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8-dot/f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": cfg.name, "batch": 1, "prompt_tokens": P, "decode_kv_len_start": P + args.warmup + 1},
            "cpu_baseline": {"value": round(tps, 4), "unit": "tok/s", "cores": cb["cores"], "kind": "port",
                             "sample": cb["sample"], "cpu": cb["cpu"],
                             "prefill": {"value": round(cb["prefill_tok_s"], 2), "unit": "tok/s",
                                         "tokens": cb["prefill_tokens"]}},
            "e2e": {"value": round(tps, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


class _Solo:
    rank, world, local = 0, 1, 0

    def barrier(self):
        pass


def run_ours(args, dist):
    import numpy as np
    import torch

    from tpt_spark_b200 import synth
    from tpt_spark_b200.engine import CudaEngine

    cfg = workload(args.workload)
    torch.cuda.set_device(dist.local)
    path = model_file(cfg, args.model_dir, args.seed, dist)
    P = args.prompt if args.prompt is not None else PROMPT_LEN[cfg.name]
    ctx_len = cfg.context_length
    # N > 1: one Megatron tensor-parallel engine over the N GPUs (NCCL), every rank running
    # the same calls in lockstep; the NCCL id travels over the benchmark's gloo group
    if dist.world > 1:
        from tpt_spark_b200.engine import nccl_unique_id

        box = [nccl_unique_id() if dist.rank == 0 else None]
        dist.pg.broadcast_object_list(box, src=0)
        eng = CudaEngine(dist.local, tp_rank=dist.rank, tp_size=dist.world, nccl_uid=box[0])
    else:
        eng = CudaEngine(dist.local)
    info = eng.load(path)
    rng = np.random.default_rng(1234 + args.seed)
    prompt = rng.integers(0, cfg.vocab, P).tolist()

    # The prompt's KV context for the decode steps: one prefill (untimed; it also allocates the
    # prefill buffers and touches them once).  Decode is timed next, and the timed prefill
    # comes after it, so the timed decode region never follows a long prefill at full power.
    eng.kv_reset()
    lg = eng.prefill(prompt)
    tok = int(np.argmax(lg))
    # The 8192-token prefill runs at the 1 kW power cap, and the power limiter keeps the SM
    # clock lowered for a few hundred ms after it (measured on a B200: 1560 MHz with
    # sw_power_cap and 2.95 ms per decode step right after the prefill, 1965 MHz and 2.21 ms
    # from 0.38 s on, at 730 W).  A decode stream does not see that transient in steady state,
    # so the GPU idles for a second before the warm-up steps.
    torch.cuda.synchronize()
    time.sleep(1.0)

    # decode: warm-up then K timed steps; the window past the prompt is reused when the
    # context would overflow (the cache is truncated back to the prompt)
    def run_steps(n, tok):
        ms = 0.0
        kv_sum = 0.0
        done = 0
        while done < n:
            room = ctx_len - eng.kv_len()
            if room <= 0:
                eng.kv_truncate(P)
                room = ctx_len - P
            k = min(n - done, room)
            kv0 = eng.kv_len()
            out = eng.decode_greedy(tok, kv0, k)
            ms += eng.last_device_ms()
            kv_sum += k * (kv0 + 1 + kv0 + k) / 2.0
            tok = out[-1]
            done += k
        return ms, tok, kv_sum / max(n, 1)

    _, tok, _ = run_steps(args.warmup, tok)
    kv_start, tok_start = eng.kv_len(), tok  # the timed region's first position and token
    dist.barrier()
    torch.cuda.synchronize()
    with Clocks(dist.local) as clk:
        time.sleep(0.02)  # the sampler is running before the region starts
        clk.mark(True)
        torch.cuda.profiler.start()  # ncu --profile-from-start off captures only this region
        ms, tok, kv_mean = run_steps(args.steps, tok)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        clk.mark(False)
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(ms)
    tps = args.steps / (ms / 1000.0)  # one sequence decoded by all ranks together

    # end to end through the C ABI with host buffers, over the same steps and positions as the
    # timed region: each step copies the token id and position in and the argmax out
    # (the window past the prompt wraps back to the prompt where run_steps wrapped it)
    eng.kv_truncate(kv_start)
    pos, tok = kv_start, tok_start
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        if pos >= ctx_len:
            eng.kv_truncate(P)
            pos = P
        tok = eng.decode(tok, pos, want_logits=False)
        pos += 1
    e2e_s = dist.max(time.perf_counter() - t0)
    e2e_tps = args.steps / e2e_s

    # the product call with the reference's default chat parameters (InferenceParams::default:
    # temperature 0.7, top-p 0.9, repeat penalty 1.1): tptc_infer, every token selected on the
    # device; the cached prompt is reused (only its last token is recomputed)
    from tpt_spark_b200.engine import InferenceParams

    n_sampled = 64
    eng.infer(InferenceParams(prompt=prompt, max_tokens=n_sampled, seed=42), lambda ev: None)
    _, dec_ms, _, n_gen = eng.last_timing()
    sampled_tps = n_gen / dist.max(dec_ms / 1000.0) if n_gen else 0.0

    # prefill (device time), after the decode measurements
    eng.kv_reset()
    eng.prefill(prompt, want_logits=False)
    prefill_ms = dist.max(eng.last_device_ms())

    pk = peaks()
    pk.setdefault("bf16_tflops_sustained", pk["bf16_tflops"])
    pf_flops = prefill_flops(cfg, P)
    step_bytes = decode_bytes(cfg, kv_mean)
    ms_step = ms / args.steps
    achieved = step_bytes / (ms_step / 1000.0) / 1e9
    launches_per_step = eng.decode_kernels()
    os.environ.setdefault("TPTC_PDL", "1")  # kernel-level GEMVs chained as in the decode graph
    from tpt_spark_b200 import synth as _s

    dom_bytes, dom_us = gemv_time(torch, _s.Q4_K, 2 * cfg.ffn, cfg.dim)
    dom_gbs = dom_bytes / (dom_us * 1e-6) / 1e9
    C = _s.GEMV_C1
    gemv_bytes, gemv_us = gemv_time(torch, C["type"], C["N"], C["K"], C["w_std"])
    gemv_gbs = gemv_bytes / (gemv_us * 1e-6) / 1e9

    line = {
        "metric": "decode tok/s (bs=1)", "value": round(tps, 3), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "q4_k/q6_k x q8_k int8-dot, f32 accum",
        "data": "synthetic (seeded random-init GGUF, random prompt ids)",
        "config": {"workload": cfg.name, "batch": 1, "prompt_tokens": P, "decode_kv_len_mean": round(kv_mean, 1),
                   "parallelism": f"tp{dist.world}" if dist.world > 1 else "single", "l2": "inputs larger than L2 (4.9 GB weights)"},
        "e2e": {"value": round(e2e_tps, 3), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 4, "steps": args.steps,
                "path": "tptc_decode per token (token id and position in, argmax out), same positions as value"},
        "sampled": {"value": round(sampled_tps, 3), "unit": "tok/s", "tokens": n_gen,
                    "params": "temperature 0.7, top-p 0.9, repeat penalty 1.1 (the reference's defaults)",
                    "path": "tptc_infer with host callbacks; penalty, softmax, nucleus and draw on the device"},
        "roofline": {"bound": "hbm", "kernel": f"act_quant + gemv_kernel, Q4_K {2 * cfg.ffn}x{cfg.dim} (ffn gate|up shape)",
                     "achieved": round(dom_gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(dom_gbs / pk["hbm_gbs"], 4),
                     "traffic": profile_traffic(f"gemv_q4k_{2 * cfg.ffn}x{cfg.dim}"),
                     "algorithmic_bytes": dom_bytes, "us_per_launch": round(dom_us, 3), "peak_src": pk["src"]},
        "decode_roofline": {"bound": "hbm", "kernel": f"decode step ({launches_per_step} launches, CUDA graph)",
                            "achieved": round(achieved, 1), "peak": pk["hbm_gbs"] * dist.world, "unit": "GB/s",
                            "frac": round(achieved / (pk["hbm_gbs"] * dist.world), 4), "algorithmic_bytes": step_bytes,
                            "note": "whole model per step over the aggregate HBM of the GPUs"},
        "gemv_c1": {"bound": "hbm", "kernel": "gemv_kernel Q4_K 4096x4096 (C1)", "us": round(gemv_us, 3),
                    "achieved": round(gemv_gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                    "frac": round(gemv_gbs / pk["hbm_gbs"], 4), "algorithmic_bytes": gemv_bytes},
        "prefill": {"tokens": P, "ms": round(prefill_ms, 3), "tok_s": round(P / (prefill_ms / 1000.0), 1),
                    "path": "batched tcgen05 GEMM + tensor-core causal attention, fp16 operands",
                    "roofline": {"bound": "tensor", "achieved": round(pf_flops / (prefill_ms * 1e-3) / 1e12, 1),
                                 "peak": pk["bf16_tflops_sustained"] * dist.world, "unit": "TFLOP/s",
                                 "frac": round(pf_flops / (prefill_ms * 1e-3) / 1e12
                                               / (pk["bf16_tflops_sustained"] * dist.world), 4),
                                 "algorithmic_flops": pf_flops,
                                 "peak_src": pk["src"] + " (sustained bf16, times the GPUs of the job)"}},
        "clocks": clk.summary(),
        "gpu_launches": launches_per_step * args.steps,
    }
    if cfg.n_expert > 1:
        line["prefill"]["path"] = ("tokens routed on the device, grouped by expert on the host once per layer, each "
                                   "expert's rows through the tcgen05 GEMMs, combined in candle's order")
        line["config"]["experts"] = f"{cfg.n_expert_used} of {cfg.n_expert} per token"
        line["config"]["l2"] = f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB of weights per step)"
    eng.close()
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(path, cfg, decode_pos=kv_start)
        line["cpu_baseline"] = {"value": round(cb["decode_tok_s"], 4), "unit": "tok/s", "cores": cb["cores"],
                                "kind": "port", "sample": cb["sample"], "cpu": cb["cpu"],
                                "prefill": {"value": round(cb["prefill_tok_s"], 2), "unit": "tok/s",
                                            "tokens": cb["prefill_tokens"]}}
    if dist.rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.model_dir is None:
        from tpt_spark_b200 import synth

        args.model_dir = synth.default_model_dir()
    if args.impl == "reference":
        rank, world, _ = dist_env()
        if rank == 0:
            run_reference(args, _Solo())
        return
    dist = Dist()
    try:
        run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
