"""One-kernel and one-pass workloads to run under a profiler (ncu): each case makes its inputs,
launches the kernel a few times through the library's public entry points and exits.

    python -m tpt_spark_b200.profile_cases gemv 12 28672 4096   # ggml type, N, K
    python -m tpt_spark_b200.profile_cases gemm 1024 28672 4096  # fp16 GEMM, M N K
    python -m tpt_spark_b200.profile_cases gemm_q 2048 14336 4096  # fused-dequant GEMM (Q4_K), M N K
    python -m tpt_spark_b200.profile_cases attn_prefill 4096     # causal prefill attention, T
    python -m tpt_spark_b200.profile_cases attn_decode 8192      # decode attention (C5 heads), position
    python -m tpt_spark_b200.profile_cases prefill 2048          # C5 batched prefill, prompt tokens

The launch counts are what the summaries under profiles/ select with ncu's -s / -c.
"""
from __future__ import annotations

import sys


def gemv(t: int, N: int, K: int) -> None:
    """Six copies of a seeded N(0, 0.02) matrix (larger than L2 together), seven tptc_gemv calls
    cycling through them: the sixth launch is a cold read of the sixth copy."""
    import torch

    from . import synth
    from .kernels import Matrix

    raw = synth.encode(t, synth.normal(1, N * K, 0.02))
    mats = [Matrix(t, raw, N, K) for _ in range(6)]
    x = torch.randn(K, device="cuda")
    y = torch.empty(N, device="cuda")
    for i in range(7):
        mats[i % 6].gemv(x, y)
    torch.cuda.synchronize()
    print("ok", float(y.abs().sum()))


def gemm(M: int, N: int, K: int) -> None:
    """tptc_gemm_f16 three times on random fp16 A [M x K] and B [N x K] (B scaled by 0.02)."""
    import torch

    from . import kernels

    a = torch.randn(M, K, device="cuda").half()
    b = (torch.randn(N, K, device="cuda") * 0.02).half()
    c = torch.empty(M, N, device="cuda")
    for _ in range(3):
        kernels.gemm_f16(a, b, c, M, N, K)
    torch.cuda.synchronize()
    print("ok", float(c[0, 0]))


def gemm_q(M: int, N: int, K: int) -> None:
    """tptc_gemm_q four times: random fp16 A [M x K] times a Q4_K matrix of random blocks whose
    d and dmin are 0.0005 (values within +-0.5)."""
    import numpy as np
    import torch

    from .kernels import Matrix
    from .synth import Q4_K

    rng = np.random.default_rng(0)
    raw = rng.integers(0, 256, (N * K // 256, 144), dtype=np.uint8)
    h = np.frombuffer(np.float16(0.0005).tobytes(), np.uint8)
    raw[:, 0:2] = h
    raw[:, 2:4] = h
    m = Matrix(Q4_K, raw.reshape(-1), N, K)
    a = torch.randn(M, K, device="cuda").half()
    c = torch.empty(M, N, device="cuda")
    for _ in range(4):
        m.gemm(a, c, M)
    torch.cuda.synchronize()
    print("ok", float(c[0, 0]))


def attn_prefill(T: int) -> None:
    """tptc_attn_prefill three times: T query rows, 32 heads / 8 kv heads, head_dim 128, over a
    random fp16 cache of T positions."""
    import torch

    from . import kernels

    H, KV, hd = 32, 8, 128
    q = torch.randn(T, H * hd, device="cuda").half()
    kc = torch.randn(KV, T, hd, device="cuda").half()
    vc = torch.randn(KV, T, hd, device="cuda").half()
    o = torch.empty(T, H * hd, device="cuda").half()
    for _ in range(3):
        kernels.attn_prefill(q, kc, vc, o, T, 0, H, KV, hd, T)
    torch.cuda.synchronize()
    print("ok", float(o[0, 0]))


def attn_decode(pos: int) -> None:
    """tptc_attn_decode five times at position `pos` (keys 0..pos): 32 query heads over 8 kv
    heads of 128, fp16 caches of 9216 positions, one of five separate cache pairs per launch
    (188 MB together, more than L2): the fifth launch reads its keys and values cold."""
    import torch

    from . import kernels

    H, KV, hd, S = 32, 8, 128, 9216
    half = hd // 2
    theta = 500000.0 ** (-torch.arange(half, dtype=torch.float64) * 2 / hd)
    ang = torch.arange(S, dtype=torch.float64)[:, None] * theta[None, :]
    cs, sn = ang.cos().float().cuda(), ang.sin().float().cuda()
    caches = [(torch.randn(KV, S, hd, device="cuda").half(), torch.randn(KV, S, hd, device="cuda").half())
              for _ in range(5)]
    q = torch.randn(H * hd, device="cuda")
    kraw = torch.randn(KV * hd, device="cuda")
    d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    out = torch.empty(H * hd, device="cuda")
    nbytes = kernels.attn_decode_workspace_bytes(H, KV, hd, S)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    for kc, vc in caches:
        kernels.attn_decode(q, kraw, kc, vc, kernels.F16, cs, sn, d_pos, H, KV, hd, S, out, ws, nbytes)
    torch.cuda.synchronize()
    print("ok", float(out.abs().sum()))


def prefill(P: int) -> None:
    """The C5 model (the bench's synthetic GGUF in synth.default_model_dir(), written on first
    use): one warm-up prefill of P random token ids, then the same prefill bracketed by
    cudaProfilerStart / Stop (for ncu --profile-from-start off)."""
    import numpy as np
    import torch

    from . import synth
    from .engine import CudaEngine

    cfg = synth.CONFIGS["c5_llama8b_q4km"]
    path = synth.model_file(cfg)
    e = CudaEngine(0)
    e.load(path)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, P).tolist()
    e.prefill(prompt, want_logits=False)
    e.kv_reset()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    e.prefill(prompt, want_logits=False)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print("prefill ms", e.last_device_ms())


CASES = {"gemv": gemv, "gemm": gemm, "gemm_q": gemm_q, "attn_prefill": attn_prefill, "attn_decode": attn_decode,
         "prefill": prefill}


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if not argv or argv[0] not in CASES:
        print(__doc__)
        return 2
    CASES[argv[0]](*(int(v) for v in argv[1:]))
    return 0


if __name__ == "__main__":
    sys.exit(main())
