"""Megatron tensor-parallel sharding on CPU: the loader's shard plan (tptc_tp_shard) and the
sharded layer arithmetic it implies, checked with gloo ranks (world size 2) against the
unsharded layer.

Each rank keeps whole query heads with their kv heads (column-parallel q / k / v), whole ffn
rows (column-parallel gate / up) and the matching input columns of o and down (row-parallel);
after each row-parallel projection the ranks sum-allreduce into the replicated residual
stream.  The float64 layer below is the engine's per-rank step written out in numpy over the
oracle's dequantised weights: with the plan's windows its allreduced result must equal the
unsharded layer to rounding.
"""
import os

import numpy as np
import pytest

from tpt_spark_b200 import synth
from tpt_spark_b200.engine import EngineError, tp_shard

SHAPES = {name: cfg for name, cfg in synth.CONFIGS.items()}
SHAPES["tiny_tp_q4km"] = synth.TINY["tiny_tp_q4km"]


def _windows(cfg, which, size):
    return [tp_shard(which, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.dim, cfg.ffn, r, size) for r in range(size)]


@pytest.mark.parametrize("name", sorted(SHAPES))
@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_shards_partition_every_weight(name, size):
    cfg = SHAPES[name]
    full = {"q": (cfg.n_heads * cfg.head_dim, cfg.dim), "k": (cfg.n_kv_heads * cfg.head_dim, cfg.dim),
            "v": (cfg.n_kv_heads * cfg.head_dim, cfg.dim), "o": (cfg.dim, cfg.n_heads * cfg.head_dim),
            "gate": (cfg.ffn, cfg.dim), "up": (cfg.ffn, cfg.dim), "down": (cfg.dim, cfg.ffn)}
    try:
        win = {w: _windows(cfg, w, size) for w in full}
    except EngineError:
        # only shapes that cannot split evenly are refused
        qd = cfg.n_heads // size * cfg.head_dim if cfg.n_heads % size == 0 else 1
        assert cfg.n_kv_heads % size or cfg.ffn % (256 * size) or (size > 1 and qd % 256)
        return
    for w, (N, K) in full.items():
        rows = sorted((r0, r1) for r0, r1, _, _ in win[w])
        cols = sorted((k0, k1) for _, _, k0, k1 in win[w])
        col_parallel = w in ("q", "k", "v", "gate", "up")
        if col_parallel:
            assert all(c == (0, K) for c in cols)
            assert rows[0][0] == 0 and rows[-1][1] == N
            assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))
        else:
            assert all(r == (0, N) for r in rows)
            assert cols[0][0] == 0 and cols[-1][1] == K
            assert all(a[1] == b[0] for a, b in zip(cols, cols[1:]))
            assert all((k1 - k0) % 256 == 0 for k0, k1 in cols)  # whole quant blocks
    for r in range(size):
        # the rank's query heads read only its own kv heads (GQA group h // G)
        G = cfg.n_heads // cfg.n_kv_heads
        q0, q1 = win["q"][r][:2]
        k0, k1 = win["k"][r][:2]
        heads = range(q0 // cfg.head_dim, q1 // cfg.head_dim)
        assert all(k0 // cfg.head_dim <= h // G < k1 // cfg.head_dim for h in heads)
        # o's input columns are exactly the rank's attention outputs, down's its ffn rows
        assert win["o"][r][2:] == (q0, q1)
        assert win["down"][r][2:] == win["gate"][r][:2] == win["up"][r][:2]


def _layer(x, W, cfg, pos, heads, kvh, cache):
    """One decoder layer for one token (float64): q/k/v of `heads` / `kvh` only, attention over
    `cache` (appended), partial o and down products over those heads / ffn rows."""
    hd, G = cfg.head_dim, cfg.n_heads // cfg.n_kv_heads

    def rms(v, g):
        return v / np.sqrt((v * v).mean() + 1e-5) * g

    xn = rms(x, W["attn_norm"])
    q = (W["q"] @ xn).reshape(-1, hd)
    k = (W["k"] @ xn).reshape(-1, hd)
    v = (W["v"] @ xn).reshape(-1, hd)
    ang = pos / cfg.rope_base ** (np.arange(0, hd, 2) / hd)
    c, s = np.cos(ang), np.sin(ang)

    def rope(t):
        r = t.copy()
        r[:, 0::2] = t[:, 0::2] * c - t[:, 1::2] * s
        r[:, 1::2] = t[:, 0::2] * s + t[:, 1::2] * c
        return r

    q, k = rope(q), rope(k)
    cache.append((k, v))
    K = np.stack([kv[0] for kv in cache], 1)  # [kvh, pos+1, hd]
    V = np.stack([kv[1] for kv in cache], 1)
    att = np.empty_like(q)
    for i, h in enumerate(heads):
        j = h // G - kvh[0]
        sc = K[j] @ q[i] / np.sqrt(hd)
        p = np.exp(sc - sc.max())
        att[i] = (p / p.sum()) @ V[j]
    o_part = W["o"] @ att.reshape(-1)
    return o_part


def _ffn(x, W):
    xn = x / np.sqrt((x * x).mean() + 1e-5) * W["ffn_norm"]
    g, u = W["gate"] @ xn, W["up"] @ xn
    return W["down"] @ (g / (1 + np.exp(-g)) * u)


def _weights(cfg, seed):
    rng = np.random.default_rng(seed)
    D, hd = cfg.dim, cfg.head_dim
    return {"attn_norm": 1 + 0.1 * rng.standard_normal(D), "ffn_norm": 1 + 0.1 * rng.standard_normal(D),
            "q": 0.05 * rng.standard_normal((cfg.n_heads * hd, D)),
            "k": 0.05 * rng.standard_normal((cfg.n_kv_heads * hd, D)),
            "v": 0.05 * rng.standard_normal((cfg.n_kv_heads * hd, D)),
            "o": 0.05 * rng.standard_normal((D, cfg.n_heads * hd)),
            "gate": 0.05 * rng.standard_normal((cfg.ffn, D)), "up": 0.05 * rng.standard_normal((cfg.ffn, D)),
            "down": 0.05 * rng.standard_normal((D, cfg.ffn))}


def _shard(W, cfg, rank, size):
    out = {"attn_norm": W["attn_norm"], "ffn_norm": W["ffn_norm"]}
    for w in ("q", "k", "v", "o", "gate", "up", "down"):
        r0, r1, k0, k1 = tp_shard(w, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.dim, cfg.ffn, rank, size)
        out[w] = W[w][r0:r1, k0:k1]
    return out


def _rank_main(rank, size, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        cfg = synth.TINY["tiny_tp_q4km"]
        W = _weights(cfg, 3)
        S = _shard(W, cfg, rank, size)
        hd = cfg.head_dim
        q0, q1 = tp_shard("q", cfg.n_heads, cfg.n_kv_heads, hd, cfg.dim, cfg.ffn, rank, size)[:2]
        k0, k1 = tp_shard("k", cfg.n_heads, cfg.n_kv_heads, hd, cfg.dim, cfg.ffn, rank, size)[:2]
        heads, kvh = list(range(q0 // hd, q1 // hd)), list(range(k0 // hd, k1 // hd))
        x = np.random.default_rng(9).standard_normal(cfg.dim)
        cache = []
        for pos in range(5):  # a few positions through the sharded layer
            t = torch.from_numpy(_layer(x, S, cfg, pos, heads, kvh, cache))
            dist.all_reduce(t)  # row-parallel o: sum of partial products
            x = x + t.numpy()
            t = torch.from_numpy(_ffn(x, S))
            dist.all_reduce(t)  # row-parallel down
            x = x + t.numpy()
        q.put((rank, x))
    finally:
        dist.destroy_process_group()


def test_sharded_layer_matches_unsharded_gloo():
    import socket

    import torch.multiprocessing as mp

    cfg = synth.TINY["tiny_tp_q4km"]
    W = _weights(cfg, 3)
    x = np.random.default_rng(9).standard_normal(cfg.dim)
    cache = []
    for pos in range(5):
        x = x + _layer(x, W, cfg, pos, list(range(cfg.n_heads)), list(range(cfg.n_kv_heads)), cache)
        x = x + _ffn(x, W)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        np.testing.assert_allclose(got[r], x, rtol=1e-12, atol=1e-12)
