"""The synthetic-model writer: files read back by gguf-py with the metadata the reference's
loader expects, and block encodings that gguf-py decodes.  CPU only."""
import numpy as np
import pytest

from tpt_spark_b200 import synth


def test_roundtrip_through_gguf_py(tiny_models):
    import gguf

    cfg = synth.TINY["tiny_q4km"]
    r = gguf.GGUFReader(tiny_models["tiny_q4km"])

    def field(k):
        f = r.fields[k]
        v = f.parts[f.data[0]]
        return bytes(v).decode() if f.types[0] == gguf.GGUFValueType.STRING else v[0].item()

    assert field("general.architecture") == "llama"
    assert field("llama.embedding_length") == cfg.dim
    assert field("llama.block_count") == cfg.n_layers
    assert field("llama.attention.head_count") == cfg.n_heads
    assert field("llama.attention.head_count_kv") == cfg.n_kv_heads
    assert field("llama.feed_forward_length") == cfg.ffn
    assert field("llama.rope.dimension_count") == cfg.head_dim
    assert abs(field("llama.rope.freq_base") - cfg.rope_base) < 1e-3
    names = {t.name: t for t in r.tensors}
    for name, kind, ne in cfg.tensors():
        t = names[name]
        assert list(t.shape) == ne
        assert int(t.tensor_type) == cfg.type_of(kind)
    # every tensor decodes with gguf-py
    from gguf import quants as Q

    for t in r.tensors:
        v = Q.dequantize(np.asarray(t.data), t.tensor_type)
        assert np.isfinite(v).all()


@pytest.mark.parametrize("t", [synth.Q8_0, synth.F16])
def test_encoders_match_gguf_py(t):
    from gguf import GGMLQuantizationType as G
    from gguf import quants as Q

    x = synth.normal(99, 32 * 256, 0.02)
    mine = synth.encode(t, x)
    ref = Q.quantize(x.reshape(1, -1), G.Q8_0 if t == synth.Q8_0 else G.F16).view(np.uint8).ravel()
    np.testing.assert_array_equal(mine, ref)


@pytest.mark.parametrize("t", [synth.Q4_K, synth.Q6_K])
def test_kquant_encoders_within_bounds(t):
    from gguf import GGMLQuantizationType as G
    from gguf import quants as Q

    x = synth.normal(5, 64 * 256, 0.02)
    raw = synth.encode(t, x)
    y = Q.dequantize(raw, G.Q4_K if t == synth.Q4_K else G.Q6_K).ravel()
    err = np.abs(y - x)
    assert err.max() < (0.01 if t == synth.Q4_K else 0.004)
    assert np.sqrt((err ** 2).mean()) < (0.004 if t == synth.Q4_K else 0.001)


def test_normal_draw_is_stable():
    a = synth.normal(1234, 1000, 1.0)
    b = synth.normal(1234, 500, 1.0, start=500)
    np.testing.assert_array_equal(a[500:], b)
    assert abs(a.mean()) < 0.15 and abs(a.std() - 1) < 0.1


def test_moe_models_roundtrip_and_bench_accounting(tiny_models):
    """The mixture-of-experts writers: expert metadata, stacked ([E][rows][K]) and per-expert
    tensors and the router read back by gguf-py; bench.py counts the chosen experts' bytes
    per decode step and their FLOPs per prefilled token, the dense configurations unchanged."""
    import os
    import sys

    import gguf

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench

    for name in ("tiny_mixtral", "tiny_moe"):
        cfg = synth.TINY[name]
        r = gguf.GGUFReader(tiny_models[name])
        t = {x.name: x for x in r.tensors}
        f = r.fields
        assert f["llama.expert_count"].parts[-1][0] == cfg.n_expert
        assert f["llama.expert_used_count"].parts[-1][0] == cfg.n_expert_used
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            if not cfg.is_moe_layer(i):
                assert p + "ffn_gate.weight" in t and p + "ffn_gate_inp.weight" not in t
                continue
            assert list(t[p + "ffn_gate_inp.weight"].shape) == [cfg.dim, cfg.n_expert]
            assert int(t[p + "ffn_gate_inp.weight"].tensor_type) == cfg.router_type
            if cfg.stacked_experts:
                assert list(t[p + "ffn_down_exps.weight"].shape) == [cfg.expert_ffn, cfg.dim, cfg.n_expert]
            else:
                assert list(t[p + f"ffn_up.{cfg.n_expert - 1}.weight"].shape) == [cfg.dim, cfg.expert_ffn]
            assert (p + "ffn_gate_shexp.weight" in t) == bool(cfg.shared_ffn)

    # decode bytes: one of each dense tensor, the router and n_used of n_expert experts
    def layer_bytes(cfg, i):
        tb = synth.type_bytes
        d, ef = cfg.dim, cfg.expert_ffn
        router = tb(cfg.type_of("ffn_gate_inp"), d * cfg.n_expert)
        experts = cfg.n_expert_used * (2 * tb(cfg.type_of("ffn_gate"), d * ef) + tb(cfg.type_of("ffn_down"), d * ef))
        return router + experts

    for name in ("tiny_mixtral", "tiny_moe"):
        cfg = synth.TINY[name]
        dense = __import__("dataclasses").replace(cfg, n_expert=0, n_expert_used=0, expert_ffn=0, moe_layers=None,
                                                   shared_ffn=0)
        moe_part = sum(layer_bytes(cfg, i) for i in range(cfg.n_layers) if cfg.is_moe_layer(i))
        dense_ffn = sum(2 * synth.type_bytes(dense.type_of("ffn_gate"), cfg.dim * cfg.ffn)
                        + synth.type_bytes(dense.type_of("ffn_down"), cfg.dim * cfg.ffn)
                        for i in range(cfg.n_layers) if cfg.is_moe_layer(i))
        shared = sum(2 * synth.type_bytes(cfg.type_of("ffn_gate"), cfg.dim * cfg.shared_ffn)
                     + synth.type_bytes(cfg.type_of("ffn_down"), cfg.dim * cfg.shared_ffn)
                     for i in range(cfg.n_layers) if cfg.is_moe_layer(i))
        assert bench.decode_bytes(cfg, 100) == bench.decode_bytes(dense, 100) - dense_ffn + moe_part + shared
    # prefill FLOPs: per token 2 * 3 * dim * expert_ffn per chosen expert (+ router, shared)
    w = synth.WORKLOADS["mixtral8x7b_l4_q4km"]
    dense = __import__("dataclasses").replace(w, n_expert=0, n_expert_used=0, expert_ffn=0)
    moe_minus_dense = 2.0 * 512 * w.n_layers * (3 * w.dim * w.expert_ffn * (w.n_expert_used - 1) + w.dim * w.n_expert)
    assert bench.prefill_flops(w, 512) == bench.prefill_flops(dense, 512) + moe_minus_dense
    assert bench.decode_bytes(synth.CONFIGS["c5_llama8b_q4km"], 8704.5) == 6017837312
