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
