"""tptc_attn_decode_noalloc (static device scratch, no allocation) against tptc_attn_decode.

Collected last on purpose: it must pass alone and after every other test in the process,
whatever state the other entry points left behind.  Each case runs the no-alloc entry point
twice in a row and compares both results bit for bit with the workspace entry point's result
on the same inputs (same kernel, same split count, so the same arithmetic).  A flagged launch
(a position outside the cache) is reported by tptc_attn_decode_noalloc_status and leaves
nothing behind that changes the next call's result.
"""
import pytest

torch = pytest.importorskip("torch")

from tpt_spark_b200 import kernels as K  # noqa: E402
from tpt_spark_b200._lib import EngineError  # noqa: E402

pytestmark = pytest.mark.gpu


def rope_tables(max_seq, hd, base=500000.0):
    j = torch.arange(0, hd, 2, dtype=torch.float32)
    theta = 1.0 / torch.pow(torch.tensor(base, dtype=torch.float32), j / hd)
    ang = torch.arange(max_seq, dtype=torch.float32)[:, None] * theta[None, :]
    return torch.cos(ang).contiguous(), torch.sin(ang).contiguous()


CASES = [
    # n_heads, n_kv, hd, max_seq, pos, kv_type
    (32, 8, 128, 9216, 8500, K.F16),  # Llama-3-8B shape near the end of its cache
    (32, 8, 128, 9216, 0, K.F16),
    (8, 1, 128, 512, 300, K.F32),     # MQA: 64 splits
    (24, 8, 96, 700, 63, K.F32),
]


def inputs(case, dev):
    n_heads, n_kv, hd, max_seq, pos, kv_type = case
    g = torch.Generator(device="cpu").manual_seed(99 + pos)
    kv_dtype = torch.float32 if kv_type == K.F32 else torch.float16
    q = torch.randn(n_heads * hd, generator=g).to(dev)
    kraw = torch.randn(n_kv * hd, generator=g).to(dev)
    kc = torch.randn(n_kv, max_seq, hd, generator=g).to(kv_dtype).to(dev)
    vc = torch.randn(n_kv, max_seq, hd, generator=g).to(kv_dtype).to(dev)
    cs, sn = (t.to(dev) for t in rope_tables(max_seq, hd))
    return q, kraw, kc, vc, cs, sn


def workspace_result(case, q, kraw, kc, vc, cs, sn, dev):
    n_heads, n_kv, hd, max_seq, pos, kv_type = case
    d_pos = torch.tensor([pos], dtype=torch.int32, device=dev)
    nbytes = K.attn_decode_workspace_bytes(n_heads, n_kv, hd, max_seq)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    want = torch.full((n_heads * hd,), float("nan"), device=dev)
    K.attn_decode(q, kraw, kc, vc, kv_type, cs, sn, d_pos, n_heads, n_kv, hd, max_seq, want, ws, nbytes)
    torch.cuda.synchronize()
    assert torch.isfinite(want).all()
    return want


@pytest.mark.parametrize("case", CASES, ids=lambda c: "h%d_kv%d_d%d_s%d_p%d_t%d" % c)
def test_noalloc_matches_workspace_entry(cuda_device, case):
    n_heads, n_kv, hd, max_seq, pos, kv_type = case
    dev = cuda_device
    q, kraw, kc, vc, cs, sn = inputs(case, dev)
    want = workspace_result(case, q, kraw, kc, vc, cs, sn, dev)
    d_pos = torch.tensor([pos], dtype=torch.int32, device=dev)
    for call in range(2):
        out = torch.full((n_heads * hd,), float("nan"), device=dev)
        K.attn_decode_noalloc(q, kraw, kc, vc, kv_type, cs, sn, d_pos, n_heads, n_kv, hd, max_seq, out)
        torch.cuda.synchronize()
        assert torch.equal(out, want), "call %d differs from tptc_attn_decode" % call
        assert K.attn_decode_noalloc_status() == 0


def test_noalloc_flagged_call_is_reported_and_leaves_no_trace(cuda_device):
    """A position outside the cache: the kernel writes nothing and flags TPTC_ERR_ARG, which
    the status query reports (once); the calls after it -- with or without a status query in
    between -- are again bit-identical to the workspace entry point."""
    case = (32, 8, 128, 9216, 4097, K.F16)
    n_heads, n_kv, hd, max_seq, pos, kv_type = case
    dev = cuda_device
    q, kraw, kc, vc, cs, sn = inputs(case, dev)
    kc_before = kc.clone()
    bad_pos = torch.tensor([max_seq], dtype=torch.int32, device=dev)
    good_pos = torch.tensor([pos], dtype=torch.int32, device=dev)
    out = torch.full((n_heads * hd,), float("nan"), device=dev)
    K.attn_decode_noalloc(q, kraw, kc, vc, kv_type, cs, sn, bad_pos, n_heads, n_kv, hd, max_seq, out)
    assert K.attn_decode_noalloc_status() == -1  # TPTC_ERR_ARG
    assert K.attn_decode_noalloc_status() == 0   # reported once; the array was re-zeroed
    assert torch.isnan(out).all() and torch.equal(kc, kc_before)
    want = workspace_result(case, q, kraw, kc.clone(), vc, cs, sn, dev)
    for query_between in (True, False):
        K.attn_decode_noalloc(q, kraw, kc, vc, kv_type, cs, sn, bad_pos, n_heads, n_kv, hd, max_seq, out)
        if query_between:
            assert K.attn_decode_noalloc_status() == -1
        kcx = kc_before.clone()
        got = torch.full((n_heads * hd,), float("nan"), device=dev)
        K.attn_decode_noalloc(q, kraw, kcx, vc, kv_type, cs, sn, good_pos, n_heads, n_kv, hd, max_seq, got)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        assert K.attn_decode_noalloc_status() == 0  # each call starts from a zeroed error word


def test_noalloc_rejects_sizes_beyond_static_scratch(cuda_device):
    # 256 kv heads x 8 query heads x hd 128 needs one split of 2048 * 130 * 4 B > 1 MiB
    n_heads, n_kv, hd, max_seq = 2048, 256, 128, 64
    t = torch.zeros(16, device=cuda_device)
    d_pos = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    with pytest.raises(EngineError, match="static maximum of 1048576 bytes"):
        K.attn_decode_noalloc(t, t, t, t, K.F16, t, t, d_pos, n_heads, n_kv, hd, max_seq, t)
