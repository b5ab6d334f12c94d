"""Kernel parity through the C ABI on a B200: dequantisation and activation quantisation
bit-exact against the oracle / gguf-py fixtures, per-block integer dots bit-exact, GEMV
outputs within 1e-3 relative (north_star level 2)."""
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "blocks.npz"))
REL_TOL = 1e-3  # fp32 GEMV outputs vs the oracle, relative to the output scale


def dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("name,t", [("q4k", O.Q4_K), ("q6k", O.Q6_K), ("q80", O.Q8_0), ("f16", O.F16),
                                    ("q40", O.Q4_0), ("q41", O.Q4_1), ("q50", O.Q5_0), ("q51", O.Q5_1),
                                    ("q2k", O.Q2_K), ("q3k", O.Q3_K), ("q5k", O.Q5_K)])
def test_dequant_bitexact_vs_gguf_py(cuda_device, name, t):
    import torch

    from tpt_spark_b200 import kernels as K

    ref = GOLD[f"{name}_f32"]
    raw = dev(GOLD[f"{name}_raw"])
    out = torch.empty(ref.size, dtype=torch.float32, device="cuda")
    K.dequant(t, raw, ref.size, out)
    np.testing.assert_array_equal(host(out).view(np.uint32), ref.view(np.uint32))


def activations(k, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(k).astype(np.float32) * rng.choice([1e-3, 1.0, 30.0], k).astype(np.float32)
    if k >= 1024:
        x[:256] = 0.0                   # all-zero block
        x[256:512] = 0.75               # constant block
        x[512:768] = np.float32(-1.0)   # negative constant (max is negative)
        x[800] = 1e4                    # isolated extreme
    return x


@pytest.mark.parametrize("k", [256 * 4, 4096, 14336])
def test_quant_q8k_bitexact(cuda_device, k):
    import torch

    from tpt_spark_b200 import kernels as K

    x = activations(k, k)
    ref = O.quant_q8k(x)
    out = torch.zeros(ref.nbytes, dtype=torch.uint8, device="cuda")
    K.quant_q8k(dev(x), k, out)
    np.testing.assert_array_equal(host(out), ref.view(np.uint8))


def test_quant_q80_bitexact(cuda_device):
    import torch

    from tpt_spark_b200 import kernels as K

    x = GOLD["q80_x"]
    out = torch.zeros(x.size // 32 * 34, dtype=torch.uint8, device="cuda")
    K.quant_q80(dev(x), x.size, out)
    np.testing.assert_array_equal(host(out), GOLD["q80_q"])
    y = activations(4096, 1)
    out = torch.zeros(4096 // 32 * 34, dtype=torch.uint8, device="cuda")
    K.quant_q80(dev(y), 4096, out)
    np.testing.assert_array_equal(host(out), O.quant_q80(y))


SHAPES = [(O.Q4_K, 40, 4096), (O.Q4_K, 8, 256), (O.Q4_K, 1024, 4096), (O.Q4_K, 64, 14336),
          (O.Q6_K, 40, 4096), (O.Q6_K, 24, 14336), (O.Q6_K, 17, 2048), (O.Q8_0, 40, 4096), (O.Q8_0, 16, 14336),
          (O.F16, 40, 4096), (O.F16, 8, 3072), (O.Q5_K, 40, 4096), (O.Q5_K, 24, 14336), (O.Q5_K, 9, 2048),
          (O.Q4_0, 40, 4096), (O.Q4_0, 16, 14336), (O.Q5_0, 40, 4096), (O.Q5_0, 17, 2048),
          (O.Q2_K, 40, 4096), (O.Q2_K, 24, 14336), (O.Q3_K, 40, 4096), (O.Q3_K, 17, 2048),
          (O.Q4_1, 40, 4096), (O.Q4_1, 9, 14336), (O.Q5_1, 40, 4096), (O.Q5_1, 17, 2048)]
Q80_FAMILY = (O.Q8_0, O.Q4_0, O.Q5_0, O.Q4_1, O.Q5_1)
BLOCK_BYTES = {O.Q4_K: 144, O.Q5_K: 176, O.Q6_K: 210, O.Q8_0: 34, O.Q4_0: 18, O.Q5_0: 22, O.Q2_K: 84, O.Q3_K: 110,
               O.Q4_1: 20, O.Q5_1: 24}


def make_matrix(t, N, K, seed=0):
    from tpt_spark_b200 import synth
    from tpt_spark_b200.kernels import Matrix

    w = synth.normal(1000 + seed, N * K, 0.02)
    raw = synth.encode(t, w)
    return raw, Matrix(t, raw, N, K)


@pytest.mark.parametrize("t,N,K", [s for s in SHAPES if s[0] != O.F16])
def test_block_dots_bitexact(cuda_device, t, N, K):
    import torch

    raw, m = make_matrix(t, N, K)
    x = activations(K, 7)
    per_row = K // 32 if t in Q80_FAMILY else K // 256
    isum = torch.zeros(N * per_row, dtype=torch.int32, device="cuda")
    msum = torch.zeros(N * per_row, dtype=torch.int32, device="cuda")
    m.block_dots(dev(x), isum, msum)
    gi, gm = host(isum).reshape(N, per_row), host(msum).reshape(N, per_row)
    xq = O.quant_for(t, x)
    bb = BLOCK_BYTES[t]
    rows = raw.reshape(N, per_row * bb)
    for r in range(N):
        ri, rm = O.block_dots(t, rows[r], xq, per_row)
        np.testing.assert_array_equal(gi[r], ri, err_msg=f"row {r} isum")
        if t in (O.Q4_K, O.Q5_K, O.Q2_K):
            np.testing.assert_array_equal(gm[r], rm, err_msg=f"row {r} msum")


@pytest.mark.parametrize("t,N,K", SHAPES)
def test_gemv_vs_oracle(cuda_device, t, N, K):
    import torch

    raw, m = make_matrix(t, N, K, seed=3)
    x = activations(K, 11)
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    m.gemv(dev(x), y)
    got = host(y)
    ref = O.matmul(t, raw, N, K, x)[0]
    scale = np.abs(ref).max()
    np.testing.assert_array_less(np.abs(got - ref), REL_TOL * scale + 1e-30)
    # elementwise relative error for entries away from zero
    big = np.abs(ref) > 0.05 * scale
    assert (np.abs(got - ref)[big] / np.abs(ref[big])).max() < REL_TOL


def test_gemv_f16_vs_torch_fp32(cuda_device):
    import torch

    from tpt_spark_b200 import synth
    from tpt_spark_b200.kernels import Matrix

    N, K = 96, 3072
    w = synth.normal(5, N * K, 0.02).astype(np.float16)
    m = Matrix(O.F16, w.view(np.uint8), N, K)
    x = torch.randn(K, device="cuda")
    y = torch.empty(N, device="cuda")
    m.gemv(x, y)
    ref = torch.from_numpy(w.astype(np.float32)).cuda().reshape(N, K) @ x
    torch.testing.assert_close(y, ref, rtol=1e-4, atol=1e-4)


def test_gemv_repeatable(cuda_device):
    import torch

    raw, m = make_matrix(O.Q4_K, 512, 4096, seed=9)
    x = dev(activations(4096, 2))
    y1 = torch.empty(512, device="cuda")
    y2 = torch.empty(512, device="cuda")
    m.gemv(x, y1)
    m.gemv(x, y2)
    assert torch.equal(y1, y2)


# Every matrix shape of the benchmark configurations C2-C5, out x in:
# q/o, k, v, gate (= up), down and the output projection of each.
CONFIG_MATRICES = {
    "c2": [(O.Q4_K, 2048, 2048), (O.Q4_K, 512, 2048), (O.Q6_K, 512, 2048), (O.Q4_K, 8192, 2048),
           (O.Q6_K, 2048, 8192), (O.Q6_K, 128256, 2048)],
    "c3": [(O.Q8_0, 4096, 4096), (O.Q8_0, 1024, 4096), (O.Q8_0, 14336, 4096), (O.Q8_0, 4096, 14336),
           (O.Q8_0, 32000, 4096)],
    "c4": [(O.F16, 3072, 3072), (O.F16, 8192, 3072), (O.F16, 3072, 8192), (O.F16, 32064, 3072)],
    "c5": [(O.Q4_K, 4096, 4096), (O.Q4_K, 1024, 4096), (O.Q6_K, 1024, 4096), (O.Q4_K, 14336, 4096),
           (O.Q6_K, 4096, 14336), (O.Q6_K, 128256, 4096)],
}
CONFIG_CASES = [(c, t, n, k) for c, ms in CONFIG_MATRICES.items() for (t, n, k) in ms]


@pytest.mark.parametrize("cfg,t,N,K", CONFIG_CASES, ids=lambda v: str(v))
def test_gemv_config_shapes(cuda_device, cfg, t, N, K):
    """y within 1e-3 relative of the oracle for every row, and the per-block integer sums
    bit-exact on up to 2048 rows spread over the matrix (first, last and a stride between)."""
    import torch

    raw, m = make_matrix(t, N, K, seed=N + K)
    try:
        x = activations(K, 31)
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        m.gemv(dev(x), y)
        got = host(y)
        ref = O.matmul(t, raw, N, K, x)[0]
        scale = np.abs(ref).max()
        assert np.abs(got - ref).max() <= REL_TOL * scale
        big = np.abs(ref) > 0.05 * scale
        assert (np.abs(got - ref)[big] / np.abs(ref[big])).max() < REL_TOL
        if t == O.F16:
            return
        per_row = K // 32 if t == O.Q8_0 else K // 256
        isum = torch.zeros(N * per_row, dtype=torch.int32, device="cuda")
        msum = torch.zeros(N * per_row, dtype=torch.int32, device="cuda")
        m.block_dots(dev(x), isum, msum)
        gi, gm = host(isum).reshape(N, per_row), host(msum).reshape(N, per_row)
    finally:
        m.close()
    xq = O.quant_for(t, x)
    bb = {O.Q4_K: 144, O.Q6_K: 210, O.Q8_0: 34}[t]
    rows = raw.reshape(N, per_row * bb)
    for r in sorted(set(range(0, N, max(1, N // 2046))) | {N - 1}):
        ri, rm = O.block_dots(t, rows[r], xq, per_row)
        np.testing.assert_array_equal(gi[r], ri, err_msg=f"row {r} isum")
        if t == O.Q4_K:
            np.testing.assert_array_equal(gm[r], rm, err_msg=f"row {r} msum")


@pytest.mark.parametrize("t,N,K", SHAPES)
def test_matrix_dequant_f16_bitexact(cuda_device, t, N, K):
    """The prefill GEMM's B operand: the device-layout matrix expanded to dense fp16 equals the
    oracle's bit-exact dequantisation rounded to nearest fp16, element for element."""
    import torch

    raw, m = make_matrix(t, N, K, seed=5)
    out = torch.full((N, K), float("nan"), dtype=torch.float16, device="cuda")
    m.dequant_f16(out)
    want = O.dequant(t, raw, N * K).reshape(N, K).astype(np.float16)
    np.testing.assert_array_equal(host(out).view(np.uint16), want.view(np.uint16))
