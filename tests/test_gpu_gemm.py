"""tptc_gemm_f16 (tcgen05 tensor-core GEMM of the prefill path) against torch fp32.

C = A . B^T with fp16 A [M x K] and B [N x K]: every fp16 product is exact in f32, so the only
difference from torch's fp32 matmul is the summation order (tolerance written below).
"""
import pytest

torch = pytest.importorskip("torch")

from tpt_spark_b200 import kernels as K  # noqa: E402
from tpt_spark_b200._lib import EngineError  # noqa: E402

pytestmark = pytest.mark.gpu

SHAPES = [
    # M, N, K
    (128, 128, 64),      # one tile, one k-step
    (128, 128, 4096),    # one tile, the full ring several times over
    (300, 384, 1024),    # ragged M (zero-filled rows), three column tiles
    (77, 200, 256),      # ragged M and N
    (1, 128, 512),       # a single token
    (1024, 6144, 4096),  # the C5 q|k|v shape for a 1024-token chunk
    (64, 130, 64),       # leading dimension not a multiple of 4 (scalar epilogue)
    (4096, 4096, 512),   # 512 tiles: several per persistent CTA, both accumulators cycling
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "m%d_n%d_k%d" % s)
def test_gemm_f16_matches_torch(cuda_device, shape):
    M, N, Kd = shape
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N * 3 + Kd)
    a = torch.randn(M, Kd, generator=g).half().to(cuda_device)
    b = (torch.randn(N, Kd, generator=g) * 0.05).half().to(cuda_device)
    c = torch.full((M, N), float("nan"), device=cuda_device)
    K.gemm_f16(a, b, c, M, N, Kd)
    torch.cuda.synchronize()
    want = a.float() @ b.float().T
    # f32 accumulation of exact products: relative error ~ K * 2^-24
    torch.testing.assert_close(c, want, rtol=1e-4, atol=1e-4 * (Kd ** 0.5))


def test_gemm_f16_rejects_bad_shapes(cuda_device):
    a = torch.zeros(128, 100, dtype=torch.half, device=cuda_device)
    c = torch.zeros(128, 128, device=cuda_device)
    with pytest.raises(EngineError, match="multiple of 64"):
        K.gemm_f16(a, a, c, 128, 128, 100)
