"""GPU: the tcgen05 (TMEM-accumulator) bf16 GEMM against torch's fp32
matmul of the same bf16 inputs.  Products of bf16 are exact in fp32, so only
the summation order differs."""
import numpy as np
import pytest

from tests.conftest import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 64, 64), (128, 128, 128), (128, 256, 64), (256, 100, 1024),
                                   (384, 300, 512), (128, 16, 2048), (200, 256, 192)])
def test_gemm_bf16_nt_vs_torch(M, N, K, cuda):
    torch = pytest.importorskip("torch")
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    B = torch.randn((N, K), generator=g, device="cuda").to(torch.bfloat16)
    D = torch.full((M, N), float("nan"), device="cuda")
    torch.cuda.synchronize()
    cuda.gemm_bf16_nt(A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, K)
    cuda.check_device_errors()
    ref = A.double() @ B.double().T
    torch.cuda.synchronize()
    assert rel_err(D.cpu().numpy(), ref.cpu().numpy()) <= 1e-5
