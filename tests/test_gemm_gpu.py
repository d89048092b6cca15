"""The tcgen05/TMA GEMM core against a torch fp32 matmul of the same bf16 operands (fp32 accumulation, so the only
difference is summation order: rtol 1e-5 relative to the row scale)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('m,n,k', [(128, 256, 64), (256, 512, 512), (384, 1536, 512), (1024, 512, 2048),
                                   (128 * 149, 256, 128)])
def test_gemm_matches_torch(m, n, k):
    from noise_b200 import _lib
    g = torch.Generator(device='cuda').manual_seed(m + n + k)
    a = torch.randn(m, k, device='cuda', generator=g).bfloat16()
    b = torch.randn(n, k, device='cuda', generator=g).bfloat16()
    got = _lib.gemm_bf16_tn(a, b)
    torch.cuda.synchronize()
    assert _lib.read_status(got._noise_workspace) == 0
    ref = a.double() @ b.double().t()
    err = (got.double() - ref).abs().max().item()
    assert err <= 1e-5 * k ** 0.5 * 4, err
