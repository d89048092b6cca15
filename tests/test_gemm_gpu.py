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


@pytest.mark.parametrize('m,n,k', [(130, 544, 72), (1, 32, 8), (300, 96, 1000)])
def test_gemm_bf16_partial_tiles(m, n, k):
    """M, N and K tails: the last tiles read zeros past the operands and store only inside D."""
    from noise_b200 import _lib
    g = torch.Generator(device='cuda').manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, device='cuda', generator=g).bfloat16()
    b = torch.randn(n, k, device='cuda', generator=g).bfloat16()
    out = torch.full((m, n), float('nan'), device='cuda')
    got = _lib.gemm_bf16_tn(a, b, out)
    torch.cuda.synchronize()
    assert _lib.read_status(got._noise_workspace) == 0
    ref = a.double() @ b.double().t()
    assert (got.double() - ref).abs().max().item() <= 1e-5 * k ** 0.5 * 4


@pytest.mark.parametrize('m,n,k', [(128, 256, 32), (512, 4096, 512), (4096, 512, 4096), (200, 96, 60),
                                   (512, 2048, 12288)])
def test_gemm_tf32_matches_fp64(m, n, k):
    """The kind::tf32 GEMM against fp64 on the same fp32 operands: the tensor core reads 10 of the 23 mantissa bits of
    each operand, so products carry a relative error below 2^-9 and the sum about 2^-9 sqrt(k) of the term scale
    (bound 4x that); and against the fp64 product of the operands rounded to tf32, far tighter."""
    from noise_b200 import _lib
    g = torch.Generator(device='cuda').manual_seed(m + 3 * n + k)
    a = torch.randn(m, k, device='cuda', generator=g)
    b = torch.randn(n, k, device='cuda', generator=g)
    got = _lib.gemm_tf32_tn(a, b)
    torch.cuda.synchronize()
    assert _lib.read_status(got._noise_workspace) == 0
    ref = a.double() @ b.double().t()
    err = (got.double() - ref).abs().max().item()
    assert err <= 4 * 2 ** -9 * k ** 0.5, err
    assert err > 0  # tf32, not fp32: the low mantissa bits are not read
