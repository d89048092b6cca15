"""Seeded inputs of the identity-phase GEMM fixture (tests/golden/id_kernels.pt), regenerated identically by
make_golden.py (for the reference's Triton kernels) and by the tests (for the CUDA kernel and the oracle)."""
import torch


def hidden_inputs(layers=8, m=128, n=256, k=128, seed=21):
    """us: eight bf16 (m, n) pre-activations (separate tensors, as the cache's c_fc outputs), steps fp32 (L, m) (some
    steps larger than |u|, so both relu branches and the kink are exercised), credb bf16 (L, m, k), w_out_t bf16
    (L, k, n)."""
    g = torch.Generator().manual_seed(seed)
    us = [torch.randn(m, n, generator=g).bfloat16() for _ in range(layers)]
    steps = torch.rand(layers, m, generator=g) * 0.5 + 0.01
    credb = (torch.randn(layers, m, k, generator=g) * 0.1).bfloat16()
    w_out_t = (torch.randn(layers, k, n, generator=g) * 0.05).bfloat16()
    return us, steps, credb, w_out_t


def at_b_inputs(k=128, p=128, q=256, seed=22):
    """Eight (k, p) and eight (k, q) bf16 matrices, the first of each a 3-D (2, k / 2, .) view (any leading shape)."""
    g = torch.Generator().manual_seed(seed)
    As = [torch.randn(k, p, generator=g).bfloat16() for _ in range(8)]
    Bs = [(torch.randn(k, q, generator=g) * 0.3).bfloat16() for _ in range(8)]
    As[0] = As[0].view(2, k // 2, p)
    Bs[0] = Bs[0].view(2, k // 2, q)
    return As, Bs


def square_inputs(world=2, layers=8, m=64, seed=23):
    """n1s: eight bf16 (m, world * 64) matrices; got2 bf16 (world, layers, 3, m, 64)."""
    g = torch.Generator().manual_seed(seed)
    d = world * 64
    n1s = [torch.randn(m, d, generator=g).bfloat16() for _ in range(layers)]
    got2 = (torch.randn(world, layers, 3, m, 64, generator=g) * 0.2).bfloat16()
    return n1s, got2
