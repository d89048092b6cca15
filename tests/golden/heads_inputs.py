"""Seeded inputs of the head-sharding fixtures (tests/golden/heads.pt), regenerated identically by make_golden.py
(for the reference's kernels) and by the tests (for the CUDA kernels and the oracle)."""
import math

import torch

H, HD, PACK = 8, 64, 5 * 64 + 2


def rotary(t):
    """fp32 cos / sin [t, 32] of RoPE base 10000 over head_dim 64 (the identity phase's rope32)."""
    inv_freq = 1.0 / 10000 ** (torch.arange(0, HD, 2, dtype=torch.float32) / HD)
    freqs = torch.outer(torch.arange(t, dtype=torch.float32), inv_freq)
    return freqs.cos(), freqs.sin()


def pack_inputs(layers=2, n=64, t=32, seed=11):
    """Per layer: q, k, v, o, target bf16 (n, 512) views (some strided, as slices of wider rows) and lse fp32
    (n / t, 8, t)."""
    g = torch.Generator().manual_seed(seed)
    out = {name: [] for name in ('qs', 'ks', 'vals', 'outs', 'targets', 'lses')}
    for _ in range(layers):
        for j, name in enumerate(('qs', 'ks', 'vals', 'outs', 'targets')):
            width = (H * HD) + (128 if j % 2 == 0 else 0)  # q, v, target: strided views of wider rows
            z = torch.randn(n, width, generator=g).bfloat16()
            out[name].append(z[:, :H * HD] if width > H * HD else z)
        out['lses'].append(torch.randn(n // t, H, t, generator=g) + 3)
    return out


def got_inputs(world=8, layers=2, n=64, t=64, seed=13):
    """The received buffer got (W, L, N, PACK) bf16: N(0, 1) pieces and the fp32 bits of an lse ~ N(3, 1) in the
    last two elements; b = W N / t rows per layer (N a multiple of t, as in the identity phase: every rank sends whole
    rows)."""
    g = torch.Generator().manual_seed(seed)
    got = torch.randn(world, layers, n, PACK, generator=g).bfloat16()
    lse = torch.randn(world, layers, n, generator=g) + 3
    got.view(torch.int16)[..., 5 * HD:] = lse.unsqueeze(-1).view(torch.int16).view(world, layers, n, 2)
    b = world * n // t
    assert b * t == world * n and math.gcd(n, 32) == 32
    return got, b
