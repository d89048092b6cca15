"""Seeded inputs of the readout-scorer fixtures (tests/golden/readout.pt), regenerated identically by make_golden.py
(for the reference's ops) and by the tests (for the CUDA kernels and the oracle). Strided views where the reference
accepts them."""
import torch

HD = 64


def _windowed(h, rows, cols, row_pos, col_pos, window, g, causal_strict=False):
    """Probabilities-like [h, rows, cols]: positive inside the window (row_pos - col_pos in [0 or 1, window]), 0
    outside."""
    lag = row_pos[:, None] - col_pos[None, :]
    inside = ((lag > 0) if causal_strict else (lag >= 0)) & (lag <= window)
    return torch.rand(h, rows, cols, generator=g) * 0.1 * inside


def future_inputs(h=2, t=192, p=3, m=40, source_start=48, window=64, seed=17):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(t, h, HD, generator=g).permute(1, 0, 2)           # a (t, h, d) buffer seen as [h, t, d]
    target = torch.randn(h, t, HD, generator=g) / 8
    dk = torch.randn(h, p, m, HD, generator=g) * 0.05
    dv = torch.randn(h, p, m, HD, generator=g) * 0.05
    a = torch.rand(h, m, t, generator=g).transpose(1, 2) * 0.1       # [h, t, m] view of an (h, m, t) buffer
    contrast = torch.randn(h, t, m, generator=g)
    return dict(q=q, target=target, dk=dk, dv=dv, a=a, contrast=contrast, source_start=source_start, window=window)


def key_inputs(h=2, t=160, p=3, m=40, source_start=32, query_start=24, window=64, seed=19):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(h, t, HD, generator=g)
    dk = torch.randn(h, p, m, HD, generator=g) * 0.05
    A = _windowed(h, t, m, query_start + torch.arange(t), source_start + torch.arange(m), window, g)
    C = torch.randn(h, t, m, generator=g)
    return dict(q=q, dk=dk, A=A, C=C, source_start=source_start, query_start=query_start, window=window)


def query_inputs(m=5, p=40, h=2, t=200, window=96, seed=23):
    g = torch.Generator().manual_seed(seed)
    dq = torch.randn(m, p, h, HD, generator=g) * 0.3
    keys = torch.randn(h, t, HD, generator=g)
    values = torch.randn(t, h, HD, generator=g).permute(1, 0, 2)
    pos = torch.tensor([17, 63, 120, 150, 199])[:m]
    prob = _windowed(h, m, t, pos, torch.arange(t), window, g)
    prob = prob / prob.sum(-1, keepdim=True).clamp_min(1e-6)
    base = torch.randn(h, m, HD, generator=g)
    return dict(dq=dq, keys=keys, values=values, probabilities=prob, base=base)


def routed_inputs(m=4, p=40, h=2, k=40, seed=29):
    g = torch.Generator().manual_seed(seed)
    dq = (torch.randn(m, p, h, HD, generator=g) * 0.3).bfloat16()
    keys = torch.randn(m, h, k, HD, generator=g).bfloat16()
    values = torch.randn(m, h, k, HD, generator=g).bfloat16()
    prob = torch.rand(m, h, k, generator=g)
    prob = prob / prob.sum(-1, keepdim=True) * 0.7  # the routed keys hold 70% of the mass
    rest = torch.randn(m, h, HD, generator=g) * 0.1
    return dict(dq=dq, keys=keys, values=values, probabilities=prob, rest=rest)
