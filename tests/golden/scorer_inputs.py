"""Seeded inputs of the readout-scorer fixtures (tests/golden/scorer.pt), regenerated identically by make_golden.py
(for the reference's kernels) and by the tests: one chunk of m tokens starting at global token `start` of a T-token
sequence, n moved rows per token (of d_rows), block tables for every token."""
import torch

H, D, W = 8, 64, 512


def rope(T):
    inv = 1.0 / 10000 ** (torch.arange(0, D, 2, dtype=torch.float32) / D)
    f = torch.outer(torch.arange(T, dtype=torch.float32), inv)
    return f.cos().contiguous(), f.sin().contiguous()


def scorer_inputs(T=40, start=8, m=6, n=70, d_rows=80, seed=31):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s, scale=1.0: torch.randn(*s, generator=g) * scale
    nc = 2 * W + 16
    x = {}
    x['delta'] = r(m, d_rows, W, scale=0.05)
    x['X'] = r(T, W)
    x['SQX'] = x['X'].square().sum(-1)
    x['UP'] = r(m * n, nc, scale=0.05).bfloat16()
    x['R0'], x['VC'], x['GZ'], x['VE'] = r(T, H, D), r(T, W), r(T, H), r(T, H, D, scale=0.1)
    x['CS'], x['SN'] = rope(T)
    x['U'], x['W'] = r(T, H, D, scale=0.1), r(T, H, D, scale=0.1)
    x['M1'], x['M2'] = r(T, H, D, D, scale=0.05).bfloat16(), r(T, H, D, D, scale=0.05).bfloat16()
    x['QD'], x['GD'] = r(T, H, D), r(T, H, D, scale=0.1)
    x['AD'] = torch.rand(T, H, generator=g) * 0.2
    x['CD'] = r(T, H)
    x['VT'], x['OT'] = r(T, H, D), r(T, H, D)
    x['PJ'] = r(m, n, 2, H, D, scale=0.05)
    x['GC'] = r(m, n, H, scale=0.1)
    x.update(T=T, start=start, m=m, n=n, d_rows=d_rows, nc=nc, eps=1.1920928955078125e-07)
    return x


def tables(x):
    return tuple(x[k] for k in ('U', 'W', 'M1', 'M2', 'QD', 'GD', 'AD', 'CD', 'VT', 'OT'))
