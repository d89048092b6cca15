"""Seeded inputs of the Dust block-rerun fixture (tests/golden/dust.pt), regenerated identically by make_golden.py and
the tests: one value-embedding block and one plain block, 2 sequences x 256 tokens, informative weights, jitter at
every site."""
import torch

C, HD = 512, 64


def rotary(t):
    inv = 1.0 / 10000 ** (torch.arange(0, HD, 2, dtype=torch.float32) / HD)
    f = torch.outer(torch.arange(t, dtype=torch.float32), inv)
    return f.cos(), f.sin()


def dust_inputs(B=2, T=256, seed=41, sigma=0.05):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s, scale=1.0: torch.randn(*s, generator=g) * scale
    u = lambda *s: (torch.rand(*s, generator=g) * 2 - 1) * 3 ** 0.5 / C ** 0.5
    w = dict(q=u(C, C), k=u(C, C), v=u(C, C), gate=r(8, 32, scale=0.3), proj=u(C, C) * 1.5, fc=u(4 * C, C),
             out=u(C, 4 * C) * 0.75)
    plain = {k: v for k, v in w.items() if k != 'gate'}
    jitter = dict(o=r(B, T, C, scale=sigma), attn=r(B, T, C, scale=sigma), fc=r(B, T, 4 * C, scale=sigma),
                  mlp=r(B, T, C, scale=sigma))
    cos, sin = rotary(T)
    return dict(x=r(B, T, C), ve=r(B, T, C, scale=0.5), w=w, plain=plain, jitter=jitter, cos=cos, sin=sin,
                windows=(128, 256))


def head_error_inputs(b=2, t=128, draws=64, nrep=16, seed=43):
    """Cached LM-head logits (bf16 [b, t, 4096]), targets (two ignored), clean losses, and the draws' generator
    (bf16 N(0, 1) in the reference's call order)."""
    g = torch.Generator().manual_seed(seed)
    raw = (torch.randn(b, t, 4096, generator=g) * 3).bfloat16()
    y = torch.randint(0, 4096, (b, t), generator=g)
    y[0, 5] = y[1, 17] = -1
    clean = torch.randn(b, t, generator=g).abs() + 8
    draw_gen = torch.Generator().manual_seed(seed + 1)
    noise = lambda *shape: torch.randn(*shape, generator=draw_gen).bfloat16()
    return dict(raw=raw, y=y, clean_loss=clean, draws=draws, nrep=nrep, noise=noise, sigma=0.1)
