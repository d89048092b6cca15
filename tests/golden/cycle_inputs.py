"""Seeded inputs of the readout-cycle fixture (tests/golden/cycle.pt), regenerated identically by make_golden.py (for
the reference's functions) and by the tests."""
import torch

D, VOCAB = 512, 4096


def hadamard(d=D):
    h = torch.ones(1, 1)
    while h.shape[0] < d:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h


def cycle_inputs(n=96, seed=37, step=7):
    g = torch.Generator().manual_seed(seed)
    return dict(x=torch.randn(n, D, generator=g), lm_head=torch.randn(D, VOCAB, generator=g) * 0.05,
                y=torch.randint(0, VOCAB, (n,), generator=g), step_t=torch.tensor(step),
                raw=torch.randn(n, VOCAB, generator=g) * 3, H=hadamard())
