"""The seed-rebuilt update and AdamW on the GPU against the CPU oracle, the reference's golden step and torch.

Tolerance of the rebuilt update: relative to the largest |G| of each parameter, 4e-3. The GEMM reads its fp32
operands as tf32, as the reference's fp32 matmul does at torch.set_float32_matmul_precision('high') (eggroll.py:184):
each product carries a relative error below 2^-9 and the sum over pairs about 2^-9 sqrt(pairs) of the term scale,
against a largest |G| of a few sqrt(pairs) term scales."""
import math

import pytest
import torch

from oracle import eggroll as oe, gpt

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None
GTOL = 4e-3


def _rel(a, r):
    return ((a.double().cpu() - r.double().cpu()).abs().max() / r.double().abs().max().clamp(min=1e-30)).item()


def _rebuild_gpu(buf, offs, weight, count, shard=None):
    from noise_b200 import train
    from noise_b200.population import PARAMS
    shapes = [s for _, s in PARAMS]
    fp = train.FlatParams({n: torch.zeros(s) for n, s in PARAMS}, DEV)
    grad = torch.zeros_like(fp.flat)
    table = torch.stack([offs[n] for n, _ in PARAMS]).to(DEV)
    pairs = weight.shape[0]
    st, _ = train.rebuild_update(buf.to(DEV), table, weight.to(DEV), count, shard or (0, pairs), grad, fp)
    torch.cuda.synchronize()
    assert int(st[0]) == 0
    return {n: grad[o:o + math.prod(s)].view(s).cpu() for (n, s), o in zip(PARAMS, fp.offsets)}


def test_rebuild_matches_oracle():
    pairs, n_noise = 200, 2 ** 20
    shapes = gpt.param_shapes()
    buf = oe.make_buffer(n_noise, seed=0)
    offs = oe.offsets(shapes, pairs, step=2, n_noise=n_noise)
    weight = torch.randn(pairs, generator=torch.Generator().manual_seed(3))
    ref = oe.rebuild_update(buf, offs, weight, 2 * pairs, shapes)
    got = _rebuild_gpu(buf, offs, weight, 2 * pairs)
    for name, _ in shapes:
        assert _rel(got[name], ref[name]) < GTOL, name


def test_sharded_rebuild_sums_to_full():
    from noise_b200.train import pair_shard
    pairs, n_noise = 130, 2 ** 20
    shapes = gpt.param_shapes()
    buf = oe.make_buffer(n_noise, seed=0)
    offs = oe.offsets(shapes, pairs, step=5, n_noise=n_noise)
    weight = torch.randn(pairs, generator=torch.Generator().manual_seed(4))
    full = _rebuild_gpu(buf, offs, weight, 2 * pairs)
    parts = [_rebuild_gpu(buf, offs, weight, 2 * pairs, pair_shard(pairs, r, 3)) for r in range(3)]
    for name, _ in shapes:
        total = parts[0][name] + parts[1][name] + parts[2][name]
        assert _rel(total, full[name]) < GTOL, name


def test_rebuild_matches_reference_step(golden):
    """The reference's own gradients of one Eggroll.step (tests/golden/eggroll_step.pt): losses from the oracle
    (pinned to the reference), fitness weights, then the rebuild on the GPU."""
    g = golden('eggroll_step.pt')
    pairs, rows, n = g['pairs'], g['rows'], g['noise_size']
    shapes = gpt.param_shapes()
    members, per_seq, _, directions, positive, row = oe.member_layout(pairs, rows)
    buf = oe.make_buffer(n, seed=0)
    offs = oe.offsets(shapes, pairs, step=g['step'], n_noise=n)
    w = gpt.init_weights(0, eggroll=True)
    tokens = g['tokens'].long()
    losses = []
    for start in range(0, members, 2 * g['chunk']):
        sel = torch.arange(start, start + 2 * g['chunk'])
        nz = oe.noise(buf, offs, directions[sel], shapes)
        sign = torch.where(positive[sel], oe.SIGMA, -oe.SIGMA)
        r = int(row[start])
        losses.append(oe.population_loss(w, nz, sign, tokens[r, :-1], tokens[r, 1:]))
    weight, count = oe.fitness_weights(torch.cat(losses), pairs)
    got = _rebuild_gpu(buf, offs, weight, count)
    for name, ref in g['grad_small'].items():
        assert _rel(got[name], ref) < GTOL, name
    for name, ref in g['grad_corner'].items():
        scale = abs(g['grad_abs'][name]) / math.prod(got[name].shape)  # mean |G| of the whole tensor
        assert (got[name][:8, :8] - ref).abs().max().item() < 5 * GTOL * max(scale, ref.abs().max().item()), name


def test_adam_matches_torch():
    from noise_b200.train import AdamW
    gen = torch.Generator(device='cuda').manual_seed(0)
    p0 = torch.randn(10_000, device='cuda', generator=gen)
    ours, ref = p0.clone(), p0.clone().requires_grad_(True)
    opt_ref = torch.optim.AdamW([ref], lr=1e-3, betas=(0.5, 0.95), eps=1e-8, weight_decay=0.0)
    opt = AdamW(ours, lr=1e-3, betas=(0.5, 0.95), eps=1e-8)
    for k in range(5):
        grad = torch.randn(10_000, device='cuda', generator=gen) * (k + 1)
        ref.grad = grad.clone()
        opt_ref.step()
        opt.step(grad)
    torch.testing.assert_close(ours, ref.detach(), rtol=1e-5, atol=1e-6)


def test_trainer_step_moves_weights_like_the_oracle(monkeypatch):
    """One full update (forward, fitness, rebuild, AdamW) against the oracle's (bf16-autocast CPU forward): the sign
    of every weight change agrees for almost all entries (Adam's first step is ~ -lr sign(g)). Offsets come from the
    CPU generator on both sides (CPU and CUDA generators draw different numbers)."""
    from noise_b200 import train
    from noise_b200.train import EggrollTrainer
    cpu_offsets = train.step_offsets
    monkeypatch.setattr(train, 'step_offsets',
                        lambda pairs, step, device, seed=0, size=oe.NOISE: cpu_offsets(pairs, step, 'cpu', seed,
                                                                                       size).to(device))
    pairs, rows, length, n_noise, lr = 8, 2, 256, 2 ** 20, 1e-3
    w = gpt.informative_weights(0)
    buf = oe.make_buffer(n_noise, seed=0)
    tokens = gpt.zipf_tokens(rows, length + 1, seed=9)
    tr = EggrollTrainer({k: v.to(DEV) for k, v in w.items()}, pairs, rows, sigma=oe.SIGMA, lr=lr, buffer=buf.to(DEV),
                        noise_size=n_noise)
    tr.step(tokens.to(DEV), step=1)
    torch.cuda.synchronize()
    shapes = gpt.param_shapes()
    members, per_seq, _, directions, positive, row = oe.member_layout(pairs, rows)
    offs = oe.offsets(shapes, pairs, step=1, n_noise=n_noise, device='cpu')
    losses = []
    for start in range(0, members, per_seq):
        sel = torch.arange(start, start + per_seq)
        nz = oe.noise(buf, offs, directions[sel], shapes)
        sign = torch.where(positive[sel], oe.SIGMA, -oe.SIGMA)
        losses.append(oe.population_loss(w, nz, sign, tokens[int(row[start]), :-1], tokens[int(row[start]), 1:],
                                         autocast=True))
    weight, count = oe.fitness_weights(torch.cat(losses), pairs)
    grads = oe.rebuild_update(buf, offs, weight, count, shapes)
    agree = total = 0
    for name, _ in shapes:
        delta = tr.params[name].cpu() - w[name]
        g = grads[name]
        mask = g.abs() > 1e-3 * g.abs().max()
        agree += ((delta < 0) == (g > 0))[mask].sum().item()
        total += mask.sum().item()
    assert agree / total > 0.97, agree / total
