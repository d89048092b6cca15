"""Generate the golden fixtures under tests/golden/ by running the reference itself on the CPU.

Runs only where the reference checkout is readable (pass its path as argv[1] or set NOISE_REFERENCE); the GPU box
never runs this script, it only reads the committed ``*.pt`` files. Reference files used:

- ``utils/model.py``: GPT(GPTConfig()), init_weights, forward (config 1 of the benchmark plan).
- ``archive/10M/train/val/eggroll.py``: make_model, lowrank, lowrank_embed, population_loss, Eggroll.offsets/noise
  and one Eggroll.step (member layout, fitness, seed-rebuilt gradient).
- ``train/speedrun/moment_kernels.py``: _implicit_key_context under TRITON_INTERPRET=1 (its dots are fp32 tf32 dots,
  which the interpreter evaluates in fp32).

Compiled flex attention does not lower on the CPU, so ``utils.model.flex`` is switched to the eager
``flex_attention`` (same function, no compilation). The noise buffer is shrunk from 2**28 to 2**20 values
(``eggroll.NOISE``) and the chunk from 256 to 2 pairs (``eggroll.CHUNK``) so one step finishes in seconds.

Usage: python tests/golden/make_golden.py /path/to/reference
"""
import importlib.util
import os
import sys
from pathlib import Path

os.environ.setdefault('TRITON_INTERPRET', '1')  # read when triton is first imported; only the credit fixture uses it
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
SMALL_NOISE = 2 ** 20


def load_reference(root):
    sys.path.insert(0, str(root))
    import utils.model as model
    from torch.nn.attention.flex_attention import flex_attention
    model.flex = flex_attention
    spec = importlib.util.spec_from_file_location('ref_eggroll', root / 'archive/10M/train/val/eggroll.py')
    eggroll = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(eggroll)
    return model, eggroll


def checksums(sd):
    """Per tensor: (sum, sum |x|, first 8 values) — enough to pin an init draw for draw."""
    return {k: (float(v.double().sum()), float(v.double().abs().sum()), v.flatten()[:8].clone())
            for k, v in sd.items()}


def zipf(rows, length, seed=0):
    p = torch.arange(1, 4097, dtype=torch.float64) ** -1.1
    g = torch.Generator().manual_seed(seed)
    return torch.multinomial((p / p.sum()).float(), rows * length, replacement=True, generator=g).view(rows, length)


def golden_forward(model):
    """Config 1: torch.manual_seed(0); GPT(GPTConfig()); init_weights(); fp32 eval forward on Zipf rows."""
    torch.manual_seed(0)
    gpt = model.GPT(model.GPTConfig())
    gpt.init_weights()
    gpt.eval()
    tokens = zipf(4, 2049, seed=0)
    with torch.no_grad():
        ce = gpt(tokens[:, :-1], tokens[:, 1:].contiguous(), loss_reduction='none').view(4, 2048)
    torch.save(dict(tokens=tokens.short(), ce=ce, loss_sum=ce.double().sum(),
                    weights=checksums(dict(gpt.named_parameters()))), HERE / 'gpt_forward.pt')
    print('gpt_forward: sum CE', float(ce.double().sum()))


def golden_population(eggroll, length=2048, pairs=2, sigma=0.002):
    """population_loss on 2 antithetic pairs (4 members) of EGGROLL's make_model weights, fp32 (native CPU) and
    under CPU bf16 autocast, plus the noise map pieces (offsets, gathered slices)."""
    eggroll.NOISE = SMALL_NOISE
    model = eggroll.make_model(torch.device('cpu'), 0)
    es = eggroll.Eggroll(model, pairs)
    offsets = es.offsets(step=1)
    directions = torch.tensor([0, 0, 1, 1])
    nz = es.noise(offsets, directions)
    sign = torch.tensor([sigma, -sigma]).repeat(pairs)
    tokens = zipf(1, length + 1, seed=1)[0]
    idx, tgt = tokens[:-1], tokens[1:].contiguous()
    with torch.no_grad():
        fp32 = eggroll.population_loss(model, es.params, nz, sign, idx, tgt)
        with torch.autocast('cpu', dtype=torch.bfloat16):
            bf16 = eggroll.population_loss(model, es.params, nz, sign, idx, tgt)
    gathered = {k: (tuple(t[:, :4].clone() for t in v) if isinstance(v, tuple) else v[:, :4].clone())
                for k, v in nz.items()}
    torch.save(dict(length=length, pairs=pairs, sigma=sigma, noise_size=SMALL_NOISE, buffer_sum=es.buffer.double().sum(),
                    buffer_head=es.buffer[:16].clone(), offsets={k: v.clone() for k, v in offsets.items()},
                    directions=directions, tokens=tokens.short(), loss_fp32=fp32, loss_autocast=bf16.float(),
                    gathered=gathered, weights=checksums(es.params)), HERE / f'population_T{length}.pt')
    print(f'population T={length}: fp32', fp32.tolist(), 'autocast', bf16.float().tolist())


def golden_step(eggroll, length=256, pairs=4, rows=2):
    """One Eggroll.step with CHUNK = 2 pairs: member layout, losses, fitness weights and the rebuilt gradient."""
    eggroll.NOISE = SMALL_NOISE
    eggroll.CHUNK = 2
    model = eggroll.make_model(torch.device('cpu'), 0)
    es = eggroll.Eggroll(model, pairs)
    es.loss = eggroll.population_loss
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, betas=(0.5, 0.95), eps=1e-8, weight_decay=0.0)
    tokens = zipf(rows, length + 1, seed=2)
    grads = {}
    orig = opt.step

    def capture(*a, **k):
        for n, p in model.named_parameters():
            grads[n] = p.grad.clone()
        return orig(*a, **k)

    opt.step = capture
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter('ignore')
        mean_loss = es.step(tokens[:, :-1].contiguous(), tokens[:, 1:].contiguous(), opt, step=3)
    small = {n: g for n, g in grads.items() if g.numel() <= 4096}
    corner = {n: g[:8, :8].clone() for n, g in grads.items() if g.dim() == 2}
    torch.save(dict(length=length, pairs=pairs, rows=rows, chunk=2, step=3, noise_size=SMALL_NOISE,
                    tokens=tokens.short(), mean_loss=mean_loss, grad_small=small, grad_corner=corner,
                    grad_sums={n: float(g.double().sum()) for n, g in grads.items()},
                    grad_abs={n: float(g.double().abs().sum()) for n, g in grads.items()}),
               HERE / 'eggroll_step.pt')
    print('eggroll step: mean loss', mean_loss)


def golden_implicit(root):
    """lse and center from the reference Triton kernel under the interpreter (fp32 inputs, tf32 dots evaluated in
    fp32), rows = 2, T = 256, window 128 and 256. Inputs are regenerated from the CPU generator seed by the test:
    q, k, v = randn / 8 and hub = randn, drawn in that order."""
    spec = importlib.util.spec_from_file_location('ref_moments', root / 'train/speedrun/moment_kernels.py')
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    g = torch.Generator().manual_seed(5)
    rows, t = 2, 256
    q, k, v, hub = (torch.randn(rows, t, 64, generator=g) / 8 for _ in range(4))
    hub = hub * 8
    out = {}
    for window in (128, 256):
        lse, center = mk._implicit_key_context(q, k, v, hub, window, edges=True)
        out[window] = (lse.clone(), center.clone())
    torch.save(dict(seed=5, rows=rows, length=t, out=out), HERE / 'implicit_key_context.pt')
    print('implicit_key_context: ok')


def main():
    root = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get('NOISE_REFERENCE', ''))
    assert (root / 'utils/model.py').exists(), 'pass the reference checkout as argv[1]'
    torch.set_num_threads(os.cpu_count())
    model, eggroll = load_reference(root)
    golden_forward(model)
    golden_population(eggroll, length=256)
    golden_population(eggroll, length=2048)
    golden_step(eggroll)
    golden_implicit(root)


if __name__ == '__main__':
    main()
