"""CPU restatement of the identity phase's readout cycle (reference train/speedrun/run.py:3569-3686) — test
infrastructure only: the checker of noise_b200.cycle, never called by the product path. Written directly from the
cycle's definition: the moved partition's third-order expansion, fp64 by default, with the reference's bf16 roundings
of the fast weights, of the powers of c and of the bf16 GEMMs' outputs."""
import torch

D, VOCAB, CAP = 512, 4096, 15.0
SIGMA, HEAD_SIGMA = 0.005, 0.1
EPS = torch.finfo(torch.float32).eps


def _rb(t):
    return t.to(torch.bfloat16).to(t.dtype)


def softcap(x):
    return CAP * torch.tanh(x / CAP)


def coordinate_change(raw, targets, dtype=torch.float64):
    raw = raw.to(dtype)
    z = softcap(raw)
    up, down = softcap(raw + HEAD_SIGMA), softcap(raw - HEAD_SIGMA)
    w = torch.softmax(z, -1)
    change = torch.log1p(w * torch.expm1(up - z)) - torch.log1p(w * torch.expm1(down - z))
    change = change - torch.nn.functional.one_hot(targets, VOCAB).to(dtype) * (up - down)
    return change / (2 * HEAD_SIGMA)


def top_credit(H, signs, lm_head, x, y, dtype=torch.float64):
    """[n, 512] for the basis H * signs, lm_head [512, 4096], stream x [n, 512], targets y [n]."""
    h = (H * signs[None, :]).to(dtype)
    W = lm_head.to(dtype)
    x = x.to(dtype)
    c, base = h @ W, x @ W
    sq = (x * x).sum(-1, keepdim=True)
    steps = SIGMA * torch.clamp(torch.sqrt(sq / D), min=1e-6)
    inv = torch.rsqrt((sq + 2 * steps * (x @ h.T) + steps * steps * D) / D + EPS)
    inv0 = torch.rsqrt(sq / D + EPS)
    delta, sigma = inv / inv0 - 1, steps * inv
    z = base * inv0
    t = torch.tanh(z / CAP)
    f = torch.exp(CAP * t)
    g1 = 1 - t * t
    d1, d2 = -2 * t * g1 / CAP, -2 * g1 * (1 - 3 * t * t) / CAP ** 2
    g2, g3 = g1 * g1 + d1, g1 ** 3 + 3 * g1 * d1 + d2
    fz, fzz = f * z, f * z * z
    total = f.sum(-1, keepdim=True)
    rows = torch.stack([(fz * g1).sum(-1), (fzz * g2).sum(-1), (fzz * z * g3).sum(-1)], -1)
    fast = [_rb(v) for v in (fz * g2, fzz * g3, f * g2, fz * g3, f * g3)]
    powers = [_rb(c), _rb(c * c), _rb(c * c * c)]
    prods = [_rb(fast[k] @ powers[p].T) for k, p in enumerate((0, 0, 1, 1, 2))]
    ratio = (sigma * ((f * g1) @ c.T) + delta * sigma * prods[0] + 0.5 * delta ** 2 * sigma * prods[1]
             + 0.5 * sigma ** 2 * prods[2] + 0.5 * delta * sigma ** 2 * prods[3] + sigma ** 3 / 6 * prods[4]
             + delta * rows[:, :1] + 0.5 * delta ** 2 * rows[:, 1:2] + delta ** 3 / 6 * rows[:, 2:])
    part = torch.log(total)
    base_y = base.gather(1, y[:, None])
    clean = part - softcap(base_y * inv0)
    moved = part + torch.log1p(ratio / total) - softcap((base_y + steps * c.T[y]) * inv)
    return ((moved - clean) / steps) @ h / D
