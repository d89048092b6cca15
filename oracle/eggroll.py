"""CPU restatement of EGGROLL's population-perturbed forward and update (reference
``archive/10M/train/val/eggroll.py``) — test infrastructure only.

Two arithmetic modes:
- ``autocast=False``: everything fp32, which is how the reference runs on the CPU.
- ``autocast=True``: the rounding points of ``torch.autocast('cuda', torch.bfloat16)`` around the reference's
  matmuls (eggroll.py:144-145): every ``@`` takes bf16 operands, accumulates in fp32 and returns bf16; the rank-1
  correction's ``sign * (x @ b)`` then promotes back to fp32 and multiplies the fp32 ``a`` (eggroll.py:56-58), so a
  perturbed linear returns fp32 = bf16(x W^T) + sign bf16(x b) a. Attention follows flex attention's autocast rule
  (``gpt.attention_autocast``: q, k, v cast to bf16, fp32 softmax, bf16 probabilities and output). Embeddings, norms,
  RoPE and the cross-entropy stay fp32 as in the reference.
"""
import torch
from torch.nn import functional as F

from . import gpt

NOISE = 2 ** 28   # eggroll.py:35
SIGMA = 0.002     # eggroll.py:31
CHUNK = 256       # eggroll.py:34


def _rb(t):
    """Round to bf16 and back."""
    return t.bfloat16().float()


def make_buffer(n=NOISE, seed=0, device='cpu'):
    """The fixed N(0, 1) buffer every perturbation is sliced from (eggroll.py:114)."""
    return torch.randn(n, device=device, generator=torch.Generator(device).manual_seed(seed))


def offsets(shapes, pairs, step, seed=0, n_noise=NOISE, device='cpu'):
    """Per parameter, in ``named_parameters()`` order, ``pairs`` slice starts drawn from a generator seeded
    1_000_003 * seed + step (eggroll.py:117-120). shapes: list of (name, shape). Returns name -> int64 [pairs]."""
    g = torch.Generator(device).manual_seed(1_000_003 * seed + step)
    return {name: torch.randint(0, n_noise - sum(shape), (pairs,), device=device, generator=g)
            for name, shape in shapes}


def noise(buffer, offs, directions, shapes):
    """name -> (a [n, out], b [n, in]) for matrices and embeddings, eps [n, numel] for 1-D parameters: the slice
    buffer[off : off + out + in] split into its first ``out`` and next ``in`` values (eggroll.py:122-128)."""
    out = {}
    for name, shape in shapes:
        rows = buffer[offs[name][directions, None] + torch.arange(sum(shape), device=buffer.device)]
        out[name] = rows.split(list(shape), dim=1) if len(shape) == 2 else rows
    return out


def lowrank(x, weight, a, b, sign, autocast=False):
    """x [m, T, in] through W [out, in] + sign a b^T per member (eggroll.py:56-58)."""
    if autocast:
        base = _rb(_rb(x) @ _rb(weight).t())
        s = _rb(_rb(x) @ _rb(b).unsqueeze(-1))
        return base + sign[:, None, None] * s * a[:, None, :]
    return x @ weight.t() + sign[:, None, None] * (x @ b.unsqueeze(-1)) * a[:, None, :]


def lowrank_embed(weight, a, b, idx, sign):
    """Rows of W [V, d] + sign a b^T for token ids idx [T] (eggroll.py:61-63), fp32."""
    return weight[idx].unsqueeze(0) + sign[:, None, None] * a[:, idx].unsqueeze(-1) * b[:, None, :]


def population_loss(w, nz, sign, idx, targets, autocast=False, reduction='mean', head_slice=32, ignore_index=-100):
    """Per-member cross-entropy [m] of m perturbed models on one sequence (eggroll.py:66-103).

    w: name -> fp32 weight; nz: ``noise()`` output for the m members; sign [m] (+-sigma); idx, targets [T] int64.
    reduction 'mean' is the reference's output; 'sum' is mean * T (the summed per-member fitness); 'none' the
    per-token losses [m, T] it averages. ignore_index as F.cross_entropy's (the reference leaves the default)."""
    heads, dim = gpt.N_HEAD, gpt.HEAD_DIM
    m, length = sign.shape[0], idx.shape[0]
    cos, sin = (z[:length].float() for z in gpt.rotary())
    s = sign[:, None, None]
    x = x0 = gpt.norm(lowrank_embed(w['transformer.wte.weight'], *nz['transformer.wte.weight'], idx, sign))
    for i in range(gpt.N_LAYER):
        pre = f'transformer.h.{i}.'
        resid = w['resid_lambdas'][i] + s * nz['resid_lambdas'][:, i, None, None]
        mix = w['x0_lambdas'][i] + s * nz['x0_lambdas'][:, i, None, None]
        x = resid * x + mix * x0

        def linear(name, inp):
            return lowrank(inp, w[pre + name], *nz[pre + name], sign, autocast)

        h = gpt.norm(x)
        q = linear('attn.c_q.weight', h).view(m, length, heads, dim)
        k = linear('attn.c_k.weight', h).view(m, length, heads, dim)
        v = linear('attn.c_v.weight', h).view(m, length, heads, dim)
        if gpt.has_ve(i):
            name = f'value_embeds.{i}.weight'
            ve = lowrank_embed(w[name], *nz[name], idx, sign).view(m, length, heads, dim)
            gate = 2 * torch.sigmoid(linear('attn.ve_gate.weight', h[..., :gpt.VE_GATE_CHANNELS]))
            v = v + gate.unsqueeze(-1) * ve
        q, k = gpt.norm(gpt.apply_rotary_emb(q, cos, sin)), gpt.norm(gpt.apply_rotary_emb(k, cos, sin))
        attend = gpt.attention_autocast if autocast else gpt.attention
        y = torch.cat([attend(q[j:j + 1], k[j:j + 1], v[j:j + 1], gpt.WINDOWS[i]) for j in range(m)])
        x = x + linear('attn.c_proj.weight', y.reshape(m, length, -1))
        x = x + linear('mlp.c_proj.weight', F.relu(linear('mlp.c_fc.weight', gpt.norm(x))).square())
    h = gpt.norm(x)
    losses = []
    for c in range(0, m, head_slice):
        part = slice(c, c + head_slice)
        a, b = (t[part] for t in nz['lm_head.weight'])
        logits = lowrank(h[part], w['lm_head.weight'], a, b, sign[part], autocast)[..., :gpt.VOCAB].float()
        logits = 15 * torch.tanh(logits / 15)
        ce = F.cross_entropy(logits.flatten(0, 1), targets.repeat(logits.shape[0]), reduction='none',
                             ignore_index=ignore_index)
        ce = ce.view(-1, length)
        losses.append(ce if reduction == 'none' else ce.sum(-1) if reduction == 'sum' else ce.mean(-1))
    return torch.cat(losses)


def zero_noise(m=1):
    """``noise()``-shaped all-zero perturbations for m members: the un-perturbed model."""
    return {name: (tuple(torch.zeros(m, n) for n in shape) if len(shape) == 2 else torch.zeros(m, shape[0]))
            for name, shape in gpt.param_shapes()}


def forward_rows(w, idx, targets, autocast=True, loss_reduction='mean'):
    """GPT.forward(idx, targets, loss_reduction) (utils/model.py:193-209: softcap 15, ignore_index -1) on B distinct
    rows, with the population forward's arithmetic (``population_loss`` at sign 0, one row at a time). idx, targets
    int64 [B, T]; 'mean' / 'sum' give a 0-d tensor, 'none' [B * T]."""
    ce = torch.cat([population_loss(w, zero_noise(1), torch.zeros(1), idx[b], targets[b], autocast, 'none',
                                    ignore_index=-1) for b in range(idx.shape[0])]).flatten()
    if loss_reduction == 'none':
        return ce
    total = ce.double().sum()
    return (total if loss_reduction == 'sum' else total / (targets != -1).sum()).float()


def head_loss(x, weight, targets, autocast=True):
    """dust.head_loss (train/val/dust.py:94-99): norm, LM head, [:vocab], softcap 15, per-token cross-entropy with
    ignore_index -1 (reduction 'none'). x [N, T, 512] fp32; weight [>= vocab, 512]; targets [N, T] -> [N * T]. With
    autocast the head matmul takes bf16 operands and returns bf16, as under torch.autocast."""
    h = gpt.norm(x.float())
    wv = weight[:gpt.VOCAB].float()
    logits = _rb(_rb(h) @ _rb(wv).t()) if autocast else h @ wv.t()
    logits = 15 * torch.tanh(logits.float() / 15)
    return F.cross_entropy(logits.flatten(0, 1), targets.flatten(), ignore_index=-1, reduction='none')


def member_layout(pairs, rows, world=1, rank=0):
    """Eggroll.step's member bookkeeping (eggroll.py:134-143): members = max(2 pairs, 2 rows); member i uses pair
    (i mod 2 pairs) // 2 with sign +sigma for even i and -sigma for odd i, and data row i // per_seq.
    Returns (members, per_seq, per_rank, directions [members], positive [members] bool, row [members])."""
    members = max(2 * pairs, 2 * rows)
    per_seq, per_rank = members // rows, members // world
    i = torch.arange(members)
    return members, per_seq, per_rank, (i % (2 * pairs)) // 2, i % 2 == 0, i // per_seq


def fitness_weights(losses, pairs):
    """Antithetic fitness l[odd] - l[even], z-scored, summed per pair (eggroll.py:151-154)."""
    fitness = losses[1::2] - losses[0::2]
    fitness = fitness / (fitness.std() + 1e-8)
    weight = torch.zeros(pairs, dtype=losses.dtype).index_add_(0, torch.arange(len(fitness)) % pairs, fitness)
    return weight, len(fitness)


def rebuild_update(buffer, offs, weight, count, shapes, chunk=CHUNK):
    """The seed-rebuilt gradient -sum_j w_j a_j b_j^T / count per parameter (eggroll.py:155-166), fp32."""
    pairs = weight.shape[0]
    grads = {name: torch.zeros(shape) for name, shape in shapes}
    for start in range(0, pairs, chunk):
        directions = torch.arange(start, min(pairs, start + chunk))
        w = weight[directions]
        for name, n in noise(buffer, offs, directions, shapes).items():
            if isinstance(n, tuple):
                grads[name] -= (w[:, None] * n[0]).t() @ n[1]
            else:
                grads[name] -= w @ n
    return {name: g / count for name, g in grads.items()}
