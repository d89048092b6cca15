"""CPU restatement of Dust's jittered block rerun (reference train/val/dust.py:102-125, block_forward) — test
infrastructure only: the checker of noise_b200.dust. ``autocast=False`` is fp32 throughout (the reference on the
CPU); ``autocast=True`` the rounding points of the population forward (bf16 operands and bf16 outputs of every
linear, fp32 residual stream), which noise_b200.dust.block_forward follows."""
import torch
from torch.nn import functional as F

from . import gpt


def _rb(t):
    return t.to(torch.bfloat16).to(t.dtype)


def block_forward(x, w, ve, cos, sin, window, o=None, attn=None, fc=None, mlp=None, autocast=True):
    """x [B, T, 512] -> [B, T, 512]; w: q, k, v, gate (or None), proj, fc, out; cos / sin [T, 32]."""
    add = lambda t, j: t if j is None else t + j.float()
    lin = (lambda a, W: _rb(_rb(a) @ _rb(W.float()).t())) if autocast else (lambda a, W: a @ W.float().t())
    B, T, C = x.shape
    x = x.float()
    h = gpt.norm(x)
    q, k, v = (lin(h, w[n]).view(B, T, gpt.N_HEAD, gpt.HEAD_DIM) for n in ('q', 'k', 'v'))
    if ve is not None:
        gate = 2 * torch.sigmoid(lin(h[..., :w['gate'].shape[1]], w['gate']))
        v = v + gate.unsqueeze(-1) * ve.float().view_as(v)
    q, k = gpt.norm(gpt.apply_rotary_emb(q, cos, sin)), gpt.norm(gpt.apply_rotary_emb(k, cos, sin))
    y = add(gpt.attention(q, k, v, window).reshape(B, T, C), o)
    x = x + add(lin(y, w['proj']), attn)
    hidden = add(lin(gpt.norm(x), w['fc']), fc)
    return x + add(lin(F.relu(hidden).square(), w['out']), mlp)


def head_error(raw, y, clean_loss, noises, sigma=0.1, vocab=4096, slab=256):
    """DUST.head_error (dust.py:265-303) with the chunks' draws given (noises[i]: [n * b, t, slab], bf16): fp32
    [b, t, V]; the draw contraction rounded to bf16 as the reference's bf16 einsum."""
    b, t = y.shape
    n = noises[0].shape[0] // b
    slabs = vocab // slab
    logits = 15 * torch.tanh(raw[..., :vocab].float() / 15)
    slab_sums = logits.exp().view(b, t, slabs, slab).sum(-1)
    total = slab_sums.sum(-1)
    target = y.clamp(min=0)
    clean_target = logits.gather(-1, target.unsqueeze(-1)).squeeze(-1)
    target = target.repeat(n, 1)
    error = torch.zeros(raw.shape, dtype=torch.float32)
    for chunk, a in enumerate(noises):
        block = chunk % slabs
        lo = block * slab
        changed = 15 * torch.tanh((raw[..., lo:lo + slab].float().repeat(n, 1, 1) + sigma * a.float()) / 15)
        partition = (total - slab_sums[..., block]).repeat(n, 1) + changed.exp().sum(-1)
        in_slab = (target >= lo) & (target < lo + slab)
        tl = torch.where(in_slab, changed.gather(-1, (target - lo).clamp(0, slab - 1).unsqueeze(-1)).squeeze(-1),
                         clean_target.repeat(n, 1))
        loss = (partition.log() - tl).view(n, b, t)
        reward = torch.where(y.unsqueeze(0) != -1, clean_loss.unsqueeze(0) - loss, 0)
        if b > 1:
            reward = reward - reward.mean(1, keepdim=True)
        w = _rb(reward / sigma)
        upd = torch.einsum('nbt,nbtd->btd', w, a.float().view(n, b, t, slab))
        error[..., lo:lo + slab] -= _rb(upd)
    return error / (len(noises) * n // slabs)  # draws // slabs
