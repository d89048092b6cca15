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
