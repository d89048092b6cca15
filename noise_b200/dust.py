"""Dust's jittered block reruns (reference train/val/dust.py) on libnoise_b200.so.

``block_forward(x, w, ve, cos, sin, window, o=None, attn=None, fc=None, mlp=None)`` has dust.block_forward's
arguments and result (dust.py:102-125): Block.forward of one block with a draw's additive jitter at the attention
output (o), the attention or MLP output projections (attn, mlp) or the MLP hidden layer (fc). It runs the population
forward's block kernels with zero weight noise and the jitter added in their epilogues (numerics as the population
forward's: bf16 linears, fp32 residual stream). ``head_loss`` (dust.py:94-99) is noise_b200.head_loss.

``head_error(raw, y, clean_loss, draws, sigma, nrep, noise, vocab)`` is DUST.head_error (dust.py:265-303): one
256-column slab of the cached LM-head logits jittered per chunk of draws, each draw's loss recomputed from the cached
slab sums, the centred rewards contracted with the draws' noise, all on the GPU in one kernel per chunk. The draws
come from the caller's ``noise`` (DUST.noise), in the reference's order. ``install(DUST)`` makes it the class's
head_error.
"""
import ctypes

import torch

from . import _lib

D, HD = 512, 64


class _Packed:
    """bf16 packs of one block's weights (dust's self.weights[i]: q, k, v, proj, fc, out, gate), refreshed when a
    tensor's storage or version changes."""

    def __init__(self):
        self.key, self.keep, self.struct = None, None, None

    def get(self, w, layer, cos, sin, T):
        names = ('q', 'k', 'v', 'proj', 'fc', 'out', 'gate')
        key = (layer, T, cos.data_ptr(), sin.data_ptr()) + tuple(
            (w[n].data_ptr(), w[n]._version) if w.get(n) is not None else None for n in names)
        if key != self.key:
            shapes = dict(q=(D, D), k=(D, D), v=(D, D), proj=(D, D), fc=(4 * D, D), out=(D, 4 * D), gate=(8, 32))
            for n in names:
                if w.get(n) is not None and tuple(w[n].shape) != shapes[n]:
                    raise ValueError(f'{n}: shape {tuple(w[n].shape)}, expected {shapes[n]}')
            bf = lambda t: t.detach().to(torch.bfloat16).contiguous()
            qkv = torch.cat([bf(w['q']), bf(w['k']), bf(w['v'])]).contiguous()
            proj, fc, out = bf(w['proj']), bf(w['fc']), bf(w['out'])
            gate = w['gate'].detach().float().contiguous() if w.get('gate') is not None else None
            c = cos.detach().reshape(-1, HD // 2)[:T].to(torch.bfloat16).contiguous()
            s = sin.detach().reshape(-1, HD // 2)[:T].to(torch.bfloat16).contiguous()
            if c.shape[0] < T or s.shape[0] < T:
                raise ValueError(f'cos / sin: {T} positions of {HD // 2} values needed')
            _lib.require_cuda(*(z for z in (qkv, proj, fc, out, gate, c, s) if z is not None))
            st = _lib.GPT()
            st.wqkv[layer], st.wproj[layer], st.wfc[layer], st.wmproj[layer] = (z.data_ptr() for z in (qkv, proj, fc,
                                                                                                       out))
            st.wgate[layer] = gate.data_ptr() if gate is not None else None
            st.cos, st.sin = c.data_ptr(), s.data_ptr()
            self.key, self.keep, self.struct = key, (qkv, proj, fc, out, gate, c, s), st
        return self.struct


_packs = {}


def block_forward(x, w, ve, cos, sin, window, o=None, attn=None, fc=None, mlp=None):
    """dust.block_forward: x [B, T, 512] -> the block's output [B, T, 512] fp32. w: the block's weights by dust's names
    (q, k, v, gate (value-embedding blocks), proj, fc, out); ve [B, T, 512] or None; cos / sin the RoPE tables
    (any layout with 32 values per position); window the block's window; o, attn, fc, mlp the jitter sites (fp32
    [B, T, 512], [B, T, 512], [B, T, 2048], [B, T, 512]) or None. T % 128 == 0, T <= 2048."""
    B, T, C = x.shape
    if C != D:
        raise ValueError('width 512')
    layer = 1 if w.get('gate') is not None else 0  # the slot the packs use (any block of the right kind)
    pack = _packs.setdefault(id(w), _Packed())
    st = pack.get(w, layer, cos, sin, T)
    out = x.detach().float().contiguous().clone().view(B * T, D)
    keep = []

    def rows(t, width):
        if t is None:
            return None
        t = t.detach().float().contiguous().view(B * T, width)
        keep.append(t)
        return t.data_ptr()
    ve_p = rows(ve, D)
    jit = _lib.Jitter(rows(o, D), rows(attn, D), rows(fc, 4 * D), rows(mlp, D))
    _lib.require_cuda(out, *keep)
    L = _lib.lib()
    nbytes = L.noise_block_workspace_bytes(B, T)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=out.device)
    _lib.check(L.noise_block_forward(ctypes.byref(st), layer, out.data_ptr(), ve_p, ctypes.byref(jit), B, T,
                                     int(window), ws.data_ptr(), nbytes, _lib.stream_handle(out.device)),
               'noise_block_forward')
    out._noise_workspace = ws
    return out.view(B, T, D)


SLAB = 256


def chunk_size(draws, cap):
    """The largest count up to cap that divides draws (draws that share one pass, dust.py:80-82)."""
    return next(n for n in range(min(cap, draws), 0, -1) if draws % n == 0)


def head_error(raw, y, clean_loss, draws, sigma=0.1, nrep=16, noise=None, vocab=4096):
    """DUST.head_error: fp32 [b, t, V] error of the LM head's logits raw [b, t, V] (fp32 or bf16) for targets y [b, t]
    (-1: ignored) and the clean per-token losses clean_loss [b, t]; noise(n * b, t, 256) draws the jitter (bf16)."""
    if vocab != 4096:
        raise ValueError('vocab must be 4096')
    b, t = y.shape
    if tuple(raw.shape) != (b, t, vocab) or tuple(clean_loss.shape) != (b, t):
        raise ValueError(f'raw [b, t, {vocab}] and clean_loss [b, t] for y [b, t]: got {tuple(raw.shape)}, '
                         f'{tuple(clean_loss.shape)}, {tuple(y.shape)}')
    n = chunk_size(draws, nrep)
    slabs = vocab // SLAB
    raw2 = raw.detach()
    if raw2.dtype not in (torch.float32, torch.bfloat16):
        raw2 = raw2.float()
    raw2 = raw2.contiguous().view(b * t, raw.shape[-1])
    y2 = y.detach().long().contiguous().view(-1)
    cl = clean_loss.detach().float().contiguous().view(-1)
    _lib.require_cuda(raw2, y2, cl)
    dt = 1 if raw2.dtype == torch.bfloat16 else 0
    dev = raw2.device
    sums, total, clean_t = torch.empty(b * t, slabs, device=dev), torch.empty(b * t, device=dev), \
        torch.empty(b * t, device=dev)
    error = torch.zeros(b * t, raw.shape[-1], device=dev)
    L, stream = _lib.lib(), _lib.stream_handle(dev)
    _lib.check(L.noise_head_error_prep(raw2.data_ptr(), dt, raw2.stride(0), y2.data_ptr(), b * t, sums.data_ptr(),
                                       total.data_ptr(), clean_t.data_ptr(), stream), 'noise_head_error_prep')
    for chunk in range(draws // n):
        a = noise(n * b, t, SLAB).to(torch.bfloat16).contiguous()
        if tuple(a.shape) != (n * b, t, SLAB):
            raise ValueError(f'noise drew {tuple(a.shape)}, expected {(n * b, t, SLAB)}')
        _lib.require_cuda(a)
        _lib.check(L.noise_head_error_chunk(raw2.data_ptr(), dt, raw2.stride(0), a.data_ptr(), y2.data_ptr(),
                                            cl.data_ptr(), sums.data_ptr(), total.data_ptr(), clean_t.data_ptr(), b,
                                            t, n, chunk % slabs, float(sigma), error.data_ptr(), stream),
                   'noise_head_error_chunk')
    return error.view(b, t, -1) / (draws // slabs)


def install(DUST):
    """DUST.head_error -> this implementation (same arguments: draws, sigma), reading the instance's cached logits,
    targets, clean losses, chunk cap and noise generator. Returns DUST."""
    def method(self, draws, sigma=0.1):
        return head_error(self.outputs['lm_head'], self.y, self.clean_loss, draws, sigma, self.recipe.nrep,
                          self.noise, self.model.config.vocab_size)
    DUST.head_error = method
    return DUST

