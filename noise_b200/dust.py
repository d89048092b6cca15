"""Dust's jittered block reruns (reference train/val/dust.py) on libnoise_b200.so.

``block_forward(x, w, ve, cos, sin, window, o=None, attn=None, fc=None, mlp=None)`` has dust.block_forward's
arguments and result (dust.py:102-125): Block.forward of one block with a draw's additive jitter at the attention
output (o), the attention or MLP output projections (attn, mlp) or the MLP hidden layer (fc). It runs the population
forward's block kernels with zero weight noise and the jitter added in their epilogues (numerics as the population
forward's: bf16 linears, fp32 residual stream). ``head_loss`` (dust.py:94-99) is noise_b200.head_loss.
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
            bf = lambda t: t.detach().to(torch.bfloat16).contiguous()
            qkv = torch.cat([bf(w['q']), bf(w['k']), bf(w['v'])]).contiguous()
            proj, fc, out = bf(w['proj']), bf(w['fc']), bf(w['out'])
            gate = w['gate'].detach().float().contiguous() if w.get('gate') is not None else None
            c = cos.detach().reshape(-1, HD // 2)[:T].to(torch.bfloat16).contiguous()
            s = sin.detach().reshape(-1, HD // 2)[:T].to(torch.bfloat16).contiguous()
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
    _lib.require_cuda(out)
    L = _lib.lib()
    nbytes = L.noise_block_workspace_bytes(B, T)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=out.device)
    _lib.check(L.noise_block_forward(ctypes.byref(st), layer, out.data_ptr(), ve_p, ctypes.byref(jit), B, T,
                                     int(window), ws.data_ptr(), nbytes, _lib.stream_handle(out.device)),
               'noise_block_forward')
    out._noise_workspace = ws
    return out.view(B, T, D)
