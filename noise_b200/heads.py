"""The identity phase's head-sharding kernels (reference train/speedrun/run.py:3694-3804) on libnoise_b200.so.

Same names, arguments and results as the reference's functions:

- ``pack_heads_kernel(qs, ks, vals, outs, targets, lses)`` -> the (H, L, n, PACK) bf16 all_to_all send buffer
  (run.py:3718-3731): every head's q, k, v, attention-output and target pieces and its lse's fp32 bits.
- ``head_prep_fused(got, cos, sin, b, t)`` -> the received heads' RoPE'd and normed queries and keys, values, hubs,
  fp32 queries, the keys' pair features, lse, hub . o, square norms and steps (run.py:3781-3796).
- ``id_head_scores(got, rope32, back, b, t)``: head_prep, then the query- and key-moment credits into
  back (W, L, 3, N, 64) bf16 (run.py:3799-3803), in one library call.
"""
import ctypes

import torch

from . import _lib

H, HD, PACK = 8, 64, 5 * 64 + 2
KEY_SIGMA, NORM_EPS = 0.003, 1e-6  # run.py's KEY_SIGMA and NORM_EPS


def _two_byte(t, what):
    if t.element_size() != 2 or t.stride(-1) != 1:
        raise ValueError(f'{what}: a 16-bit tensor with a unit last stride')
    return t


def pack_heads_kernel(qs, ks, vals, outs, targets, lses):
    """identity_grad's (H, L, n, PACK) all_to_all send buffer from each layer's (tokens, D) pieces and its lse
    (rows, H, t) (run.py:3718-3731)."""
    n, t = qs[0].shape[0], lses[0].shape[-1]
    dev = qs[0].device
    layers = len(qs)
    out = torch.empty(H, layers, n, PACK, device=dev, dtype=torch.bfloat16)
    pieces = (_lib.HeadPieces * layers)()
    keep = []
    for i, group in enumerate(zip(qs, ks, vals, outs, targets, lses)):
        *mats, lse = group
        mats = [_two_byte(m.detach(), 'q, k, v, o, target') for m in mats]
        lse = lse.detach().float().contiguous()
        _lib.require_cuda(*mats, lse)
        keep += mats + [lse]
        p = pieces[i]
        p.q, p.k, p.v, p.o, p.target = (m.data_ptr() for m in mats)
        p.q_stride, p.k_stride, p.v_stride, p.o_stride, p.target_stride = (m.stride(0) for m in mats)
        p.lse = lse.data_ptr()
    _lib.check(_lib.lib().noise_pack_heads(pieces, layers, n, t, out.data_ptr(), _lib.stream_handle(dev)),
               'noise_pack_heads')
    return out


def _prep_struct(got, b, t, keep_k32):
    w, layers, n, _ = got.shape
    rows = layers * b
    dev = got.device
    new = lambda *s, dtype=torch.float32: torch.empty(*s, device=dev, dtype=dtype)
    bf = torch.bfloat16
    q16, k16, v16, hub16 = (new(rows, t, HD, dtype=bf) for _ in range(4))
    q32 = new(rows, t, HD)
    k32 = new(rows, t, HD) if keep_k32 else None
    pairs = (new(rows, t, HD, dtype=bf), new(rows, t, 2 * HD, dtype=bf), new(rows, t, HD // 2, dtype=bf))
    lse, hub_out, sq_q, sq_k, steps_q, steps_k = (new(rows, t) for _ in range(6))
    s = _lib.HeadPrep()
    s.q16, s.k16, s.v16, s.hub16, s.q32 = (z.data_ptr() for z in (q16, k16, v16, hub16, q32))
    s.k32 = k32.data_ptr() if k32 is not None else None
    s.f2, s.f4, s.xy = (z.data_ptr() for z in pairs)
    s.lse, s.hub_out, s.sq_q, s.sq_k, s.steps_q, s.steps_k = (z.data_ptr() for z in
                                                             (lse, hub_out, sq_q, sq_k, steps_q, steps_k))
    return s, (q16, k16, v16, hub16, q32, pairs, lse, hub_out, sq_q, sq_k, steps_q, steps_k), k32


def _got(got, b, t):
    got = _two_byte(got.detach(), 'got')
    if got.dim() != 4 or got.shape[-1] != PACK or not got.is_contiguous():
        raise ValueError(f'got: contiguous (W, L, N, {PACK})')
    w, _, n, _ = got.shape
    if w * n != b * t:
        raise ValueError('got holds W * N = b * t tokens per layer')
    _lib.require_cuda(got)
    return got


def head_prep_fused(got, cos, sin, b: int, t: int):
    """The received heads' RoPE'd queries and keys, values, hubs, lse and square norms and steps from got (W, L, N,
    PACK), in one kernel pass (run.py:3781-3796). Returns (q16, k16, v16, hub16, q32, (f2, f4, xy), lse, hub_out,
    sq_q, sq_k, steps_q, steps_k)."""
    got = _got(got, b, t)
    w, layers, n, _ = got.shape
    cos, sin = (z.detach().float().contiguous() for z in (cos, sin))
    s, result, _ = _prep_struct(got, b, t, keep_k32=False)
    _lib.check(_lib.lib().noise_head_prep(got.data_ptr(), w, layers, n, cos.data_ptr(), sin.data_ptr(), t, KEY_SIGMA,
                                          NORM_EPS, ctypes.byref(s), _lib.stream_handle(got.device)),
               'noise_head_prep')
    return result


def id_head_scores(got, rope32, back, b, t):
    """head_prep_fused, then the query credits into back[:, :, 0] and the key credits and value sums into
    back[:, :, 1], back[:, :, 2] (run.py:3799-3803); back: bf16 (W, L, 3, N, 64), written in place."""
    got = _got(got, b, t)
    w, layers, n, _ = got.shape
    if back.dtype != torch.bfloat16 or tuple(back.shape) != (w, layers, 3, n, HD) or not back.is_contiguous():
        raise ValueError('back: contiguous bf16 (W, L, 3, N, 64)')
    cos, sin = (z.detach().float().contiguous() for z in rope32)
    L = _lib.lib()
    nbytes = L.noise_id_head_scores_workspace_bytes(w, layers, n)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=got.device)
    _lib.check(L.noise_id_head_scores(got.data_ptr(), w, layers, n, cos.data_ptr(), sin.data_ptr(), t, KEY_SIGMA,
                                      NORM_EPS, back.data_ptr(), ws.data_ptr(), nbytes,
                                      _lib.stream_handle(got.device)), 'noise_id_head_scores')
