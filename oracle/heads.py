"""CPU restatement of the identity phase's head-sharding kernels (reference train/speedrun/run.py:3694-3804) — test
infrastructure only: the checker of noise_b200.heads, never called by the product path.

- ``pack_heads``: _pack_heads_kernel / pack_heads_kernel (run.py:3698-3731), a byte-exact gather.
- ``head_prep``: _head_prep_kernel / head_prep_fused (run.py:3734-3796), fp32 arithmetic.
- ``id_head_scores``: id_head_scores (run.py:3799-3803) = head_prep, then the query- and key-moment credits of
  oracle.credit on the received rows, scattered back to the (W, L, 3, N, 64) return layout.
"""
import torch

from . import credit

H, HD, PACK = 8, 64, 5 * 64 + 2
KEY_SIGMA, NORM_EPS = 0.003, 1e-6


def pack_heads(qs, ks, vals, outs, targets, lses):
    """(H, L, n, PACK) bf16: row (h, l, tok) = head h's 64 columns of q, k, v, o, target of layer l at tok, then the
    fp32 bits of lse[tok // t, h, tok % t] as two 16-bit words (run.py:3699-3715)."""
    n, t = qs[0].shape[0], lses[0].shape[-1]
    out = torch.empty(H, len(qs), n, PACK, dtype=torch.int16)
    for i, (q, k, v, o, tg, lse) in enumerate(zip(qs, ks, vals, outs, targets, lses)):
        for j, piece in enumerate((q, k, v, o, tg)):
            bits = piece[:, :H * HD].contiguous().view(torch.int16).view(n, H, HD)
            out[:, i, :, j * HD:(j + 1) * HD] = bits.permute(1, 0, 2)
        lse_tok = lse.float().permute(1, 0, 2).reshape(H, n).contiguous()  # [h, tok]
        out[:, i, :, 5 * HD:] = lse_tok.view(torch.int32).unsqueeze(-1).view(torch.int16).view(H, n, 2)
    return out.view(torch.bfloat16)


def received_rows(got, b, t):
    """got (W, L, N, C) -> (L * b, t, C): received row (w, l, i) is token (l * W + w) * N + i (run.py:3743-3746)."""
    w, layers, n, c = got.shape
    return got.permute(1, 0, 2, 3).reshape(layers * b, t, c)


def return_layout(x, w, n):
    """(L * b, t, 64) -> (W, L, N, 64), the inverse of ``received_rows`` (moment_kernels._query_store's layout)."""
    layers = x.shape[0] * x.shape[1] // (w * n)
    return x.reshape(layers, w, n, x.shape[-1]).permute(1, 0, 2, 3)


def head_prep(got, cos, sin, b, t, sigma=KEY_SIGMA, eps=NORM_EPS):
    """run.py:3734-3775 in fp32 on the received rows: dict of q16, k16, v16, hub16 (bf16), q32, k32 (fp32), f2, f4,
    xy (bf16 pair features of the keys), lse, hub_out, sq_q, sq_k, steps_q, steps_k."""
    rows = received_rows(got, b, t)
    w, layers, n, _ = got.shape
    pos = (torch.arange(n) % t).expand(layers, w, n).reshape(layers * b, t)  # pos = i % T of received row (w, l, i)
    c, s = cos.float()[pos], sin.float()[pos]
    out = {}
    for j, name in enumerate(('q', 'k')):
        x = rows[..., j * HD:(j + 1) * HD].float()
        x1, x2 = x[..., :HD // 2], x[..., HD // 2:]
        r1, r2 = x1 * c + x2 * s, x1 * -s + x2 * c
        inv = torch.rsqrt(((r1 * r1).sum(-1) + (r2 * r2).sum(-1)) / HD + eps)[..., None]
        r = torch.cat([r1 * inv, r2 * inv], -1)
        sq = (x1 * x1).sum(-1) + (x2 * x2).sum(-1)
        out[name + '16'] = r.bfloat16()
        out[name + '32'] = r
        out['sq_' + name] = sq
        out['steps_' + name] = sigma * torch.clamp(torch.sqrt(sq / HD), min=1e-6)
    x, y = out['k32'][..., :HD // 2] * HD ** -0.5, out['k32'][..., HD // 2:] * HD ** -0.5
    out['f2'] = torch.stack([x, y], -1).flatten(-2).bfloat16()                      # (x_i, y_i)
    out['f4'] = torch.stack([x, x * x, y, y * y], -1).flatten(-2).bfloat16()         # (x_i, x_i^2, y_i, y_i^2)
    out['xy'] = (x * y).bfloat16()
    out['v16'] = rows[..., 2 * HD:3 * HD].contiguous()
    out['hub16'] = rows[..., 4 * HD:5 * HD].contiguous()
    out['hub_out'] = (rows[..., 4 * HD:5 * HD].float() * rows[..., 3 * HD:4 * HD].float()).sum(-1)
    out['lse'] = rows[..., 5 * HD:].contiguous().view(torch.float32)[..., 0]
    return out


def id_head_scores(got, cos, sin, b, t, dtype=torch.float64):
    """back (W, L, 3, N, 64) in ``dtype``: slot 0 the query credits (full causal window), 1 the key credits, 2 the
    value sums, from head_prep's tensors and the raw q / k pieces of got (run.py:3799-3803)."""
    w, layers, n, _ = got.shape
    p = head_prep(got, cos, sin, b, t)
    rows = received_rows(got, b, t)
    bf = lambda z: z.float()
    cs, sn = cos[:t].float(), sin[:t].float()
    query = credit.moment_query_scores(bf(p['q16']), bf(p['k16']), bf(p['v16']), bf(p['hub16']),
                                       rows[..., :HD].float(), p['sq_q'], p['k32'], cs, sn, p['lse'], p['hub_out'],
                                       p['steps_q'], t, dtype=dtype, emulate=True)
    keys, values = credit.moment_key_scores(bf(p['q16']), bf(p['k16']), bf(p['v16']), bf(p['hub16']),
                                            rows[..., HD:2 * HD].float(), p['sq_k'], p['q32'], cs, sn, p['lse'],
                                            p['hub_out'], p['steps_k'], dtype=dtype, emulate=True)
    return torch.stack([return_layout(z, w, n) for z in (query, keys, values)], 2)
