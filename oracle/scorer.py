"""CPU restatement of the true-path readout's scorer (reference train/val/run.py, `readout` section :5900-6040) —
test infrastructure only: the checker of noise_b200.scorer, never called by the product path."""
import torch

H, D, W = 8, 64, 512
NEPS = 1.1920928955078125e-07


def _rb(t):
    return t.to(torch.bfloat16).to(t.dtype)


def stats(delta, X, SQX, start, n, eps, dtype=torch.float64):
    """(DB bf16 [m, n, 512], ST [m, n, 2]) (stats_kernel, :5968-5988)."""
    m = delta.shape[0]
    d = delta[:, :n].to(dtype)
    tok = start + torch.arange(m)
    x, sq = X[tok].to(dtype), SQX[tok].to(dtype)[:, None]
    dotx, sqd = (d * x[:, None]).sum(-1), (d * d).sum(-1)
    inv0, inv = torch.rsqrt(sq / W + eps), torch.rsqrt((sq + 2 * dotx + sqd) / W + eps)
    return delta[:, :n].to(torch.bfloat16), torch.stack([inv, (inv - inv0) / inv0], -1)


def _score(dr, dv, r0, tok, tb, diag, dtype):
    """Scores [m, n] (summed over heads) and the self-edge [m, n, 512] of rows with key change dr, value change dv
    [m, n, H, D] against the tables of tokens tok [m]; r0 [m, H, D]."""
    U, Wv, M1, M2, QD, GD, AD, CD, VT, OT = (z[tok].to(dtype) for z in tb)
    r0 = r0.to(dtype)[:, None]
    square = (r0 * r0).sum(-1, keepdim=True)
    grow = (2 * (r0 * dr).sum(-1, keepdim=True) + (dr * dr).sum(-1, keepdim=True)) / D
    inverse, moved = torch.rsqrt(square / D + NEPS), torch.rsqrt(square / D + grow + NEPS)
    dk = dr * moved - r0 * (grow * (inverse * moved) ** 2 / (inverse + moved))
    x = (dk * QD[:, None]).sum(-1) * D ** -0.5
    a = AD[:, None]
    e = torch.expm1(x)
    gain, vgain = a * e / (1 + a * e), (a + a * e) / (1 + a * e)
    total = (dk * U[:, None]).sum(-1) * D ** -0.5 + (dv * Wv[:, None]).sum(-1)
    dkb = _rb(dk)
    total = total + (torch.einsum('mnhi,mhij->mnhj', dkb, M1) * dk).sum(-1) / D
    total = total + (torch.einsum('mnhi,mhij->mnhj', dkb, M2) * dv).sum(-1) * D ** -0.5
    if diag:
        total = total + gain * CD[:, None] + vgain * (dv * GD[:, None]).sum(-1)
    se = gain[..., None] * (VT - OT)[:, None] + vgain[..., None] * dv
    return total.sum(-1), se.flatten(-2)


def staged(UP, ST, R0, VC, GZ, VE, CS, SN, tables, start, n, gated, diag, dtype=torch.float64):
    """(out [m, n], se [m, n, 512]) of staged_kernel (:5991-6040); tables = (U, W, M1, M2, QD, GD, AD, CD, VT, OT)."""
    m = ST.shape[0] // n if ST.dim() == 2 else ST.shape[0]
    st = ST.reshape(m, n, 2).to(dtype)
    inv, coef = st[..., 0:1, None], st[..., 1:2, None]       # [m, n, 1, 1]
    tok = start + torch.arange(m)
    up = UP.reshape(m, n, -1).to(dtype)
    uk = up[..., :W].reshape(m, n, H, D)
    uv = up[..., W:2 * W].reshape(m, n, H, D)
    r0 = R0[tok].to(dtype)                                    # [m, H, D]
    c, s = CS[tok].to(dtype)[:, None, None], SN[tok].to(dtype)[:, None, None]  # [m, 1, 1, 32]
    ul, uh = uk[..., :D // 2], uk[..., D // 2:]
    dr = inv * torch.cat([ul * c + uh * s, uh * c - ul * s], -1) + coef * r0[:, None]
    dv = inv * uv + coef * VC[tok].to(dtype).reshape(m, 1, H, D)
    if gated:
        ug = up[..., 2 * W:2 * W + H]                         # [m, n, H]
        gz = GZ[tok].to(dtype)[:, None]
        gch = 2 * (torch.sigmoid(gz + inv[..., 0] * ug + coef[..., 0] * gz) - torch.sigmoid(gz))
        dv = dv + gch[..., None] * VE[tok].to(dtype)[:, None]
    return _score(dr, dv, r0, tok, tables, diag, dtype)


def direct(PJ, R0, CS, SN, GC, VE, tables, start, gated, diag, dtype=torch.float64):
    """(out [m, P], se [m, P, 512]) of readout_kernel (:5906-5965); CS / SN [m, 32] rows of the chunk's tokens."""
    m, P = PJ.shape[:2]
    pj = PJ.to(dtype)
    pk, dv = pj[:, :, 0], pj[:, :, 1]                        # [m, P, H, D]
    c, s = CS.to(dtype)[:, None, None], SN.to(dtype)[:, None, None]
    lo, hi = pk[..., :D // 2], pk[..., D // 2:]
    dr = torch.cat([lo * c + hi * s, -lo * s + hi * c], -1)
    if gated:
        dv = dv + GC.to(dtype)[..., None] * VE.to(dtype)[:, None]
    tok = start + torch.arange(m)
    return _score(dr, dv, R0.to(dtype), tok, tables, diag, dtype)
