"""Dense CPU restatements of the credit-readout kernels (reference ``train/speedrun/moment_kernels.py``) — test
infrastructure only.

All inputs are stacked rows ``[rows, T, 64]`` (a row is one head of one layer of one sequence). Receiver/query s and
key t interact iff 0 <= s - t <= window (the reference's causal left window, moment_kernels.py:100, 514, 632).
Functions compute in ``dtype`` (float64 by default); the ``emulate`` switches reproduce the reference kernels'
bf16 operand roundings where they exist.
"""
import torch

SCALE = 0.125  # 1 / sqrt(64)


def _allowed(length, window):
    t = torch.arange(length)
    lag = t[:, None] - t[None, :]           # [query s, key t] = s - t
    return (lag >= 0) & (lag <= window)


def _rb(t):
    return t.to(torch.bfloat16).to(t.dtype)


def implicit_key_context(q, k, values, hub, window, dtype=torch.float64):
    """Per query s: lse_s = logsumexp_t q_s.k_t / 8 and center_s = sum_t p(s, t) (hub_s . v_t) over the window
    (moment_kernels.py:80-110, 137-194). Returns (lse, center) [rows, T]."""
    q, k, values, hub = (z.to(dtype) for z in (q, k, values, hub))
    logits = (q @ k.transpose(-1, -2)) * SCALE
    logits = logits.masked_fill(~_allowed(q.shape[1], window), float('-inf'))
    lse = torch.logsumexp(logits, -1)
    p = torch.exp(logits - lse[..., None])
    scores = hub @ values.transpose(-1, -2)
    return lse, (p * scores).sum(-1)


def probabilities(q, k, lse, window, dtype=torch.float64):
    """p[row, s, t] = exp(q_s.k_t / 8 - lse_s) inside the window, 0 outside."""
    q, k, lse = (z.to(dtype) for z in (q, k, lse))
    logits = (q @ k.transpose(-1, -2)) * SCALE
    p = torch.exp(logits - lse[..., None])
    return p.masked_fill(~_allowed(q.shape[1], window), 0.0)


def value_pass(q, k, lse, source, window, dtype=torch.float64, emulate=False):
    """out_t = sum_{s: 0 <= s - t <= window} exp(q_s.k_t / 8 - lse_s) source_s (moment_kernels.py:612-661).

    emulate=True reproduces the Triton kernel's operands: p rounded to bf16 and source split into bf16 hi + lo, the
    two products accumulated in fp32 (moment_kernels.py:633-637)."""
    p = probabilities(q, k, lse, window, dtype)
    src = source.to(dtype)
    if emulate:
        p = _rb(p.float()).to(dtype)
        hi = _rb(source.float())
        lo = _rb(source.float() - hi)
        return p.transpose(-1, -2) @ hi.to(dtype) + p.transpose(-1, -2) @ lo.to(dtype)
    return p.transpose(-1, -2) @ src


def _interleave(x, y):
    """[..., J] x2 -> [..., 2J] with (x_i, y_i) adjacent: Triton's reshape(join(x, y), (.., 2J))."""
    return torch.stack([x, y], -1).flatten(-2)


def _pair_xy(z, scale):
    """x_i = z[..., i] * scale, y_i = z[..., i + D/2] * scale for the D/2 rotary pairs."""
    half = z.shape[-1] // 2
    return z[..., :half] * scale, z[..., half:] * scale


def key_perturbation_geometry(k_raw, cos, sin, sigma, dtype=torch.float64):
    """(ca, bu, bw, step) [rows, T, 64] of a finite step sigma * rms(k_raw) along each raw key coordinate through RoPE
    and the RMS norm (moment_kernels.py:467-480). cos, sin: [T, 32]."""
    raw = k_raw.to(dtype)
    d = raw.shape[-1]
    sq = raw.square().sum(-1, keepdim=True) / d
    step = sigma * sq.sqrt().clamp(min=1e-6)
    ratio = (2 * step * raw + step * step) / d / (sq + 1.1920928955078125e-07)
    ca = torch.expm1(-0.5 * torch.log1p(ratio))
    cb = step * torch.rsqrt(sq + 1.1920928955078125e-07) * (1 + ca)
    cs, sn = cos.to(dtype).repeat(1, 2), sin.to(dtype).repeat(1, 2)
    first = torch.arange(d) < d // 2
    bu = cb * torch.where(first, cs, sn)
    bw = cb * torch.where(first, -sn, cs)
    return ca, bu, bw, step.expand_as(raw)


def _by_pair(m, d):
    """Moment sums over pair features [.., 2J] interleaved (x, y) -> (px, py) gathered per raw direction d (pair
    d % J): [.., D] each."""
    j = m.shape[-1] // 2
    px, py = m[..., 0::2], m[..., 1::2]
    idx = torch.arange(d) % j
    return px[..., idx], py[..., idx]


def key_scan(qp, kp, k_raw, lse, values, hub, center, cos, sin, window, sigma, with_values=False,
             dtype=torch.float64, emulate=False):
    """Key credits of every key t and raw key coordinate d: the degree-2 moment response of the receivers' softmax to
    a finite step of k_raw[t, d] (moment_kernels.py:483-558). Receivers s: 0 <= s - t <= window.
    Returns key [rows, T, 64] (and the raw value credit sum_s p hub with with_values).

    emulate=True rounds the moment dots' operands to bf16 as the Triton kernel does (w1, w2, w2 * logit and the pair
    features; the value credit's p and hub hi/lo)."""
    rows, t, d = k_raw.shape
    qp, kp, values, hub = (z.to(dtype) for z in (qp, kp, values, hub))
    lse, center = lse.to(dtype), center.to(dtype)
    logit = (kp @ qp.transpose(-1, -2)) * d ** -0.5                    # [row, t (key), s (receiver)]
    lag = torch.arange(t)[None, :] - torch.arange(t)[:, None]          # s - t
    valid = (lag >= 0) & (lag <= window)
    score = values @ hub.transpose(-1, -2)
    c = torch.where(valid, score - center[:, None, :], 0.0)
    a = torch.where(valid, torch.exp(logit - lse[:, None, :]), 0.0)
    x, y = _pair_xy(qp, d ** -0.5)
    f2, g2, xy = _interleave(x, y), _interleave(x * x, y * y), x * y
    w1, w2 = a * c, (0.5 * a - a * a) * c
    w2l = w2 * logit
    r = (lambda z: _rb(z.float()).to(dtype)) if emulate else (lambda z: z)
    p2, q2 = r(w1) @ r(f2), r(w2) @ r(g2)
    qxy, r2 = r(w2) @ r(xy), r(w2l) @ r(f2)
    s1, s2 = (w1 * logit).sum(-1, keepdim=True), (w2 * logit * logit).sum(-1, keepdim=True)
    ca, bu, bw, step = key_perturbation_geometry(k_raw, cos, sin, sigma, dtype)
    px, py = _by_pair(p2, d)
    qx, qy = _by_pair(q2, d)
    rx, ry = _by_pair(r2, d)
    qxy = qxy[..., torch.arange(d) % (d // 2)]
    response = (px * bu + py * bw + qx * bu * bu + qy * bw * bw + 2 * qxy * bu * bw + 2 * ca * (rx * bu + ry * bw)
                + s1 * ca + s2 * ca * ca)
    key = response / step
    if not with_values:
        return key
    if emulate:
        pb = _rb(a.float()).to(dtype)
        hi = _rb(hub.float())
        lo = _rb(hub.float() - hi)
        return key, pb @ hi.to(dtype) + pb @ lo.to(dtype)
    return key, a @ hub


def query_coefficients(raw, sq, steps, cos, sin, dtype=torch.float64):
    """(ca, bu, bw) [rows, T, 64] of a finite step `steps` of each raw coordinate through RoPE and the RMS norm
    (moment_kernels.py:199-214): raw [rows, T, 64], sq / steps [rows, T], cos / sin [T, 32]."""
    raw, sq, steps = raw.to(dtype), sq.to(dtype)[..., None], steps.to(dtype)[..., None]
    d = raw.shape[-1]
    change = (2 * steps * raw + steps * steps) / d / (sq / d + 1e-6)
    a = torch.expm1(-0.5 * torch.log1p(change))
    b = steps * torch.rsqrt(sq / d + 1e-6) * (1 + a)
    cs, sn = cos.to(dtype).repeat(1, 2), sin.to(dtype).repeat(1, 2)
    first = torch.arange(d) < d // 2
    return a, b * torch.where(first, cs, sn), b * torch.where(first, -sn, cs)


def moment_query_scores(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, window, dtype=torch.float64,
                        emulate=False):
    """Query credits z [rows, T, 64] of every query s and raw query coordinate: numerator / denominator degree-2
    moments of its own softmax under a finite coordinate step (moment_kernels.py:231-316). Keys t: 0 <= s - t <=
    window. side: the keys whose pair features enter the moments (kp at the reference's call site).
    emulate=True rounds the moment dots' operands to bf16 (wn, a, wn * logit, a * logit, pair features)."""
    rows, t, d = q.shape
    q, k, v, hub, side = (z.to(dtype) for z in (q, k, v, hub, side))
    lse, hub_out = lse.to(dtype), hub_out.to(dtype)
    logits = (q @ k.transpose(-1, -2)) * d ** -0.5                     # [row, s (query), t (key)]
    lag = torch.arange(t)[:, None] - torch.arange(t)[None, :]          # s - t
    valid = (lag >= 0) & (lag <= window)
    c = hub @ v.transpose(-1, -2) - hub_out[..., None]
    a = torch.where(valid, torch.exp(logits - lse[..., None]), 0.0)
    x, y = _pair_xy(side, d ** -0.5)
    r = (lambda z: _rb(z.float()).to(dtype)) if emulate else (lambda z: z)
    fx, fy, fxx, fyy, fxy = r(x), r(y), r(x * x), r(y * y), r(x * y)
    wn = a * c
    wnl, al = r(wn * logits), r(a * logits)
    wnb, ab = r(wn), r(a)
    nx0, ny0, nx1, ny1, nxy = wnb @ fx, wnb @ fy, wnb @ fxx, wnb @ fyy, wnb @ fxy
    dx0, dy0, dx1, dy1, dxy = ab @ fx, ab @ fy, ab @ fxx, ab @ fyy, ab @ fxy
    lx0, ly0, mx0, my0 = wnl @ fx, wnl @ fy, al @ fx, al @ fy
    s1n, s2n = (wn * logits).sum(-1, keepdim=True), (wn * logits * logits).sum(-1, keepdim=True)
    s1d, s2d = (a * logits).sum(-1, keepdim=True), (a * logits * logits).sum(-1, keepdim=True)
    ca, bu, bw = query_coefficients(raw, sq, steps, cos, sin, dtype)
    g = lambda z: z[..., torch.arange(d) % (d // 2)]
    nx0, ny0, nx1, ny1, nxy, dx0, dy0, dx1, dy1, dxy, lx0, ly0, mx0, my0 = map(
        g, (nx0, ny0, nx1, ny1, nxy, dx0, dy0, dx1, dy1, dxy, lx0, ly0, mx0, my0))
    zn = (nx0 * bu + ny0 * bw + 0.5 * (nx1 * bu * bu + ny1 * bw * bw) + nxy * bu * bw + ca * (lx0 * bu + ly0 * bw)
          + s1n * ca + s2n * (0.5 * ca * ca))
    zd = (dx0 * bu + dy0 * bw + 0.5 * (dx1 * bu * bu + dy1 * bw * bw) + dxy * bu * bw + ca * (mx0 * bu + my0 * bw)
          + s1d * ca + s2d * (0.5 * ca * ca))
    return zn / (1.0 + zd) / steps.to(dtype)[..., None]


def moment_key_scores(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, dtype=torch.float64,
                      emulate=False):
    """Identity-phase key credits and value sums of every key t (moment_kernels.py:370-433): receivers s >= t (full
    causal), moments of w1 = a c, w2 = (a / 2 - a^2) c over the receivers' pair features (side = the queries'),
    combined with the key's own step coefficients. Returns (out, values) [rows, T, 64]."""
    rows, t, d = q.shape
    q, k, v, hub, side = (z.to(dtype) for z in (q, k, v, hub, side))
    lse, hub_out = lse.to(dtype), hub_out.to(dtype)
    logits = (k @ q.transpose(-1, -2)) * d ** -0.5                     # [row, t (key), s (receiver)]
    lag = torch.arange(t)[None, :] - torch.arange(t)[:, None]          # s - t
    a = torch.where(lag >= 0, torch.exp(logits - lse[:, None, :]), 0.0)
    c = v @ hub.transpose(-1, -2) - hub_out[:, None, :]
    x, y = _pair_xy(side, d ** -0.5)
    r = (lambda z: _rb(z.float()).to(dtype)) if emulate else (lambda z: z)
    f2, g2, xy = r(_interleave(x, y)), r(_interleave(x * x, y * y)), r(x * y)
    w1, w2 = a * c, (0.5 * a - a * a) * c
    values = r(a) @ (r(hub) if emulate else hub)
    p2, q2, qxy, r2 = r(w1) @ f2, r(w2) @ g2, r(w2) @ xy, r(w2 * logits) @ f2
    s1, s2 = (w1 * logits).sum(-1, keepdim=True), (w2 * logits * logits).sum(-1, keepdim=True)
    ca, bu, bw = query_coefficients(raw, sq, steps, cos, sin, dtype)
    px, py = _by_pair(p2, d)
    qx, qy = _by_pair(q2, d)
    rx, ry = _by_pair(r2, d)
    qxy = qxy[..., torch.arange(d) % (d // 2)]
    z = (px * bu + py * bw + qx * bu * bu + qy * bw * bw + qxy * (2.0 * bu * bw) + 2.0 * ca * (rx * bu + ry * bw)
         + s1 * ca + s2 * (ca * ca))
    return z / steps.to(dtype)[..., None], values
