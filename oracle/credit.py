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
