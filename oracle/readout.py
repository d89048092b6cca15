"""CPU restatement of the track-1 readout scorers (reference train/val/run.py, `recipe` section) — test
infrastructure only: the checker of noise_b200.readout, never called by the product path.

- ``future_scores``: noise_record::future_scores, whose dense form is joint_scores (run.py:1671-1681).
- ``key_response``: noise_record::key_response (kernel run.py:571-602): the sum runs over each source's window
  (the attention probabilities A vanish outside it at every call site).
- ``query_response``: noise_record::future_query_response (its CPU branch, run.py:1822-1827).
- ``routed_response``: noise_record::routed_response (kernel run.py:548-569; dense form query_change_routed
  :654-660): bf16 operands, both dots' outputs rounded to bf16.
"""
import torch


def _rb(t):
    return t.to(torch.bfloat16).to(t.dtype)


def future_scores(q, target, dk, dv, a, contrast, source_start, window, dtype=torch.float64):
    """[H, P, M]: receivers s of source m with 0 < s - (source_start + m) <= window."""
    q, target, dk, dv, a, contrast = (z.to(dtype) for z in (q, target, dk, dv, a, contrast))
    d = q.shape[-1]
    x = torch.einsum('hsd,hpmd->hpsm', q, dk) * d ** -0.5
    changed = a[:, None] * torch.expm1(x)
    value = torch.einsum('hsd,hpmd->hpsm', target, dv)
    score = (changed * contrast[:, None] + (a[:, None] + changed) * value) / (1 + changed)
    s = torch.arange(q.shape[1])[:, None]
    t = source_start + torch.arange(dk.shape[2])[None]
    allowed = (s > t) & (s - t <= window)
    return (score * allowed).sum(2)


def key_response(q, dk, A, C, source_start, query_start, window, dtype=torch.float64):
    """[H, P, M]: queries at absolute positions query_start + s in [source_start + m, source_start + m + window]."""
    q, dk, A, C = (z.to(dtype) for z in (q, dk, A, C))
    d = q.shape[-1]
    change = A[:, None] * torch.expm1(torch.einsum('hsd,hpmd->hpsm', q, dk) * d ** -0.5)
    s = query_start + torch.arange(q.shape[1])[:, None]
    t = source_start + torch.arange(dk.shape[2])[None]
    allowed = (s >= t) & (s - t <= window)
    return (change / (1 + change) * C[:, None] * allowed).sum(2)


def query_response(dq, keys, values, probabilities, base, dtype=torch.float64):
    """[M, P, H, D]: (sum_k change v_k - partition base) / (1 + partition), change = p (e^(dq . k / sqrt(D)) - 1)."""
    dq, keys, values, probabilities, base = (z.to(dtype) for z in (dq, keys, values, probabilities, base))
    x = torch.einsum('mphd,hsd->mphs', dq, keys) * dq.shape[-1] ** -0.5
    changed = probabilities.permute(1, 0, 2)[:, None] * torch.expm1(x)
    partition = changed.sum(-1, keepdim=True)
    numerator = torch.einsum('mphs,hsd->mphd', changed, values)
    return (numerator - partition * base.transpose(0, 1)[:, None]) / (1 + partition)


def routed_response(dq, keys, values, probabilities, rest):
    """[M, P, H, D] fp32: bf16 operands, fp32 sums, both dots' outputs rounded to bf16 (the reference kernel's)."""
    f = lambda z: z.to(torch.bfloat16).float()
    ds = _rb(torch.einsum('mphd,mhkd->mphk', f(dq), f(keys))) * dq.shape[-1] ** -0.5
    p = probabilities.float().unsqueeze(1)
    dlse = torch.log1p((p * torch.expm1(ds)).sum(-1, keepdim=True))
    weights = _rb(p * torch.expm1(ds - dlse))
    moved = _rb(torch.einsum('mphk,mhkd->mphd', weights, f(values)))
    return moved + torch.expm1(-dlse) * rest.float().unsqueeze(1)
