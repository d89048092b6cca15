"""The identity phase's readout cycle (reference train/speedrun/run.py:3569-3686) on libnoise_b200.so.

Same names, arguments and results as the reference's functions:

- ``coordinate_change(raw, targets)`` -> [n, 4096]: the LM head's finite coordinate change (run.py:3569-3577);
- ``cycle_weights_fused(x, base, h)`` -> (fg1, fast, rows, total, steps, inv, inv0, delta, sigma) (run.py:3636-3647);
- ``top_credit(model, x, y)`` -> [n, 512]: the readout cycle's credit of the final stream (run.py:3673-3686).

The per-logit weights, the finish and coordinate_change are this library's kernels; the five bf16 moment GEMMs run on
its tcgen05 GEMM, and the fp32 contractions (x W, h W, x h^T, fg1 c^T and the final one with h) on the same GEMM at
tf32, the precision the reference runs them at (torch.set_float32_matmul_precision('high'), run.py:4447). The GEMM
takes both operands K-major, so W and h are transposed once per call where they are the right-hand side.
"""
import ctypes

import torch

from . import _lib

D, VOCAB, SOFTCAP = 512, 4096, 15.0
SIGMA, HEAD_SIGMA, SEED = 0.005, 0.1, 0  # run.py's SIGMA, HEAD_SIGMA, SEED


def step_signs(step_t, device):
    """+-1 [512] for the update step: the reference's integer hash of (step, column) (run.py:3580-3589)."""
    x = (step_t.to(torch.int64) * 0x9E3779B1 + torch.arange(D, device=device, dtype=torch.int64) * 0x85EBCA77
         + SEED) & 0xFFFFFFFF
    x = x ^ (x >> 15)
    x = (x * 0x2C1B3C6D) & 0xFFFFFFFF
    x = x ^ (x >> 12)
    x = (x * 0x297A2D39) & 0xFFFFFFFF
    x = x ^ (x >> 15)
    return 1.0 - 2.0 * (x & 1).float()


def coordinate_change(raw, targets):
    """[n, 4096] fp32: (log1p(w expm1(up - z)) - log1p(w expm1(down - z)) - onehot (up - down)) / (2 HEAD_SIGMA)."""
    raw = raw.detach()
    if raw.dtype not in (torch.float32, torch.bfloat16):
        raw = raw.float()
    raw = raw.contiguous()
    targets = targets.detach().long().contiguous()
    _lib.require_cuda(raw, targets)
    rows = raw.shape[0]
    if raw.shape[-1] != VOCAB or targets.numel() != rows:
        raise ValueError('raw [n, 4096], targets [n]')
    out = torch.empty(rows, VOCAB, device=raw.device, dtype=torch.float32)
    _lib.check(_lib.lib().noise_coordinate_change(raw.data_ptr(), 1 if raw.dtype == torch.bfloat16 else 0,
                                                  targets.data_ptr(), rows, HEAD_SIGMA, out.data_ptr(),
                                                  _lib.stream_handle(raw.device)), 'noise_coordinate_change')
    return out


def _weights(x, base, y):
    n = x.shape[0]
    if (tuple(x.shape) != (n, D) or tuple(base.shape) != (n, VOCAB) or tuple(y.shape) != (n,)
            or x.dtype != torch.float32 or base.dtype != torch.float32 or y.dtype != torch.int64
            or not (x.is_contiguous() and base.is_contiguous() and y.is_contiguous())):
        raise ValueError(f'x fp32 [n, {D}], base fp32 [n, {VOCAB}] and y int64 [n], contiguous: got '
                         f'{tuple(x.shape)}, {tuple(base.shape)}, {tuple(y.shape)}')
    _lib.require_cuda(x, base, y)
    dev = x.device
    fg1 = torch.empty(n, VOCAB, device=dev)
    fast = torch.empty(5, n, VOCAB, device=dev, dtype=torch.bfloat16)
    rows = torch.empty(n, 3, device=dev)
    total, sq, base_y = (torch.empty(n, device=dev) for _ in range(3))
    _lib.check(_lib.lib().noise_cycle_weights(x.data_ptr(), base.data_ptr(), y.data_ptr(), n, fg1.data_ptr(),
                                              fast.data_ptr(), rows.data_ptr(), total.data_ptr(), sq.data_ptr(),
                                              base_y.data_ptr(), _lib.stream_handle(dev)), 'noise_cycle_weights')
    return fg1, fast, rows, total, sq, base_y


def cycle_weights_fused(x, base, h):
    """The readout cycle's weights (run.py:3636-3647): fg1 [n, V], fast bf16 [5, n, V], rows [n, 3], total [n, 1] and
    cycle_scales' steps, inv, inv0, delta, sigma."""
    x, base = x.detach().float().contiguous(), base.detach().float().contiguous()
    y = torch.zeros(x.shape[0], dtype=torch.int64, device=x.device)
    fg1, fast, rows, total, sq, _ = _weights(x, base, y)
    sq = sq[:, None]
    steps = SIGMA * torch.clamp(torch.sqrt(sq / D), min=1e-6)
    dots = _lib.gemm_tf32_tn(x, h.detach().float())
    eps = torch.finfo(torch.float32).eps
    inv = torch.rsqrt((sq + 2 * steps * dots + steps * steps * D) / D + eps)
    inv0 = torch.rsqrt(sq / D + eps)
    return fg1, fast, rows, total[:, None], steps, inv, inv0, inv / inv0 - 1, steps * inv


def top_credit(model, x, y):
    """[n, 512]: the readout cycle's credit of the final stream x [n, 512] for targets y [n] (run.py:3673-3686);
    model carries H (the 512 x 512 Hadamard basis), step_t and lm_head [512, 4096] fp32."""
    x = x.detach().float().contiguous()
    y = y.detach().long().contiguous()
    if x.dim() != 2 or x.shape[1] != D or tuple(y.shape) != (x.shape[0],):
        raise ValueError(f'x [n, {D}] and y [n]: got {tuple(x.shape)}, {tuple(y.shape)}')
    _lib.require_cuda(x, y)
    h = (model.H * step_signs(model.step_t, x.device)[None, :]).float().contiguous()
    Wt = model.lm_head.float().t().contiguous()  # [4096, 512]: W as the K-major right-hand side
    c = _lib.gemm_tf32_tn(h, Wt)                 # h W
    base = _lib.gemm_tf32_tn(x, Wt)              # x W
    fg1, fast, rows, total, sq, base_y = _weights(x, base, y)
    exact = _lib.gemm_tf32_tn(fg1, c)            # fg1 c^T
    dots = _lib.gemm_tf32_tn(x, h)               # x h^T
    n, R = x.shape[0], c.shape[0]
    powers = (c.bfloat16(), (c * c).bfloat16(), (c * c * c).bfloat16())
    prods = torch.empty(5, n, R, device=x.device)
    for k, p in enumerate((0, 0, 1, 1, 2)):  # fast_k against c, c, c^2, c^2, c^3 (run.py:3681-3685)
        _lib.gemm_bf16_tn(fast[k], powers[p], prods[k])
    out = torch.empty(n, R, device=x.device)
    _lib.check(_lib.lib().noise_cycle_finish(dots.data_ptr(), sq.data_ptr(), exact.data_ptr(), prods.data_ptr(),
                                             rows.data_ptr(), total.data_ptr(), base_y.data_ptr(), c.data_ptr(),
                                             y.data_ptr(), n, R, SIGMA, out.data_ptr(), _lib.stream_handle(x.device)),
               'noise_cycle_finish')
    return _lib.gemm_tf32_tn(out, h.t().contiguous()).div_(D)  # out h / D
