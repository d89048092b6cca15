"""The identity phase's batched GEMMs (reference train/speedrun/id_kernels.py) on libnoise_b200.so's tcgen05 kernel.

Same names, arguments, results and shape checks as the reference's functions (the ``config`` arguments, the Triton
launch configurations there, are accepted and ignored):

- ``hidden_credits_fused(us, steps, credb, w_out_t)`` -> (L, M, N) bf16: credb @ w_out_t per layer, the bf16 product
  scaled by the relu^2 central-difference slope of the pre-activations us at steps (id_kernels.py:19-84);
- ``square_credit_grads(n1s, got2, out)``: out[j L + l] = n1s[l]^T @ (got2[:, l, j] by token) (:87-133);
- ``at_b_layers(As, Bs, out)``: out[l] = As[l]^T @ Bs[l] (:136-170).
"""
import ctypes

import torch

from . import _lib


def _ptrs(ts, what):
    for t in ts:
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError(f'{what}: contiguous bf16 tensors')
    _lib.require_cuda(*ts)
    return (ctypes.c_void_p * len(ts))(*(t.data_ptr() for t in ts))


def _status(dev):
    return torch.empty(_lib.STATUS_BYTES, dtype=torch.uint8, device=dev)


def hidden_credits_fused(us, steps, credb, w_out_t, config=None):
    """us: eight (.., N) bf16 pre-activations with M rows each, steps (L, M) fp32 (id_kernels.py:73-84)."""
    layers, m, k = credb.shape
    n = w_out_t.shape[-1]
    assert credb.is_contiguous() and w_out_t.is_contiguous() and steps.is_contiguous()
    assert len(us) == layers and all(u.numel() == m * n for u in us)
    assert m % 128 == 0 and n % 128 == 0 and k % 64 == 0
    assert tuple(w_out_t.shape) == (layers, k, n)
    us = [u.detach() for u in us]
    u_ptrs = _ptrs(us, 'us')
    _ptrs([credb, w_out_t], 'credb, w_out_t')
    steps = steps.detach()
    if steps.dtype != torch.float32 or tuple(steps.shape) != (layers, m):
        raise ValueError(f'steps: fp32 ({layers}, {m}), got {steps.dtype} {tuple(steps.shape)}')
    _lib.require_cuda(steps)
    out = torch.empty((layers, m, n), device=credb.device, dtype=torch.bfloat16)
    ws = _status(credb.device)
    _lib.check(_lib.lib().noise_hidden_credits(u_ptrs, steps.data_ptr(), credb.data_ptr(), w_out_t.data_ptr(), layers,
                                               m, n, k, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                               _lib.stream_handle(credb.device)), 'noise_hidden_credits')
    out._noise_workspace = ws
    return out


def square_credit_grads(n1s, got2, out, config=None):
    """out (3L, D, W * HD) bf16 contiguous view: out[j * L + l] = n1s[l]^T @ (got2[:, l, j] by token); n1s: eight
    (M, D) bf16 matrices (id_kernels.py:121-133)."""
    layers, (m, d) = len(n1s), n1s[0].shape
    world, _, three, _, hd = got2.shape
    assert three == 3 and world * hd == d and out.shape == (3 * layers, d, d) and out.is_contiguous()
    assert got2.is_contiguous() and m % 64 == 0 and d % 128 == 0
    assert all(tuple(x.shape) == (m, d) for x in n1s) and got2.shape[1] == layers and got2.shape[3] == m
    if hd != 64:
        raise ValueError('square_credit_grads: head_dim 64')
    a = _ptrs([x.detach() for x in n1s], 'n1s')
    _ptrs([got2, out], 'got2, out')
    ws = _status(out.device)
    _lib.check(_lib.lib().noise_square_credit_grads(a, got2.data_ptr(), world, layers, m, d, out.data_ptr(),
                                                    ws.data_ptr(), ws.numel(), _lib.stream_handle(out.device)),
               'noise_square_credit_grads')
    out._noise_workspace = ws
    return out


def at_b_layers(As, Bs, out, config=None):
    """out[l] = As[l]^T @ Bs[l] (bf16 out, fp32 accumulation) for eight (K, P) / (K, Q) bf16 matrices each (any
    leading shape flattened to K rows) (id_kernels.py:159-170)."""
    p, q = As[0].shape[-1], Bs[0].shape[-1]
    k = As[0].numel() // p
    assert out.shape == (8, p, q) and out.is_contiguous() and all(b.numel() == k * q for b in Bs)
    assert len(As) == len(Bs) == out.shape[0]
    assert all(a.numel() == k * p for a in As) and k % 64 == 0 and p % 128 == 0 and q % 128 == 0
    a = _ptrs([x.detach() for x in As], 'As')
    b = _ptrs([x.detach() for x in Bs], 'Bs')
    _ptrs([out], 'out')
    ws = _status(out.device)
    _lib.check(_lib.lib().noise_at_b_layers(a, b, len(As), k, p, q, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                            _lib.stream_handle(out.device)), 'noise_at_b_layers')
    out._noise_workspace = ws
    return out
