"""Drop-in track-1 readout scorers (reference train/val/run.py, `recipe` section) on libnoise_b200.so.

Same names, arguments and results as the reference's custom ops:

- ``future_scores(q, target, dk, dv, a, contrast, source_start, window)`` -> [H, P, M]   (noise_record::future_scores)
- ``key_response(q, dk, A, C, source_start, query_start, window)`` -> [H, P, M]          (noise_record::key_response)
- ``query_response(dq, keys, values, probabilities, base)`` -> [M, P, H, D]    (noise_record::future_query_response)
- ``routed_response(dq, keys, values, probabilities, rest)`` -> [M, P, H, D]          (noise_record::routed_response)

Each is also registered as a ``torch.library.custom_op`` (namespace ``noise_b200``) with a fake. ``install(R)``
registers these implementations as the CUDA kernels of the record module's own ops, the seam the reference's
``fast_kernels.install`` uses (``op.register_kernel('cuda', impl)``, run.py:3440-3453), so R's callers run them
unchanged. head_dim 64. future_scores, key_response and query_response run their dots on tcgen05 at the reference's
tf32x3 precision, routed_response its bf16 dots as kind::f16 MMAs; each keeps its fp32 CUDA-core form as tc=False.
"""
import ctypes

import torch

from . import _lib

HD = 64


def _view(t):
    t = t.detach()
    if t.dtype != torch.float32:
        t = t.float()
    if t.dim() != 3:
        raise ValueError('a 3-D tensor')
    v = _lib.View3()
    v.data = t.data_ptr()
    v.stride0, v.stride1, v.stride2 = t.stride()
    return v, t


def _f32c(t):
    return t.detach().to(torch.float32).contiguous()


def _check(rc, what):
    _lib.check(rc, what)


def _shapes(**named):
    """Each keyword is (tensor, expected shape): a mismatch raises before any pointer reaches a kernel, which would
    otherwise read past a smaller operand's end."""
    for name, (t, want) in named.items():
        if tuple(t.shape) != tuple(want):
            raise ValueError(f'{name}: shape {tuple(t.shape)}, expected {tuple(want)}')


def _stream(t):
    return _lib.stream_handle(t.device)


def future_scores_impl(q, target, dk, dv, a, contrast, source_start, window, tc=True):
    """tc=True: the tcgen05 kernel at the reference's tf32x3 precision (its workspace, whose first int is the device
    status, rides on the output as ``_noise_workspace``); tc=False: the fp32 CUDA-core kernel, for comparison."""
    h, p, m, d = dk.shape
    if d != HD:
        raise ValueError('head_dim 64 only')
    t = q.shape[1]
    _shapes(q=(q, (h, t, d)), target=(target, (h, t, d)), dv=(dv, (h, p, m, d)), a=(a, (h, t, m)),
            contrast=(contrast, (h, t, m)))
    _lib.require_cuda(q, target, dk, dv, a, contrast)
    (qv, q), (gv, target), (av, a), (cv, contrast) = _view(q), _view(target), _view(a), _view(contrast)
    dk, dv = _f32c(dk), _f32c(dv)
    out = torch.empty((h, p, m), device=q.device, dtype=torch.float32)
    L = _lib.lib()
    args = (ctypes.byref(qv), ctypes.byref(gv), dk.data_ptr(), dv.data_ptr(), ctypes.byref(av), ctypes.byref(cv), h, t,
            p, m, int(source_start), int(window), out.data_ptr())
    if not tc:
        _check(L.noise_future_scores(*args, _stream(q)), 'noise_future_scores')
        return out
    nbytes = L.noise_future_scores_workspace_bytes(h, t)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    _check(L.noise_future_scores_ws(*args, ws.data_ptr(), nbytes, _stream(q)), 'noise_future_scores_ws')
    out._noise_workspace = ws
    return out


def key_response_impl(q, dk, A, C, source_start, query_start, window, tc=True):
    """tc=True: the tcgen05 kernel at the reference's tf32x3 precision (workspace on ``_noise_workspace``); tc=False:
    the fp32 CUDA-core kernel, for comparison."""
    heads, probes, sources, width = dk.shape
    if width != HD:
        raise ValueError('head_dim 64 only')
    t = q.shape[1]
    _shapes(q=(q, (heads, t, width)), A=(A, (heads, t, sources)), C=(C, (heads, t, sources)))
    _lib.require_cuda(q, dk, A, C)
    (qv, q), (av, A), (cv, C) = _view(q), _view(A), _view(C)
    dk = _f32c(dk)
    out = torch.empty((heads, probes, sources), device=q.device, dtype=torch.float32)
    L = _lib.lib()
    args = (ctypes.byref(qv), dk.data_ptr(), ctypes.byref(av), ctypes.byref(cv), heads, t, probes, sources,
            int(source_start), int(query_start), int(window), out.data_ptr())
    if not tc:
        _check(L.noise_key_response(*args, _stream(q)), 'noise_key_response')
        return out
    nbytes = L.noise_key_response_workspace_bytes(heads, t)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    _check(L.noise_key_response_ws(*args, ws.data_ptr(), nbytes, _stream(q)), 'noise_key_response_ws')
    out._noise_workspace = ws
    return out


def query_response_impl(dq, keys, values, probabilities, base, tc=True):
    """tc=True: the tcgen05 kernel at the reference's tf32x3 precision (its workspace, whose first int is the device
    status, rides on the output as ``_noise_workspace``); tc=False: the fp32 CUDA-core kernel, for comparison."""
    m, p, h, d = dq.shape
    if d != HD:
        raise ValueError('head_dim 64 only')
    t = keys.shape[1]
    _shapes(keys=(keys, (h, t, d)), values=(values, (h, t, d)), probabilities=(probabilities, (h, m, t)),
            base=(base, (h, m, d)))
    _lib.require_cuda(dq, keys, values, probabilities, base)
    dq = _f32c(dq)
    (kv, keys), (vv, values), (pv, probabilities), (bv, base) = (_view(z) for z in (keys, values, probabilities,
                                                                                   base))
    out = torch.empty((m, p, h, d), device=dq.device, dtype=torch.float32)
    L = _lib.lib()
    if not tc:
        _check(L.noise_query_response(dq.data_ptr(), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(pv),
                                      ctypes.byref(bv), m, p, h, t, out.data_ptr(), _stream(dq)), 'noise_query_response')
        return out
    nbytes = L.noise_query_response_workspace_bytes(m, p, h, t)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dq.device)
    _check(L.noise_query_response_ws(dq.data_ptr(), ctypes.byref(kv), ctypes.byref(vv), ctypes.byref(pv),
                                     ctypes.byref(bv), m, p, h, t, out.data_ptr(), ws.data_ptr(), nbytes, _stream(dq)),
           'noise_query_response_ws')
    out._noise_workspace = ws
    return out


def routed_response_impl(dq, keys, values, probabilities, rest, tc=True):
    """tc=True: the tcgen05 kernel (its status workspace rides on the output as ``_noise_workspace``); tc=False:
    the CUDA-core kernel, for comparison."""
    m, probes, heads, width = dq.shape
    if width != HD:
        raise ValueError('head_dim 64 only')
    count = keys.shape[2]
    _shapes(keys=(keys, (m, heads, count, width)), values=(values, (m, heads, count, width)),
            probabilities=(probabilities, (m, heads, count)), rest=(rest, (m, heads, width)))
    _lib.require_cuda(dq, keys, values, probabilities, rest)
    dq, keys, values = (z.detach().to(torch.bfloat16).contiguous() for z in (dq, keys, values))
    probabilities, rest = _f32c(probabilities), _f32c(rest)
    out = torch.empty((m, probes, heads, width), device=dq.device, dtype=torch.float32)
    args = (dq.data_ptr(), keys.data_ptr(), values.data_ptr(), probabilities.data_ptr(), rest.data_ptr(), m, probes,
            heads, count, out.data_ptr())
    if not tc:
        _check(_lib.lib().noise_routed_response(*args, _stream(dq)), 'noise_routed_response')
        return out
    ws = torch.empty(_lib.STATUS_BYTES, dtype=torch.uint8, device=dq.device)
    _check(_lib.lib().noise_routed_response_ws(*args, ws.data_ptr(), _lib.STATUS_BYTES, _stream(dq)),
           'noise_routed_response_ws')
    out._noise_workspace = ws
    return out


@torch.library.custom_op('noise_b200::future_scores', mutates_args=())
def future_scores(q: torch.Tensor, target: torch.Tensor, dk: torch.Tensor, dv: torch.Tensor, a: torch.Tensor,
                  contrast: torch.Tensor, source_start: int, window: int) -> torch.Tensor:
    """noise_record::future_scores (run.py:1729-1745): [H, P, M] fp32."""
    return future_scores_impl(q, target, dk, dv, a, contrast, source_start, window)


@future_scores.register_fake
def _(q, target, dk, dv, a, contrast, source_start, window):
    return torch.empty(dk.shape[:-1], device=q.device, dtype=torch.float32)


@torch.library.custom_op('noise_b200::key_response', mutates_args=())
def key_response(q: torch.Tensor, dk: torch.Tensor, A: torch.Tensor, C: torch.Tensor, source_start: int,
                 query_start: int, window: int) -> torch.Tensor:
    """noise_record::key_response (run.py:622-632): [H, P, M] fp32."""
    return key_response_impl(q, dk, A, C, source_start, query_start, window)


@key_response.register_fake
def _(q, dk, A, C, source_start, query_start, window):
    return torch.empty(dk.shape[:3], device=q.device, dtype=torch.float32)


@torch.library.custom_op('noise_b200::query_response', mutates_args=())
def query_response(dq: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, probabilities: torch.Tensor,
                   base: torch.Tensor) -> torch.Tensor:
    """noise_record::future_query_response (run.py:1818-1834): [M, P, H, D] fp32."""
    return query_response_impl(dq, keys, values, probabilities, base)


@query_response.register_fake
def _(dq, keys, values, probabilities, base):
    return torch.empty(dq.shape, device=dq.device, dtype=torch.float32)


@torch.library.custom_op('noise_b200::routed_response', mutates_args=())
def routed_response(dq: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, probabilities: torch.Tensor,
                    rest: torch.Tensor) -> torch.Tensor:
    """noise_record::routed_response (run.py:604-619): [M, P, H, D] fp32."""
    return routed_response_impl(dq, keys, values, probabilities, rest)


@routed_response.register_fake
def _(dq, keys, values, probabilities, rest):
    return torch.empty(dq.shape, device=dq.device, dtype=torch.float32)


def install(R):
    """Register these kernels as the CUDA implementations of the record module R's ops (R.fused_scores,
    R.fused_key_response, R.query_response, R.routed_response), as the reference's fast_kernels.install registers its
    own (run.py:3440-3453). Returns R."""
    for op, impl in ((R.fused_scores, future_scores_impl), (R.fused_key_response, key_response_impl),
                     (R.query_response, query_response_impl), (R.routed_response, routed_response_impl)):
        op.register_kernel('cuda', impl)
    return R
