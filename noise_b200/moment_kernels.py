"""Drop-in credit-readout ops (reference train/speedrun/moment_kernels.py) on the sm_100a kernels of
libnoise_b200.so.

Same function names, arguments, shapes and results as the reference module; each is also registered as a
``torch.library.custom_op`` (namespace ``noise_b200``) with a fake implementation, so they stay usable under
``torch.compile`` and CUDA-graph capture (no host synchronisation, outputs from the caching allocator).
``key_scan`` / ``value_pass`` have the signatures of the reference's ``KEY_IMPL`` / ``VALUE_IMPL`` plug-in seams
(moment_kernels.py:642-650), so run.py:1678-1681 can install them in place of the Gluon kernels.
"""
import ctypes

import torch

from . import _lib

F32, BF16 = 0, 1
_DT = {torch.float32: F32, torch.bfloat16: BF16}


def _rows(t, heads=1, layers=None):
    """noise_rows_t of a [rows, T, 64] stacked view (heads = 1) or a (layers, T, heads * 64) by-token view."""
    if t.stride(-1) != 1:
        raise ValueError('credit views need a unit last stride')
    m = _lib.Rows()
    m.data = t.data_ptr()
    m.layer_stride, m.token_stride = t.stride(0), t.stride(1)
    m.heads = heads
    m.layer_map = layers.data_ptr() if layers is not None else None
    return m


def _stream(t):
    return _lib.stream_handle(t.device)


def _c(t, dtype=None):
    t = t.detach()
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def _check(rc, what):
    _lib.check(rc, what)


def _rope(cos, sin, t):
    """fp32 contiguous RoPE tables holding 32 values for each of the t positions the kernels read."""
    cos, sin = _c(cos, torch.float32), _c(sin, torch.float32)
    for name, z in (('cos', cos), ('sin', sin)):
        if z.shape[-1] != 32 or z.numel() < 32 * t:
            raise ValueError(f'{name}: 32 values for each of {t} positions, got {tuple(z.shape)}')
    return cos, sin


def _shapes(**named):
    """Each keyword is (tensor, expected shape; None where any extent goes, (None, n) for at least n): a mismatch
    raises before a pointer reaches a kernel, which would otherwise read past a smaller operand's end."""
    for name, (t, want) in named.items():
        ok = t.dim() == len(want)
        for got, w in zip(t.shape, want):
            ok = ok and (w is None or (got >= w[1] if isinstance(w, tuple) else got == w))
        if not ok:
            raise ValueError(f'{name}: shape {tuple(t.shape)}, expected {want}')


def _on_device(*ts):
    _lib.require_cuda(*(z for z in ts if z is not None))


def _layer_map(layers, groups):
    """The int32 layer map of a by-token output: one entry per row group, on the device."""
    if layers is not None and (layers.dtype != torch.int32 or layers.numel() < groups):
        raise ValueError(f'layers: int32 with at least {groups} entries')


# --- lse and center -----------------------------------------------------------------------------------------------

def implicit_key_context_edges_impl(q, k, values, hub, window, tc=True):
    """(lse, center); bf16 operands with T % 128 == 0 on the tcgen05 kernel (``tc=False``: the warp-MMA kernel, for
    comparison), the workspace's status word riding on lse."""
    h, t, _ = q.shape
    _shapes(q=(q, (h, t, 64)), k=(k, (h, t, 64)), values=(values, (h, t, 64)), hub=(hub, (h, t, 64)))
    dt = torch.bfloat16 if q.dtype == torch.bfloat16 else torch.float32
    q, k, values, hub = (_c(z, dt) for z in (q, k, values, hub))
    _on_device(q, k, values, hub)
    lse = torch.empty((h, t), device=q.device, dtype=torch.float32)
    center = torch.empty_like(lse)
    if tc and dt == torch.bfloat16 and t % 128 == 0:
        ws = torch.empty(_lib.STATUS_BYTES, dtype=torch.uint8, device=q.device)
        _check(_lib.lib().noise_implicit_key_context_ws(q.data_ptr(), k.data_ptr(), values.data_ptr(), hub.data_ptr(),
                                                        _DT[dt], h, t, window, lse.data_ptr(), center.data_ptr(),
                                                        ws.data_ptr(), ws.numel(), _stream(q)),
               'noise_implicit_key_context_ws')
        lse._noise_workspace = ws
        return lse, center
    _check(_lib.lib().noise_implicit_key_context(q.data_ptr(), k.data_ptr(), values.data_ptr(), hub.data_ptr(),
                                                 _DT[dt], h, t, window, lse.data_ptr(), center.data_ptr(),
                                                 _stream(q)), 'noise_implicit_key_context')
    return lse, center


# --- value credits --------------------------------------------------------------------------------------------------

def value_pass(q, k, lse, source, window, in_heads=1, out_heads=1, out=None, layers=None, tc=True):
    """sum_s p * source (moment_kernels._value_pass): source stacked (rows, T, C) or (in_heads > 1) by token
    (rows // in_heads, T, in_heads * C); the output stacked or (out_heads > 1) by token, into ``out`` when given.
    The signature of the reference's VALUE_IMPL plug-in. bf16 q / k with T % 128 == 0 run on the tcgen05 kernel
    (``tc=False``: the warp-MMA kernel, for comparison); the workspace's status word rides on ``out``."""
    h, t, _ = q.shape
    _shapes(q=(q, (h, t, 64)), k=(k, (h, t, 64)), lse=(lse, (h, t)))
    if h % in_heads or h % out_heads:
        raise ValueError(f'{h} rows do not split into groups of {in_heads} / {out_heads} heads')
    dt = torch.bfloat16 if q.dtype == torch.bfloat16 else torch.float32
    q, k, lse = _c(q, dt), _c(k, dt), _c(lse, torch.float32)
    if source.dtype != torch.float32 or source.stride(-1) != 1:
        source = source.float().contiguous()
    channels = source.shape[-1] // in_heads
    if channels != 64:
        raise ValueError('the value pass runs 64 channels per head')
    _shapes(source=(source, ((None, h // in_heads), (None, t), in_heads * 64)))
    if out is None:
        out = source.new_empty((h // out_heads, t, out_heads * channels), dtype=torch.float32)
    _shapes(out=(out, (None if layers is not None else (None, h // out_heads), (None, t), out_heads * 64)))
    if out.dtype != torch.float32:
        raise ValueError('out: fp32')
    _layer_map(layers, h // out_heads)
    _on_device(q, k, lse, source, out, layers)
    src_rows = _rows(source, in_heads)
    out_rows = _rows(out, out_heads, layers)
    if tc and dt == torch.bfloat16 and t % 128 == 0:
        L = _lib.lib()
        nbytes = L.noise_value_pass_workspace_bytes(h, t)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        _check(L.noise_value_pass_ws(q.data_ptr(), k.data_ptr(), _DT[dt], lse.data_ptr(), ctypes.byref(src_rows),
                                     ctypes.byref(out_rows), h, t, window, ws.data_ptr(), nbytes, _stream(q)),
               'noise_value_pass_ws')
        out._noise_workspace = ws
        return out
    _check(_lib.lib().noise_value_pass(q.data_ptr(), k.data_ptr(), _DT[dt], lse.data_ptr(), ctypes.byref(src_rows),
                                       ctypes.byref(out_rows), h, t, window, _stream(q)), 'noise_value_pass')
    return out


# --- key credits ----------------------------------------------------------------------------------------------------

def key_scan(qp, kp, k_raw, lse, values, hub, center, cos, sin, window, sigma, with_values=False, out_heads=1, key=None,
             layers=None, tc=True):
    """The key credits (and with_values the raw value credits), stacked (rows, T, D) or by token
    (rows // out_heads, T, out_heads * D), into ``key`` when given (moment_kernels._key_scan). The signature of the
    reference's KEY_IMPL plug-in; returns (key, raw_value) (raw_value is key when with_values is False). T % 128 == 0
    runs on the tcgen05 kernel (``tc=False``: the warp-MMA kernel, for comparison); its workspace rides on the key
    output as ``_noise_workspace``."""
    h, t, d = k_raw.shape
    full = (h, t, 64)
    _shapes(k_raw=(k_raw, full), qp=(qp, full), kp=(kp, full), values=(values, full), hub=(hub, full),
            lse=(lse, (h, t)), center=(center, (h, t)))
    if h % out_heads:
        raise ValueError(f'{h} rows do not split into groups of {out_heads} heads')
    qp, kp, k_raw, values, hub = (_c(z, torch.float32) for z in (qp, kp, k_raw, values, hub))
    lse, center = _c(lse, torch.float32), _c(center, torch.float32)
    cos, sin = _rope(cos, sin, t)
    shape = (h // out_heads, t, out_heads * d)
    key = qp.new_empty(shape) if key is None else key
    _shapes(key=(key, (None if layers is not None else (None, h // out_heads), (None, t), out_heads * d)))
    if key.dtype != torch.float32:
        raise ValueError('key: fp32')
    _layer_map(layers, h // out_heads)
    _on_device(qp, kp, k_raw, lse, values, hub, center, cos, sin, key, layers)
    raw_value = qp.new_empty(shape) if with_values else None
    key_rows = _rows(key, out_heads, layers)
    val_rows = _rows(raw_value, out_heads, layers) if with_values else _lib.Rows()
    ws = None
    if tc and t % 128 == 0:
        L = _lib.lib()
        nbytes = L.noise_key_scan_workspace_bytes(h, t)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=qp.device)
        _check(L.noise_key_scan_ws(qp.data_ptr(), kp.data_ptr(), k_raw.data_ptr(), lse.data_ptr(), values.data_ptr(),
                                   hub.data_ptr(), center.data_ptr(), cos.data_ptr(), sin.data_ptr(), h, t, window,
                                   float(sigma), ctypes.byref(key_rows), ctypes.byref(val_rows), ws.data_ptr(), nbytes,
                                   _stream(qp)), 'noise_key_scan_ws')
    else:
        _check(_lib.lib().noise_key_scan(qp.data_ptr(), kp.data_ptr(), k_raw.data_ptr(), lse.data_ptr(),
                                         values.data_ptr(), hub.data_ptr(), center.data_ptr(), cos.data_ptr(),
                                         sin.data_ptr(), h, t, window, float(sigma), ctypes.byref(key_rows),
                                         ctypes.byref(val_rows), _stream(qp)), 'noise_key_scan')
    k_out = key.view(h, t, d) if out_heads == 1 and layers is None else key
    if ws is not None:
        key._noise_workspace = k_out._noise_workspace = ws
    if not with_values:
        return k_out, k_out
    return k_out, raw_value.view(h, t, d) if out_heads == 1 else raw_value


# --- query and key moments ------------------------------------------------------------------------------------------

def _blocked(t, rows, m, blocks, tokens):
    """noise_rows_t of one of the reference's strided 4-D raw / out arguments (G, blocks, M, >= 64): row r, token s
    at (r // (rows // blocks)) * stride(1) + (n // m) * stride(0) + (n % m) * stride(2), n = (r % (rows // blocks)) *
    T + s (moment_kernels.py:200-220: RAW_BLK, RAW_GPU, RAW_STRIDE, M). (1, rows, T, 64) is the stacked layout; the
    identity phase passes its (W, L, N, 322) received buffer and (W, L, N, 64) slices of the return buffer."""
    if t.dim() != 4 or t.stride(-1) != 1:
        raise ValueError('raw / out: 4-D with a unit last stride')
    if rows % blocks:
        raise ValueError('rows must split evenly over raw.shape[1] blocks')
    if t.shape[1] < blocks or t.shape[2] < m or t.shape[3] < 64 or t.shape[0] * m < rows // blocks * tokens:
        raise ValueError(f'raw / out {tuple(t.shape)}: too small for {rows} rows x {tokens} tokens in {blocks} blocks '
                         f'of {m} tokens a GPU')
    v = _lib.Rows()
    v.data = t.data_ptr()
    v.heads = 1
    v.block_rows = rows // blocks
    v.layer_stride, v.gpu_stride, v.token_stride = t.stride(1), t.stride(0), t.stride(2)
    v.per_gpu = m
    return v


def _raw4(raw, rows, t):
    raw = raw.detach()
    if raw.dim() == 3:
        raw = raw.unsqueeze(0)
    if raw.dtype not in _DT:
        raw = raw.float()
    return raw


def moment_query_scores_impl(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, out, window=None, out_heads=0,
                             layers=None, tc=True):
    """The query credits into out; T % 128 == 0 runs on the tcgen05 kernel when the output view allows 16-byte
    stores (``tc=False``: the warp-MMA kernel, for comparison). Returns the workspace (its first int is the device
    status word) or None."""
    rows, t, d = q.shape
    if d != 64:
        raise ValueError('head_dim 64 only (the reference asserts it)')
    if side is None:
        raise ValueError("side (the keys' fp32 pair-feature source) is required")
    full = (rows, t, 64)
    _shapes(k=(k, full), v=(v, full), hub=(hub, full), side=(side, full), sq=(sq, (rows, t)), steps=(steps, (rows, t)),
            lse=(lse, (rows, t)), hub_out=(hub_out, (rows, t)))
    q, k, v, hub = (_c(z, torch.bfloat16) for z in (q, k, v, hub))
    raw = _raw4(raw, rows, t)
    side = _c(side, torch.float32)
    sq, steps, lse, hub_out = (_c(z, torch.float32) for z in (sq, steps, lse, hub_out))
    cos, sin = _rope(cos, sin, t)
    window = t if window is None else min(window, t)
    blocks = raw.shape[1]
    if out_heads:  # a (layers, T, heads * D) fp32 view, by token
        if rows % out_heads or out.dtype != torch.float32:
            raise ValueError(f'by-token out: fp32, {rows} rows in groups of {out_heads} heads')
        _shapes(out=(out, (None if layers is not None else (None, rows // out_heads), (None, t), out_heads * 64)))
        _layer_map(layers, rows // out_heads)
        o, dt, m = _rows(out, out_heads, layers), F32, t
    else:  # the reference's 4-D out: (1, rows, T, D) bf16, or the identity phase's (W, L, N, D) slice
        if out.dtype not in _DT:
            raise ValueError('out: fp32 or bf16')
        m = out.shape[2]
        o, dt = _blocked(out, rows, m, blocks, t), _DT[out.dtype]
    rv = _blocked(raw, rows, m, blocks, t)
    _on_device(q, k, v, hub, raw, side, sq, steps, lse, hub_out, cos, sin, out, layers)
    if tc and t % 128 == 0:
        L = _lib.lib()
        nbytes = L.noise_moment_query_scores_workspace_bytes(rows, t)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        _check(L.noise_moment_query_scores_ws(q.data_ptr(), k.data_ptr(), v.data_ptr(), hub.data_ptr(),
                                              ctypes.byref(rv), _DT[raw.dtype], sq.data_ptr(), side.data_ptr(),
                                              cos.data_ptr(), sin.data_ptr(), lse.data_ptr(), hub_out.data_ptr(),
                                              steps.data_ptr(), rows, t, window, ctypes.byref(o), dt, ws.data_ptr(),
                                              nbytes, _stream(q)), 'noise_moment_query_scores_ws')
        return ws
    _check(_lib.lib().noise_moment_query_scores_v(q.data_ptr(), k.data_ptr(), v.data_ptr(), hub.data_ptr(),
                                                  ctypes.byref(rv), _DT[raw.dtype], sq.data_ptr(), side.data_ptr(),
                                                  cos.data_ptr(), sin.data_ptr(), lse.data_ptr(), hub_out.data_ptr(),
                                                  steps.data_ptr(), rows, t, window, ctypes.byref(o), dt, _stream(q)),
           'noise_moment_query_scores_v')
    return None


def moment_key_scores_impl(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, out, values, tc=True):
    """The identity phase's key moments into out / values; T % 128 == 0 runs on the tcgen05 kernel when the output
    views allow 16-byte stores (``tc=False``: the warp-MMA kernel, for comparison). Returns the workspace (its first
    int is the device status word) or None."""
    rows, t, d = q.shape
    full = (rows, t, 64)
    _shapes(q=(q, full), k=(k, full), v=(v, full), hub=(hub, full), side=(side, full), sq=(sq, (rows, t)),
            steps=(steps, (rows, t)), lse=(lse, (rows, t)), hub_out=(hub_out, (rows, t)))
    q, k, v, hub = (_c(z, torch.bfloat16) for z in (q, k, v, hub))
    raw = _raw4(raw, rows, t)
    side = _c(side, torch.float32)
    sq, steps, lse, hub_out = (_c(z, torch.float32) for z in (sq, steps, lse, hub_out))
    cos, sin = _rope(cos, sin, t)
    if out.dim() == 3:
        out, values = out.unsqueeze(0), values.unsqueeze(0)
    if values.shape != out.shape or values.stride() != out.stride() or values.dtype != out.dtype:
        raise ValueError('out and values: same shape, strides and dtype (the reference asserts it)')
    if out.dtype not in _DT:
        raise ValueError('out / values: fp32 or bf16')
    blocks, m = raw.shape[1], out.shape[2]
    rv, ro, rvals = (_blocked(z, rows, m, blocks, t) for z in (raw, out, values))
    _on_device(q, k, v, hub, raw, side, sq, steps, lse, hub_out, cos, sin, out, values)
    if tc and t % 128 == 0:
        L = _lib.lib()
        nbytes = L.noise_moment_key_scores_workspace_bytes(rows, t)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
        _check(L.noise_moment_key_scores_ws(q.data_ptr(), k.data_ptr(), v.data_ptr(), hub.data_ptr(), ctypes.byref(rv),
                                            _DT[raw.dtype], sq.data_ptr(), side.data_ptr(), cos.data_ptr(),
                                            sin.data_ptr(), lse.data_ptr(), hub_out.data_ptr(), steps.data_ptr(), rows,
                                            t, ctypes.byref(ro), ctypes.byref(rvals), _DT[out.dtype], ws.data_ptr(),
                                            nbytes, _stream(q)), 'noise_moment_key_scores_ws')
        return ws
    _check(_lib.lib().noise_moment_key_scores_v(q.data_ptr(), k.data_ptr(), v.data_ptr(), hub.data_ptr(),
                                                ctypes.byref(rv), _DT[raw.dtype], sq.data_ptr(), side.data_ptr(),
                                                cos.data_ptr(), sin.data_ptr(), lse.data_ptr(), hub_out.data_ptr(),
                                                steps.data_ptr(), rows, t, ctypes.byref(ro), ctypes.byref(rvals),
                                                _DT[out.dtype], _stream(q)),
           'noise_moment_key_scores_v')
    return None


# --- the reference's custom ops (names as in moment_kernels.py:184-717) ---------------------------------------------

@torch.library.custom_op('noise_b200::implicit_key_context_edges', mutates_args=())
def implicit_key_context_edges(q: torch.Tensor, k: torch.Tensor, values: torch.Tensor, hub: torch.Tensor,
                               window: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(lse, center) [rows, T] of the windowed softmax q k^T / 8 (moment_kernels.py:184-188)."""
    return implicit_key_context_edges_impl(q, k, values, hub, window)


@implicit_key_context_edges.register_fake
def _(q, k, values, hub, window):
    h, t, _ = q.shape
    return q.new_empty((h, t), dtype=torch.float32), q.new_empty((h, t), dtype=torch.float32)


@torch.library.custom_op('noise_b200::key_credits', mutates_args=())
def key_credits(qp: torch.Tensor, kp: torch.Tensor, k_raw: torch.Tensor, lse: torch.Tensor, values: torch.Tensor,
                hub: torch.Tensor, center: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, window: int,
                sigma: float) -> torch.Tensor:
    """batched_key_scores' key scan (moment_kernels.py:582-587)."""
    return key_scan(qp, kp, k_raw, lse, values, hub, center, cos, sin, window, sigma, False)[0]


@key_credits.register_fake
def _(qp, kp, k_raw, lse, values, hub, center, cos, sin, window, sigma):
    return torch.empty_like(k_raw, dtype=torch.float32)


@torch.library.custom_op('noise_b200::key_credits_into', mutates_args=('out',))
def key_credits_into(qp: torch.Tensor, kp: torch.Tensor, k_raw: torch.Tensor, lse: torch.Tensor, values: torch.Tensor,
                     hub: torch.Tensor, center: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, window: int,
                     sigma: float, out: torch.Tensor, layers: torch.Tensor | None = None) -> None:
    """key_credits_by_token into out, a (layers, T, heads * D) view with last stride 1 (moment_kernels.py:595-602)."""
    key_scan(qp, kp, k_raw, lse, values, hub, center, cos, sin, window, sigma, False, out.shape[-1] // k_raw.shape[-1],
             out, layers)


@key_credits_into.register_fake
def _(qp, kp, k_raw, lse, values, hub, center, cos, sin, window, sigma, out, layers=None):
    return None


@torch.library.custom_op('noise_b200::key_and_raw_value_credits', mutates_args=())
def key_and_raw_value_credits(qp: torch.Tensor, kp: torch.Tensor, k_raw: torch.Tensor, lse: torch.Tensor,
                              values: torch.Tensor, hub: torch.Tensor, center: torch.Tensor, cos: torch.Tensor,
                              sin: torch.Tensor, window: int, sigma: float) -> tuple[torch.Tensor, torch.Tensor]:
    """The key scan with the raw value credit sum_s p hub in the same pass (moment_kernels.py:17)."""
    key, raw = key_scan(qp, kp, k_raw, lse, values, hub, center, cos, sin, window, sigma, True)
    return key, raw


@key_and_raw_value_credits.register_fake
def _(qp, kp, k_raw, lse, values, hub, center, cos, sin, window, sigma):
    return torch.empty_like(k_raw, dtype=torch.float32), torch.empty_like(k_raw, dtype=torch.float32)


@torch.library.custom_op('noise_b200::raw_value_credits', mutates_args=())
def raw_value_credits(q: torch.Tensor, k: torch.Tensor, lse: torch.Tensor, hub: torch.Tensor,
                      window: int) -> torch.Tensor:
    """sum_s p * hub for (heads, tokens, 64) inputs (moment_kernels.py:664-668)."""
    return value_pass(q, k, lse, hub, window)


@raw_value_credits.register_fake
def _(q, k, lse, hub, window):
    return torch.empty_like(hub, dtype=torch.float32)


@torch.library.custom_op('noise_b200::terminal_value_credits', mutates_args=())
def terminal_value_credits(q: torch.Tensor, k: torch.Tensor, lse: torch.Tensor, corrected: torch.Tensor,
                           window: int) -> torch.Tensor:
    """sum_s p * corrected (moment_kernels.py:676-680)."""
    return value_pass(q, k, lse, corrected.contiguous(), window)


@terminal_value_credits.register_fake
def _(q, k, lse, corrected, window):
    return torch.empty_like(corrected, dtype=torch.float32)


@torch.library.custom_op('noise_b200::raw_value_credits_by_token', mutates_args=())
def raw_value_credits_by_token(q: torch.Tensor, k: torch.Tensor, lse: torch.Tensor, hub: torch.Tensor, window: int,
                               heads: int) -> torch.Tensor:
    """raw_value_credits as (layers, T, heads * 64) (moment_kernels.py:693-698)."""
    return value_pass(q, k, lse, hub, window, 1, heads)


@raw_value_credits_by_token.register_fake
def _(q, k, lse, hub, window, heads):
    rows, t, d = hub.shape
    return hub.new_empty((rows // heads, t, heads * d), dtype=torch.float32)


@torch.library.custom_op('noise_b200::terminal_value_credits_into', mutates_args=('out',))
def terminal_value_credits_into(q: torch.Tensor, k: torch.Tensor, lse: torch.Tensor, corrected: torch.Tensor,
                                window: int, out: torch.Tensor, layers: torch.Tensor | None = None) -> None:
    """terminal_value_credits_by_token into out (moment_kernels.py:706-712)."""
    heads = corrected.shape[-1] // q.shape[-1]
    value_pass(q, k, lse, corrected, window, heads, heads, out, layers)


@terminal_value_credits_into.register_fake
def _(q, k, lse, corrected, window, out, layers=None):
    return None


@torch.library.custom_op('noise_b200::moment_query_scores', mutates_args=('out',))
def moment_query_scores(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, hub: torch.Tensor, raw: torch.Tensor,
                        sq: torch.Tensor, side: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, lse: torch.Tensor,
                        hub_out: torch.Tensor, steps: torch.Tensor, out: torch.Tensor, repeat: int,
                        window: int | None = None) -> None:
    """Query credits into the reference's (1, rows, T, D) bf16 out (moment_kernels.py:338-343)."""
    if repeat != 4 or q.shape[-1] != 64:
        raise ValueError('the reference call (repeat = head_dim // 16, head_dim 64)')
    moment_query_scores_impl(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, out, window)


@moment_query_scores.register_fake
def _(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, out, repeat, window=None):
    return None


@torch.library.custom_op('noise_b200::moment_query_scores_into', mutates_args=('out',))
def moment_query_scores_into(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, hub: torch.Tensor, raw: torch.Tensor,
                             sq: torch.Tensor, side: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                             lse: torch.Tensor, hub_out: torch.Tensor, steps: torch.Tensor, out: torch.Tensor,
                             window: int | None = None, layers: torch.Tensor | None = None) -> None:
    """Query credits by token into out, a (layers, T, heads * D) fp32 view (moment_kernels.py:351-360)."""
    moment_query_scores_impl(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, out, window,
                             out.shape[-1] // q.shape[-1], layers)


@moment_query_scores_into.register_fake
def _(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, out, window=None, layers=None):
    return None


@torch.library.custom_op('noise_b200::moment_key_scores', mutates_args=('out', 'values'))
def moment_key_scores(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, hub: torch.Tensor, raw: torch.Tensor,
                      sq: torch.Tensor, side: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, lse: torch.Tensor,
                      hub_out: torch.Tensor, steps: torch.Tensor, out: torch.Tensor, values: torch.Tensor,
                      repeat: int) -> None:
    """The identity phase's key credits and value sums (moment_kernels.py:451-457); out / values fp32 or bf16,
    (rows, T, 64) or the reference's 4-D layouts (its (W, L, N, 64) return-buffer slices included)."""
    if repeat != 2 or q.shape[-1] != 64:
        raise ValueError("the identity phase's call (repeat = head_dim // 32, head_dim 64)")
    moment_key_scores_impl(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, out, values)


@moment_key_scores.register_fake
def _(q, k, v, hub, raw, sq, side, cos, sin, lse, hub_out, steps, out, values, repeat):
    return None


KEY_IMPL = key_scan      # run.py:1678-1679 installs these in the reference module
VALUE_IMPL = value_pass
