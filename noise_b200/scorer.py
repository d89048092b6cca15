"""The true-path readout's scorer (reference train/val/run.py, `readout` section :5900-6040) on libnoise_b200.so.

The reference launches three Triton kernels; these functions take the same arguments (minus the launch-only tile
sizes) and write the same outputs:

- ``stats_kernel(delta, X, SQX, DB, ST, start, n, d_rows, eps)``: bf16 copy of each token's first n move rows and
  their input-RMSNorm statistics (:5968-5988);
- ``staged_kernel(UP, ST, R0, VC, GZ, VE, CS, SN, U, W, M1, M2, QD, GD, AD, CD, VT, OT, out, SE, start, n, se_rows,
  gated, diag, self_edge, nc)``: the rows' scores against block j's future moment tables from the bf16 projection UP
  (:5991-6040);
- ``readout_kernel(PJ, R0, CS, SN, GC, VE, U, W, M1, M2, QD, GD, AD, CD, VT, OT, out, SE, start, probes, gated, diag,
  self_edge)``: the same scores from the projected change itself (:5906-5965).

Tokens of a chunk are the leading dimension of delta / out; the tables are indexed by the global token start + t.
"""
import ctypes

import torch

from . import _lib


def _p(t):
    return None if t is None else t.data_ptr()


def _need(name, t, dtype, shape, contiguous=True):
    """t has `dtype` and `shape` (None: any length of a global-token axis of at least the int that follows it, given
    as (None, n)) and is contiguous: a mismatch raises before a pointer reaches a kernel, which trusts the layout."""
    want = []
    for i, d in enumerate(shape):
        if isinstance(d, tuple):  # (None, at_least)
            if t.dim() <= i or t.shape[i] < d[1]:
                raise ValueError(f'{name}: shape {tuple(t.shape)}, dim {i} must be at least {d[1]}')
            want.append(t.shape[i])
        else:
            want.append(d)
    if tuple(t.shape) != tuple(want) or t.dtype != dtype or (contiguous and not t.is_contiguous()):
        raise ValueError(f'{name}: {t.dtype} {tuple(t.shape)}{"" if t.is_contiguous() else " strided"}, expected '
                         f'{"contiguous " if contiguous else ""}{dtype} {tuple(want)}')


def _tables(U, W, M1, M2, QD, GD, AD, CD, VT, OT, tokens):
    """The block's moment tables over at least `tokens` global tokens (start + the chunk's tokens)."""
    g = (None, tokens)
    f32, bf16 = torch.float32, torch.bfloat16
    for name, z in (('U', U), ('W', W), ('QD', QD), ('GD', GD)):
        _need(name, z, f32, (g, 8, 64))
    for name, z in (('AD', AD), ('CD', CD)):
        _need(name, z, f32, (g, 8))
    for name, z in (('M1', M1), ('M2', M2)):
        _need(name, z, bf16, (g, 8, 64, 64))
    for name, z in (('VT', VT), ('OT', OT)):
        if z is not None:
            _need(name, z, f32, (g, 8, 64))
    tab = _lib.ScorerTables()
    tab.U, tab.W, tab.M1, tab.M2, tab.QD, tab.GD, tab.AD, tab.CD = (z.data_ptr() for z in (U, W, M1, M2, QD, GD, AD,
                                                                                             CD))
    tab.VT, tab.OT = _p(VT), _p(OT)
    return tab, [z for z in (U, W, M1, M2, QD, GD, AD, CD, VT, OT) if z is not None]


def stats_kernel(delta, X, SQX, DB, ST, start, n, d_rows, eps):
    """DB [m, n, 512] bf16, ST [m, n, 2] fp32 for the m tokens of delta [m, d_rows, 512] (written in place)."""
    m, f32 = delta.shape[0], torch.float32
    _need('delta', delta, f32, (m, (None, int(n)), 512))
    if delta.shape[1] != int(d_rows):
        raise ValueError(f'delta: {delta.shape[1]} rows a token, d_rows {d_rows}')
    _need('X', X, f32, ((None, int(start) + m), 512))
    _need('SQX', SQX, f32, ((None, int(start) + m),))
    _need('DB', DB, torch.bfloat16, (m, int(n), 512))
    _need('ST', ST, f32, (m, int(n), 2))
    _lib.require_cuda(delta, X, SQX, DB, ST)
    _lib.check(_lib.lib().noise_readout_stats(delta.data_ptr(), X.data_ptr(), SQX.data_ptr(), DB.data_ptr(),
                                              ST.data_ptr(), int(start), int(n), int(d_rows), m, float(eps),
                                              _lib.stream_handle(delta.device)), 'noise_readout_stats')


def staged_kernel(UP, ST, R0, VC, GZ, VE, CS, SN, U, W, M1, M2, QD, GD, AD, CD, VT, OT, out, SE, start, n, se_rows,
                  gated, diag, self_edge, nc, tc=True):
    """out [m, n] (and SE [m, se_rows, 512] bf16 with self_edge), written in place; m = out.shape[0]. tc=True: the
    moment-table terms on tcgen05 (returns the workspace, whose first int is the device status); tc=False: all on
    the CUDA cores (returns None)."""
    m, n, f32 = out.shape[0], int(n), torch.float32
    g = (None, int(start) + m)
    tab, live = _tables(U, W, M1, M2, QD, GD, AD, CD, VT if self_edge else None, OT if self_edge else None, g[1])
    _need('out', out, f32, (m, n))
    _need('UP', UP, torch.bfloat16, (m * n, int(nc)))
    _need('ST', ST, f32, (m, n, 2))
    _need('R0', R0, f32, (g, 8, 64))
    _need('VC', VC, f32, (g, 512))
    _need('CS', CS, f32, (g, 32))
    _need('SN', SN, f32, (g, 32))
    live += [UP, ST, R0, VC, CS, SN, out]
    if gated:
        _need('GZ', GZ, f32, (g, 8))
        _need('VE', VE, f32, (g, 8, 64))
        live += [GZ, VE]
    if self_edge:
        _need('SE', SE, torch.bfloat16, (m, (None, n), 512))
        if SE.shape[1] != int(se_rows):
            raise ValueError(f'SE: {SE.shape[1]} rows a token, se_rows {se_rows}')
        live.append(SE)
    _lib.require_cuda(*live)
    args = (UP.data_ptr(), ST.data_ptr(), R0.data_ptr(), VC.data_ptr(), _p(GZ) if gated else None,
            _p(VE) if gated else None, CS.data_ptr(), SN.data_ptr(), ctypes.byref(tab), out.data_ptr(),
            _p(SE) if self_edge else None, int(start), int(n), int(se_rows), out.shape[0], int(nc), int(bool(diag)))
    if not tc:
        _lib.check(_lib.lib().noise_readout_staged(*args, _lib.stream_handle(out.device)), 'noise_readout_staged')
        return None
    ws = torch.empty(_lib.STATUS_BYTES, dtype=torch.uint8, device=out.device)
    _lib.check(_lib.lib().noise_readout_staged_ws(*args, ws.data_ptr(), _lib.STATUS_BYTES,
                                                  _lib.stream_handle(out.device)), 'noise_readout_staged_ws')
    return ws


def readout_kernel(PJ, R0, CS, SN, GC, VE, U, W, M1, M2, QD, GD, AD, CD, VT, OT, out, SE, start, probes, gated, diag,
                   self_edge, tc=True):
    """out [m, probes] (and SE [m, probes, 512] bf16 with self_edge), written in place; m = out.shape[0]. tc=True: the
    moment-table terms on tcgen05 (returns the workspace, whose first int is the device status); tc=False: all on the
    CUDA cores (returns None)."""
    m, probes, f32 = out.shape[0], int(probes), torch.float32
    tab, live = _tables(U, W, M1, M2, QD, GD, AD, CD, VT if self_edge else None, OT if self_edge else None,
                        int(start) + m)
    PJ, R0 = PJ.contiguous(), R0.contiguous()
    _need('out', out, f32, (m, probes))
    _need('PJ', PJ, f32, (m, probes, 2, 8, 64))
    _need('R0', R0, f32, (m, 8, 64))
    _need('CS', CS, f32, (m, 32), contiguous=False)  # rows of the chunk's tokens, any strides
    _need('SN', SN, f32, (m, 32), contiguous=False)
    live += [PJ, R0, CS, SN, out]
    if gated:
        GC, VE = GC.contiguous(), VE.contiguous()
        _need('GC', GC, f32, (m, probes, 8))
        _need('VE', VE, f32, (m, 8, 64))
        live += [GC, VE]
    if self_edge:
        _need('SE', SE, torch.bfloat16, (m, probes, 512))
        live.append(SE)
    _lib.require_cuda(*live)
    args = (PJ.data_ptr(), R0.data_ptr(), CS.data_ptr(), CS.stride(0), CS.stride(1), SN.data_ptr(), SN.stride(0),
            SN.stride(1), _p(GC) if gated else None, _p(VE) if gated else None,
            ctypes.byref(tab), out.data_ptr(), _p(SE) if self_edge else None, int(start), int(probes), out.shape[0],
            int(bool(diag)))
    if not tc:
        _lib.check(_lib.lib().noise_readout_direct(*args, _lib.stream_handle(out.device)), 'noise_readout_direct')
        return None
    ws = torch.empty(_lib.STATUS_BYTES, dtype=torch.uint8, device=out.device)
    _lib.check(_lib.lib().noise_readout_direct_ws(*args, ws.data_ptr(), _lib.STATUS_BYTES,
                                                  _lib.stream_handle(out.device)), 'noise_readout_direct_ws')
    return ws
