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


def _tables(U, W, M1, M2, QD, GD, AD, CD, VT, OT):
    for z in (U, W, QD, GD, AD, CD):
        if z.dtype != torch.float32 or not z.is_contiguous():
            raise ValueError('U, W, QD, GD, AD, CD: contiguous fp32')
    for z in (M1, M2):
        if z.dtype != torch.bfloat16 or not z.is_contiguous():
            raise ValueError('M1, M2: contiguous bf16')
    tab = _lib.ScorerTables()
    tab.U, tab.W, tab.M1, tab.M2, tab.QD, tab.GD, tab.AD, tab.CD = (z.data_ptr() for z in (U, W, M1, M2, QD, GD, AD,
                                                                                             CD))
    tab.VT, tab.OT = _p(VT), _p(OT)
    return tab


def stats_kernel(delta, X, SQX, DB, ST, start, n, d_rows, eps):
    """DB [m, n, 512] bf16, ST [m, n, 2] fp32 for the m tokens of delta [m, d_rows, 512] (written in place)."""
    m = delta.shape[0]
    _lib.require_cuda(delta, X, SQX, DB, ST)
    _lib.check(_lib.lib().noise_readout_stats(delta.data_ptr(), X.data_ptr(), SQX.data_ptr(), DB.data_ptr(),
                                              ST.data_ptr(), int(start), int(n), int(d_rows), m, float(eps),
                                              _lib.stream_handle(delta.device)), 'noise_readout_stats')


def staged_kernel(UP, ST, R0, VC, GZ, VE, CS, SN, U, W, M1, M2, QD, GD, AD, CD, VT, OT, out, SE, start, n, se_rows,
                  gated, diag, self_edge, nc, tc=True):
    """out [m, n] (and SE [m, se_rows, 512] bf16 with self_edge), written in place; m = out.shape[0]. tc=True: the
    moment-table terms on tcgen05 (returns the workspace, whose first int is the device status); tc=False: all on
    the CUDA cores (returns None)."""
    tab = _tables(U, W, M1, M2, QD, GD, AD, CD, VT if self_edge else None, OT if self_edge else None)
    _lib.require_cuda(UP, ST, R0, VC, CS, SN, out)
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
    tab = _tables(U, W, M1, M2, QD, GD, AD, CD, VT if self_edge else None, OT if self_edge else None)
    PJ, R0 = PJ.contiguous(), R0.contiguous()
    _lib.require_cuda(PJ, R0, CS, SN, out)
    args = (PJ.data_ptr(), R0.data_ptr(), CS.data_ptr(), CS.stride(0), CS.stride(1), SN.data_ptr(), SN.stride(0),
            SN.stride(1), _p(GC.contiguous()) if gated else None, _p(VE.contiguous()) if gated else None,
            ctypes.byref(tab), out.data_ptr(), _p(SE) if self_edge else None, int(start), int(probes), out.shape[0],
            int(bool(diag)))
    if not tc:
        _lib.check(_lib.lib().noise_readout_direct(*args, _lib.stream_handle(out.device)), 'noise_readout_direct')
        return None
    ws = torch.empty(_lib.STATUS_BYTES, dtype=torch.uint8, device=out.device)
    _lib.check(_lib.lib().noise_readout_direct_ws(*args, ws.data_ptr(), _lib.STATUS_BYTES,
                                                  _lib.stream_handle(out.device)), 'noise_readout_direct_ws')
    return ws
