"""Parity of the true-path readout's scorer (noise_b200.scorer: the reference's stats_kernel, staged_kernel,
readout_kernel) with the reference's own outputs (tests/golden/scorer.pt) and with the fp64 oracle.

Tolerances: the bf16 copy is exact; fp32 arithmetic in another order: scores within REL of max |ref|; the bf16
self-edge within one rounding on under 1% of elements."""
import sys
from pathlib import Path

import pytest
import torch

from oracle import scorer as oracle

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from scorer_inputs import scorer_inputs, tables  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None
REL = 5e-5


def _rel(a, r):
    a, r = a.double().cpu(), r.double().cpu()
    return ((a - r).abs().max() / r.abs().max()).item()


def _se_ok(a, r):
    a, r = a.cpu().float(), r.cpu().float()
    return (a != r).float().mean() < 0.01 and _rel(a, r) < 1e-2


def _dev(x):
    return {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in x.items()}


def _run(x, gated=True, diag=True, self_edge=True):
    from noise_b200 import scorer
    m, n, d_rows, start, nc = x['m'], x['n'], x['d_rows'], x['start'], x['nc']
    d = _dev(x)
    db = torch.empty(m, n, 512, dtype=torch.bfloat16, device=DEV)
    st = torch.empty(m, n, 2, device=DEV)
    scorer.stats_kernel(d['delta'], d['X'], d['SQX'], db, st, start, n, d_rows, x['eps'])
    out_s = torch.full((m, n), float('nan'), device=DEV)
    se_s = torch.zeros(m, d_rows, 512, dtype=torch.bfloat16, device=DEV)
    scorer.staged_kernel(d['UP'], st, d['R0'], d['VC'], d['GZ'], d['VE'], d['CS'], d['SN'], *tables(d), out_s, se_s,
                         start, n, d_rows, gated, diag, self_edge, nc)
    tok = slice(start, start + m)
    out_d = torch.full((m, n), float('nan'), device=DEV)
    se_d = torch.zeros(m, n, 512, dtype=torch.bfloat16, device=DEV)
    scorer.readout_kernel(d['PJ'], d['R0'][tok], d['CS'][tok], d['SN'][tok], d['GC'], d['VE'][tok], *tables(d),
                          out_d, se_d, start, n, gated, diag, self_edge)
    torch.cuda.synchronize()
    return db.cpu(), st.cpu(), out_s.cpu(), se_s.cpu(), out_d.cpu(), se_d.cpu()


def test_against_reference(golden):
    g, x = golden('scorer.pt'), scorer_inputs()
    db, st, out_s, se_s, out_d, se_d = _run(x)
    assert torch.equal(db, g['db'])
    assert _rel(st, g['st']) < 1e-6
    assert _rel(out_s, g['staged']) < REL and _se_ok(se_s, g['staged_se'])
    assert _rel(out_d, g['direct']) < REL and _se_ok(se_d, g['direct_se'])


@pytest.mark.parametrize('gated,diag,self_edge', [(False, True, False), (True, False, True), (False, False, False)])
def test_variants_against_oracle(gated, diag, self_edge):
    x = scorer_inputs(T=300, start=37, m=5, n=200, d_rows=200, seed=3)
    db, st, out_s, se_s, out_d, se_d = _run(x, gated, diag, self_edge)
    ref_db, ref_st = oracle.stats(x['delta'], x['X'], x['SQX'], x['start'], x['n'], x['eps'])
    assert torch.equal(db, ref_db) and _rel(st, ref_st) < 1e-6
    ref_s, ref_se = oracle.staged(x['UP'], st, x['R0'], x['VC'], x['GZ'], x['VE'], x['CS'], x['SN'], tables(x),
                                  x['start'], x['n'], gated, diag)
    assert _rel(out_s, ref_s) < REL
    tok = slice(x['start'], x['start'] + x['m'])
    ref_d, ref_dse = oracle.direct(x['PJ'], x['R0'][tok], x['CS'][tok], x['SN'][tok], x['GC'], x['VE'][tok],
                                   tables(x), x['start'], gated, diag)
    assert _rel(out_d, ref_d) < REL
    if self_edge:
        assert _se_ok(se_s[:, :x['n']], ref_se.float().bfloat16()) and _se_ok(se_d, ref_dse.float().bfloat16())
    else:
        assert not se_s.float().abs().sum() and not se_d.float().abs().sum()  # nothing written


@pytest.mark.parametrize('gated,diag,self_edge', [(True, True, True), (False, False, False)])
def test_staged_tc_matches_cuda_cores(gated, diag, self_edge):
    """The tcgen05 staged kernel (bf16(dk) M1 / M2 as MMAs over 128 rows of a token) against the all-CUDA-core one on
    three blocks a token, the last partial; the self-edge comes from the same arithmetic, so within one rounding."""
    from noise_b200 import _lib, scorer
    x = scorer_inputs(T=64, start=5, m=4, n=300, d_rows=300, seed=9)
    m, n, start, nc = x['m'], x['n'], x['start'], x['nc']
    d = _dev(x)
    db = torch.empty(m, n, 512, dtype=torch.bfloat16, device=DEV)
    st = torch.empty(m, n, 2, device=DEV)
    scorer.stats_kernel(d['delta'], d['X'], d['SQX'], db, st, start, n, x['d_rows'], x['eps'])
    outs, ses = [], []
    for tc in (True, False):
        out = torch.full((m, n), float('nan'), device=DEV)
        se = torch.zeros(m, n, 512, dtype=torch.bfloat16, device=DEV)
        ws = scorer.staged_kernel(d['UP'], st, d['R0'], d['VC'], d['GZ'], d['VE'], d['CS'], d['SN'], *tables(d), out,
                                  se, start, n, n, gated, diag, self_edge, nc, tc=tc)
        if tc:
            assert _lib.read_status(ws) == 0
        outs.append(out.cpu())
        ses.append(se.cpu())
    assert torch.isfinite(outs[0]).all()
    assert _rel(outs[0], outs[1]) < REL
    assert _se_ok(ses[0], ses[1]) if self_edge else not ses[0].float().abs().sum()


@pytest.mark.parametrize('gated,diag,self_edge', [(True, True, True), (False, True, False)])
def test_direct_tc_matches_cuda_cores(gated, diag, self_edge):
    """The tcgen05 direct (readout_kernel) path against the all-CUDA-core one on three 128-probe blocks a token."""
    from noise_b200 import _lib, scorer
    x = scorer_inputs(T=64, start=5, m=4, n=300, d_rows=300, seed=19)
    m, n, start = x['m'], x['n'], x['start']
    d = _dev(x)
    tok = slice(start, start + m)
    outs, ses = [], []
    for tc in (True, False):
        out = torch.full((m, n), float('nan'), device=DEV)
        se = torch.zeros(m, n, 512, dtype=torch.bfloat16, device=DEV)
        ws = scorer.readout_kernel(d['PJ'], d['R0'][tok], d['CS'][tok], d['SN'][tok], d['GC'], d['VE'][tok],
                                   *tables(d), out, se, start, n, gated, diag, self_edge, tc=tc)
        if tc:
            assert _lib.read_status(ws) == 0
        outs.append(out.cpu())
        ses.append(se.cpu())
    assert torch.isfinite(outs[0]).all()
    assert _rel(outs[0], outs[1]) < REL
    assert _se_ok(ses[0], ses[1]) if self_edge else not ses[0].float().abs().sum()
