"""The readout-scorer oracle (oracle/scorer.py) against the reference's own kernels (tests/golden/scorer.pt:
train/val/run.py's `readout` section stats_kernel, staged_kernel, readout_kernel under the patched interpreter)."""
import sys
from pathlib import Path

import torch

from oracle import scorer

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from scorer_inputs import scorer_inputs, tables  # noqa: E402


def _rel(a, r):
    return ((a.double() - r.double()).abs().max() / r.double().abs().max()).item()


def test_stats(golden):
    g, x = golden('scorer.pt'), scorer_inputs()
    db, st = scorer.stats(x['delta'], x['X'], x['SQX'], x['start'], x['n'], x['eps'])
    assert torch.equal(db, g['db'])
    assert _rel(st, g['st']) < 1e-6


def test_staged(golden):
    g, x = golden('scorer.pt'), scorer_inputs()
    out, se = scorer.staged(x['UP'], g['st'], x['R0'], x['VC'], x['GZ'], x['VE'], x['CS'], x['SN'], tables(x),
                            x['start'], x['n'], gated=True, diag=True)
    assert _rel(out, g['staged']) < 1e-5
    ref_se = g['staged_se'][:, :x['n']].float()
    assert (se.float().bfloat16().float() != ref_se).float().mean() < 0.01 and _rel(se, ref_se) < 1e-2


def test_direct(golden):
    g, x = golden('scorer.pt'), scorer_inputs()
    tok = slice(x['start'], x['start'] + x['m'])
    out, se = scorer.direct(x['PJ'], x['R0'][tok], x['CS'][tok], x['SN'][tok], x['GC'], x['VE'][tok], tables(x),
                            x['start'], gated=True, diag=True)
    assert _rel(out, g['direct']) < 1e-5
    assert (se.float().bfloat16().float() != g['direct_se'].float()).float().mean() < 0.01
