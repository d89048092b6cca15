"""Parity of Dust's jittered block rerun (noise_b200.dust.block_forward) with the oracle at the population forward's
rounding points and with the reference's fp32 block_forward (tests/golden/dust.pt).

Tolerances: against the autocast oracle within AUTOCAST_REL of max |ref| (q, k, v and the attention output are bf16
in the kernels where the oracle attends in fp32); against the reference's fp32 within FP32_REL (bf16 linears)."""
import sys
from pathlib import Path

import pytest
import torch

from oracle import dust as oracle

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from dust_inputs import dust_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None
AUTOCAST_REL = 1e-2
FP32_REL = 2e-2


def _rel(a, r):
    a, r = a.double().cpu(), r.double().cpu()
    return ((a - r).abs().max() / r.abs().max()).item()


def _dev(d):
    return {k: v.to(DEV) for k, v in d.items()}


def _run(x, w, ve, window, jitter):
    from noise_b200 import dust
    return dust.block_forward(x['x'].to(DEV), _dev(w), None if ve is None else ve.to(DEV), x['cos'].to(DEV),
                              x['sin'].to(DEV), window, **_dev(jitter)).cpu()


def test_against_reference(golden):
    g, x = golden('dust.pt'), dust_inputs()
    assert _rel(_run(x, x['w'], x['ve'], x['windows'][0], x['jitter']), g['gated']) < FP32_REL
    assert _rel(_run(x, x['plain'], None, x['windows'][1], {}), g['plain']) < FP32_REL


@pytest.mark.parametrize('sites', [('o',), ('attn',), ('fc',), ('mlp',), ('o', 'attn', 'fc', 'mlp')])
def test_each_site_against_oracle(sites):
    x = dust_inputs(B=3, T=384, seed=7, sigma=0.2)
    jit = {s: x['jitter'][s] for s in sites}
    got = _run(x, x['w'], x['ve'], 256, jit)
    ref = oracle.block_forward(x['x'], x['w'], x['ve'], x['cos'], x['sin'], 256, **jit)
    assert _rel(got, ref) < AUTOCAST_REL
    # the jitter moves the output: the site is wired
    clean = oracle.block_forward(x['x'], x['w'], x['ve'], x['cos'], x['sin'], 256)
    assert _rel(got, clean) > 10 * _rel(got, ref)
