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


def _head_case():
    from dust_inputs import head_error_inputs
    return head_error_inputs()


def test_head_error_against_reference(golden):
    """Same draws (the seeded generator, in the reference's order) on the GPU: within 1e-2 of max |ref| with under 2%
    of elements off by a bf16 rounding of the draw contraction; untouched slabs stay zero."""
    from noise_b200 import dust
    h = _head_case()
    noise = h['noise']
    err = dust.head_error(h['raw'].to(DEV), h['y'].to(DEV), h['clean_loss'].to(DEV), h['draws'], h['sigma'],
                          h['nrep'], lambda *s: noise(*s).to(DEV)).cpu()
    ref = golden('dust.pt')['head_error']
    touched = ref.shape[-1]
    assert not err[..., touched:].any()
    assert _rel(err[..., :touched], ref) < 1e-2
    assert (err[..., :touched] - ref).abs().gt(1e-2 * ref.abs().max()).float().mean() < 0.02


def test_head_error_install_and_oracle():
    """install(DUST) routes a DUST-like instance's head_error here; 96 draws of 12 per chunk (8 slabs) against the
    oracle with the same draws."""
    import types
    from noise_b200 import dust
    h = _head_case()
    draws, nrep = 96, 12
    g = torch.Generator().manual_seed(99)
    drawn = []

    def noise(*shape, dtype=None):
        a = torch.randn(*shape, generator=g).bfloat16()
        drawn.append(a)
        return a.to(DEV)

    class Dust:
        def head_error(self, draws, sigma=0.1):
            raise AssertionError('not installed')
    dust.install(Dust)
    inst = Dust()
    inst.outputs = {'lm_head': h['raw'].to(DEV)}
    inst.y, inst.clean_loss = h['y'].to(DEV), h['clean_loss'].to(DEV)
    inst.recipe, inst.noise = types.SimpleNamespace(nrep=nrep), noise
    inst.model = types.SimpleNamespace(config=types.SimpleNamespace(vocab_size=4096))
    err = inst.head_error(draws, 0.1).cpu()
    ref = oracle.head_error(h['raw'], h['y'], h['clean_loss'], drawn, 0.1)
    assert _rel(err, ref) < 1e-2
