"""Parity of the track-1 readout scorers (noise_b200.readout) with the reference's own ops (tests/golden/readout.pt)
and with the fp64 oracle at larger sizes, and the install() seam.

Tolerances: fp32 arithmetic in another order than the reference's tf32x3 dots: max |diff| within REL of max |ref|;
routed_response rounds both dots' outputs to bf16, so a sum in another order flips an occasional rounding: ROUTED_REL,
with under 1% of elements off by more than 1e-3 of the scale."""
import sys
from pathlib import Path

import pytest
import torch

from oracle import readout as oracle

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from readout_inputs import future_inputs, key_inputs, query_inputs, routed_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None
REL = 2e-5
ROUTED_REL = 1e-2


def _rel(a, r):
    a, r = a.double().cpu(), r.double().cpu()
    return ((a - r).abs().max() / r.abs().max()).item()


def _routed_ok(got, ref):
    got, ref = got.cpu().float(), ref.cpu().float()
    return _rel(got, ref) < ROUTED_REL and (got - ref).abs().gt(1e-3 * ref.abs().max()).float().mean() < 0.01


def _dev(d):
    return {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}


def _future(f):
    from noise_b200 import readout
    return readout.future_scores(f['q'], f['target'], f['dk'], f['dv'], f['a'], f['contrast'], f['source_start'],
                                 f['window'])


def _key(k):
    from noise_b200 import readout
    return readout.key_response(k['q'], k['dk'], k['A'], k['C'], k['source_start'], k['query_start'], k['window'])


def _query(q):
    from noise_b200 import readout
    return readout.query_response(q['dq'], q['keys'], q['values'], q['probabilities'], q['base'])


def _routed(r):
    from noise_b200 import readout
    return readout.routed_response(r['dq'], r['keys'], r['values'], r['probabilities'], r['rest'])


def test_against_reference(golden):
    g = golden('readout.pt')
    assert _rel(_future(_dev(future_inputs())), g['future']) < REL
    assert _rel(_key(_dev(key_inputs())), g['key']) < REL
    assert _rel(_query(_dev(query_inputs())), g['query']) < REL
    assert _routed_ok(_routed(_dev(routed_inputs())), g['routed'])


def test_future_scores_larger():
    f = future_inputs(h=8, t=1024, p=8, m=128, source_start=256, window=512, seed=3)
    ref = oracle.future_scores(f['q'], f['target'], f['dk'], f['dv'], f['a'], f['contrast'], f['source_start'],
                               f['window'])
    assert _rel(_future(_dev(f)), ref) < REL


def test_key_response_larger():
    k = key_inputs(h=8, t=768, p=6, m=128, source_start=256, query_start=256, window=512, seed=5)
    ref = oracle.key_response(k['q'], k['dk'], k['A'], k['C'], k['source_start'], k['query_start'], k['window'])
    assert _rel(_key(_dev(k)), ref) < REL


def test_query_response_larger():
    q = query_inputs(m=5, p=72, h=8, t=1024, window=512, seed=7)
    ref = oracle.query_response(q['dq'], q['keys'], q['values'], q['probabilities'], q['base'])
    assert _rel(_query(_dev(q)), ref) < REL


@pytest.mark.parametrize('k', [16, 100, 256])
def test_routed_response_sizes(k):
    r = routed_inputs(m=6, p=70, h=8, k=k, seed=11)
    ref = oracle.routed_response(r['dq'], r['keys'], r['values'], r['probabilities'], r['rest'])
    assert _routed_ok(_routed(_dev(r)), ref)


def test_install_registers_cuda_kernels():
    """install(R) makes R's ops run these kernels on CUDA tensors, as the reference's fast_kernels.install does: here
    R is a stand-in module whose ops have only their dense default implementations."""
    import types
    from noise_b200 import readout

    @torch.library.custom_op('noise_b200_test_record::future_scores', mutates_args=())
    def fused_scores(q: torch.Tensor, target: torch.Tensor, dk: torch.Tensor, dv: torch.Tensor, a: torch.Tensor,
                     contrast: torch.Tensor, source_start: int, window: int) -> torch.Tensor:
        return oracle.future_scores(q.cpu(), target.cpu(), dk.cpu(), dv.cpu(), a.cpu(), contrast.cpu(), source_start,
                                    window).float().to(q.device)

    def stub(name):
        @torch.library.custom_op(f'noise_b200_test_record::{name}', mutates_args=())
        def op(x: torch.Tensor) -> torch.Tensor:
            return x.clone()
        return op

    R = types.SimpleNamespace(fused_scores=fused_scores, fused_key_response=stub('key_response'),
                              query_response=stub('future_query_response'), routed_response=stub('routed_response'))
    f = _dev(future_inputs())
    readout.install(R)
    out = R.fused_scores(f['q'], f['target'], f['dk'], f['dv'], f['a'], f['contrast'], f['source_start'],
                         f['window'])
    torch.cuda.synchronize()
    ref = oracle.future_scores(*(v.cpu() if torch.is_tensor(v) else v for v in future_inputs().values()))
    assert out.is_cuda and _rel(out, ref) < REL
