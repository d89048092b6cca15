"""The readout-scorer oracle (oracle/readout.py) against the reference's own ops (tests/golden/readout.pt:
noise_record::future_scores and ::future_query_response through their CPU paths, ::key_response and
::routed_response through their Triton kernels under the patched interpreter)."""
import sys
from pathlib import Path

import torch

from oracle import readout

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from readout_inputs import future_inputs, key_inputs, query_inputs, routed_inputs  # noqa: E402


def _rel(a, r):
    return ((a.double() - r.double()).abs().max() / r.double().abs().max()).item()


def test_future_scores(golden):
    f = future_inputs()
    got = readout.future_scores(f['q'], f['target'], f['dk'], f['dv'], f['a'], f['contrast'], f['source_start'],
                                f['window'])
    assert _rel(got, golden('readout.pt')['future']) < 1e-5


def test_key_response(golden):
    k = key_inputs()
    got = readout.key_response(k['q'], k['dk'], k['A'], k['C'], k['source_start'], k['query_start'], k['window'])
    assert _rel(got, golden('readout.pt')['key']) < 1e-5


def test_query_response(golden):
    q = query_inputs()
    got = readout.query_response(q['dq'], q['keys'], q['values'], q['probabilities'], q['base'])
    assert _rel(got, golden('readout.pt')['query']) < 1e-5


def test_routed_response(golden):
    r = routed_inputs()
    got = readout.routed_response(r['dq'], r['keys'], r['values'], r['probabilities'], r['rest'])
    ref = golden('readout.pt')['routed']
    # bf16-rounded dot outputs: sums in another order flip an occasional rounding
    assert _rel(got, ref) < 1e-2 and (got - ref).abs().gt(1e-3 * ref.abs().max()).float().mean() < 0.01
