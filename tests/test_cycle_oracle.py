"""The readout-cycle oracle (oracle/cycle.py) against the reference's own top_credit and coordinate_change
(tests/golden/cycle.pt), and the step signs' hash against the reference's."""
import sys
from pathlib import Path

import torch

from oracle import cycle

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from cycle_inputs import cycle_inputs  # noqa: E402


def _rel(a, r):
    return ((a.double() - r.double()).abs().max() / r.double().abs().max()).item()


def test_step_signs(golden):
    from noise_b200.cycle import step_signs
    x = cycle_inputs()
    assert torch.equal(step_signs(x['step_t'], 'cpu'), golden('cycle.pt')['signs'])


def test_top_credit(golden):
    """In fp32 (the reference's arithmetic) within 1e-4; the fp64 oracle differs from both by the method's own fp32
    error (the finish divides by a step of 0.005 rms(x)): 5e-4 here."""
    g, x = golden('cycle.pt'), cycle_inputs()
    got = cycle.top_credit(x['H'], g['signs'], x['lm_head'], x['x'], x['y'], dtype=torch.float32)
    assert _rel(got, g['credit']) < 1e-4
    got64 = cycle.top_credit(x['H'], g['signs'], x['lm_head'], x['x'], x['y'])
    assert _rel(got64, g['credit']) < 2e-3


def test_coordinate_change(golden):
    g, x = golden('cycle.pt'), cycle_inputs()
    assert _rel(cycle.coordinate_change(x['raw'], x['y']), g['coords']) < 1e-5
