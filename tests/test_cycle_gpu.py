"""Parity of the readout cycle (noise_b200.cycle: top_credit, coordinate_change, cycle_weights_fused) with the
reference's own outputs (tests/golden/cycle.pt) and with the oracle at a larger size.

Tolerances: top_credit divides the moved-minus-clean cross-entropy by a step of 0.005 rms(x), so its contractions'
precision shows at CREDIT_REL of max |ref|: they run at tf32 as the reference runs them on the GPU
(torch.set_float32_matmul_precision('high')), which moves the credit by 9e-4 of max |ref| in a CPU emulation of
tf32 operands (the method's own fp32-vs-fp64 gap on these inputs is 5e-4); coordinate_change within 1e-5."""
import sys
import types
from pathlib import Path

import pytest
import torch

from oracle import cycle as oracle

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from cycle_inputs import cycle_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None
CREDIT_REL = 3e-3


def _rel(a, r):
    a, r = a.double().cpu(), r.double().cpu()
    return ((a - r).abs().max() / r.abs().max()).item()


def _model(x):
    return types.SimpleNamespace(H=x['H'].to(DEV), step_t=x['step_t'].to(DEV), lm_head=x['lm_head'].to(DEV))


@pytest.fixture(autouse=True)
def full_fp32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def test_against_reference(golden):
    from noise_b200 import cycle
    g, x = golden('cycle.pt'), cycle_inputs()
    got = cycle.top_credit(_model(x), x['x'].to(DEV), x['y'].to(DEV))
    assert _rel(got, g['credit']) < CREDIT_REL
    assert torch.equal(cycle.step_signs(x['step_t'].to(DEV), DEV).cpu(), g['signs'])
    for dt in (torch.float32, torch.bfloat16):
        coords = cycle.coordinate_change(x['raw'].to(DEV).to(dt), x['y'].to(DEV))
        ref = g['coords'] if dt == torch.float32 else oracle.coordinate_change(x['raw'].bfloat16().float(), x['y'])
        assert _rel(coords, ref) < 1e-5


def test_top_credit_larger():
    """256 tokens (the bf16 moment GEMMs on the tcgen05 core) against the fp64 oracle."""
    from noise_b200 import cycle
    x = cycle_inputs(n=256, seed=5, step=11)
    got = cycle.top_credit(_model(x), x['x'].to(DEV), x['y'].to(DEV))
    signs = cycle.step_signs(x['step_t'], 'cpu')
    ref = oracle.top_credit(x['H'], signs, x['lm_head'], x['x'], x['y'])
    assert _rel(got, ref) < CREDIT_REL


def test_cycle_weights_fused_shapes():
    from noise_b200 import cycle
    x = cycle_inputs(n=64, seed=9)
    xs = x['x'].to(DEV)
    base = xs @ x['lm_head'].to(DEV)
    h = x['H'].to(DEV)
    fg1, fast, rows, total, steps, inv, inv0, delta, sigma = cycle.cycle_weights_fused(xs, base, h)
    assert fg1.shape == (64, 4096) and fast.shape == (5, 64, 4096) and fast.dtype == torch.bfloat16
    assert rows.shape == (64, 3) and total.shape == (64, 1) and inv.shape == (64, 512)
    z = base * inv0
    f = torch.exp(15 * torch.tanh(z / 15))
    assert _rel(total[:, 0], f.sum(-1)) < 1e-5 and _rel(fg1, f * (1 - torch.tanh(z / 15) ** 2)) < 1e-5
