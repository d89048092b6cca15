"""Parity of the sm_100a credit kernels with the reference's own Triton kernels (tests/golden/credit_kernels.pt, made
by running moment_kernels.py under the Triton interpreter) and with the dense CPU oracle (oracle/credit.py).

Stated tolerances (relative to the largest |reference| of the output): lse / center 1e-5; value credits 2e-3 (bf16
probabilities, hi + lo source); key credits and key moments 5e-3; query credits 1e-2 (bf16 operands and a bf16-rounded
output, so single elements differ by a bf16 ulp). The key scan's raw value credits 4e-3: the interpreter evaluates the
reference's tf32 logit dots exactly, while on the GPU the kind::tf32 MMAs read the tf32 part of each fp32 operand, as
the reference's own Triton kernel does there (the tcgen05 key scan is within 2e-4 of that kernel at config 3,
tests/test_credit_triton_gpu.py); against the exact dots that moves these sums by up to 2.7e-3."""
import sys

import pytest
import torch

from conftest import GOLDEN
from oracle import credit

sys.path.insert(0, str(GOLDEN))
from credit_inputs import credit_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None


def rel(a, r):
    return ((a.double().cpu() - r.double().cpu()).abs().max() / r.double().abs().max()).item()


def dev(x):
    return {k: v.to(DEV) for k, v in x.items()}


@pytest.fixture(scope='module')
def mk():
    import noise_b200.moment_kernels as m
    return m


@pytest.fixture(scope='module')
def fixture(golden):
    g = golden('credit_kernels.pt')
    x = credit_inputs(g['rows'], g['length'], g['seed'])
    return g, x


@pytest.mark.parametrize('window', [128, 256])
def test_against_reference_kernels(mk, fixture, window):
    g, x = fixture
    o = g['out'][window]
    d = dev(x)
    b = {k: d[k].bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    lse, center = mk.implicit_key_context_edges(b['qp'], b['kp'], b['values'], b['hub'], window)
    assert rel(lse, o['lse']) < 1e-5 and rel(center, o['center']) < 1e-5
    lse_r, ctr_r = o['lse'].to(DEV), o['center'].to(DEV)
    raw = mk.raw_value_credits(b['qp'], b['kp'], lse_r, d['hub'], window)
    assert rel(raw, o['raw_value']) < 2e-3
    key = mk.key_credits(d['qp'], d['kp'], d['k_raw'], lse_r, d['values'], d['hub'], ctr_r, d['cos'], d['sin'],
                         window, 0.003)
    assert rel(key, o['key']) < 5e-3
    key_v, raw_v = mk.key_and_raw_value_credits(d['qp'], d['kp'], d['k_raw'], lse_r, d['values'], d['hub'], ctr_r,
                                                d['cos'], d['sin'], window, 0.003)
    assert rel(key_v, o['key_v']) < 5e-3 and rel(raw_v, o['raw_v']) < 4e-3
    qs = torch.empty(1, g['rows'], g['length'], 64, dtype=torch.bfloat16, device=DEV)
    mk.moment_query_scores(b['qp'], b['kp'], b['values'], b['hub'], d['q_raw'].unsqueeze(0), o['sq'].to(DEV),
                           d['kp'], d['cos'], d['sin'], lse_r, ctr_r, o['steps'].to(DEV), qs, 4, window)
    assert rel(qs[0].float(), o['query']) < 1e-2
    assert (qs[0].float().cpu() != o['query']).float().mean() < 0.05


def test_key_moments_against_reference_kernel(mk, fixture):
    g, x = fixture
    o = g['out']['keys']
    d = dev(x)
    b = {k: d[k].bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    out = torch.empty(1, g['rows'], g['length'], 64, device=DEV)
    vals = torch.empty_like(out)
    mk.moment_key_scores(b['qp'], b['kp'], b['values'], b['hub'], d['k_raw'].unsqueeze(0), o['sq'].to(DEV), d['qp'],
                         d['cos'], d['sin'], o['lse'].to(DEV), o['center'].to(DEV), o['steps'].to(DEV), out, vals, 2)
    assert rel(out[0], o['out']) < 5e-3 and rel(vals[0], o['values']) < 2e-3


@pytest.mark.parametrize('window', [128, 320, 512])
def test_against_oracle_larger(mk, window):
    """rows 4, T 512, against the dense oracle with bf16 operand rounding; windows that are and are not tile
    multiples (320 for the kernels that take any window)."""
    x = credit_inputs(4, 512, seed=11)
    d = dev(x)
    b = {k: d[k].bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    bd = {k: x[k].bfloat16().double() for k in ('qp', 'kp', 'values', 'hub')}
    w_ctx = window if window % 64 == 0 else 512
    lse, center = mk.implicit_key_context_edges(b['qp'], b['kp'], b['values'], b['hub'], w_ctx)
    ref_lse, ref_center = credit.implicit_key_context(bd['qp'], bd['kp'], bd['values'], bd['hub'], w_ctx)
    assert rel(lse, ref_lse) < 1e-5 and rel(center, ref_center) < 1e-5
    raw = mk.raw_value_credits(b['qp'], b['kp'], lse, d['hub'], window)
    assert rel(raw, credit.value_pass(bd['qp'], bd['kp'], lse.cpu(), x['hub'], window, emulate=True)) < 2e-3
    key = mk.key_credits(d['qp'], d['kp'], d['k_raw'], lse, d['values'], d['hub'], center, d['cos'], d['sin'], window,
                         0.003)
    ref = credit.key_scan(x['qp'], x['kp'], x['k_raw'], lse.cpu(), x['values'], x['hub'], center.cpu(), x['cos'],
                          x['sin'], window, 0.003, emulate=True)
    assert rel(key, ref) < 5e-3
    sq = x['q_raw'].square().sum(-1)
    steps = 0.01 * (sq / 64).sqrt().clamp(min=1e-6)
    qs = torch.empty(1, 4, 512, 64, dtype=torch.bfloat16, device=DEV)
    mk.moment_query_scores(b['qp'], b['kp'], b['values'], b['hub'], d['q_raw'].unsqueeze(0), sq.to(DEV), d['kp'],
                           d['cos'], d['sin'], lse, center, steps.to(DEV), qs, 4, window)
    ref = credit.moment_query_scores(bd['qp'], bd['kp'], bd['values'], bd['hub'], x['q_raw'], sq, x['kp'], x['cos'],
                                     x['sin'], lse.cpu(), center.cpu(), steps, window, emulate=True)
    assert rel(qs[0].float(), ref) < 1e-2


def test_by_token_layouts_and_layer_map(mk):
    """The *_by_token / *_into variants: rows = (layer, head) with 2 layers x 2 heads written into a (layers, T, 3 W)
    buffer's column slice through a layer map, as Cut.batched_key_scores_by_token does."""
    x = credit_inputs(4, 256, seed=5)
    d = dev(x)
    b = {k: d[k].bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    window, heads = 128, 2
    lse, center = mk.implicit_key_context_edges(b['qp'], b['kp'], b['values'], b['hub'], window)
    stacked = mk.raw_value_credits(b['qp'], b['kp'], lse, d['hub'], window)
    by_tok = mk.raw_value_credits_by_token(b['qp'], b['kp'], lse, d['hub'], window, heads)
    assert torch.equal(by_tok, stacked.view(2, heads, 256, 64).transpose(1, 2).reshape(2, 256, heads * 64))
    buf = torch.zeros(3, 256, 3 * heads * 64, device=DEV)
    layers = torch.tensor([2, 0], dtype=torch.int32, device=DEV)
    key = mk.key_credits(d['qp'], d['kp'], d['k_raw'], lse, d['values'], d['hub'], center, d['cos'], d['sin'], window,
                         0.003)
    mk.key_credits_into(d['qp'], d['kp'], d['k_raw'], lse, d['values'], d['hub'], center, d['cos'], d['sin'], window,
                        0.003, buf[:, :, heads * 64:2 * heads * 64], layers)
    want = key.view(2, heads, 256, 64).transpose(1, 2).reshape(2, 256, heads * 64)
    assert torch.equal(buf[2, :, heads * 64:2 * heads * 64], want[0])
    assert torch.equal(buf[0, :, heads * 64:2 * heads * 64], want[1])
    assert buf[1].abs().sum() == 0 and buf[:, :, :heads * 64].abs().sum() == 0
    corrected = by_tok.clone()
    out = torch.zeros(2, 256, heads * 64, device=DEV)
    mk.terminal_value_credits_into(b['qp'], b['kp'], lse, corrected, window, out)
    ref = mk.terminal_value_credits(b['qp'], b['kp'], lse, stacked, window)
    assert torch.equal(out, ref.view(2, heads, 256, 64).transpose(1, 2).reshape(2, 256, heads * 64))


def test_plugin_seams_match_reference_signatures(mk):
    """KEY_IMPL / VALUE_IMPL take the reference's plug-in arguments (moment_kernels.py:642-650)."""
    x = credit_inputs(2, 128, seed=3)
    d = dev(x)
    lse, center = mk.implicit_key_context_edges(d['qp'], d['kp'], d['values'], d['hub'], 128)
    key, same = mk.KEY_IMPL(d['qp'], d['kp'], d['k_raw'], lse, d['values'], d['hub'], center, d['cos'], d['sin'], 128,
                            0.003, False, 1, None, None)
    assert key is same and key.shape == (2, 128, 64)
    out = mk.VALUE_IMPL(d['qp'], d['kp'], lse, d['hub'], 128, 1, 1, None, None)
    assert out.shape == (2, 128, 64)
