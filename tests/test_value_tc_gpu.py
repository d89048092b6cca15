"""The tcgen05 value pass (noise_value_pass_ws, bf16 operands, T % 128 == 0) against the dense CPU oracle
(oracle/credit.value_pass with the kernel's bf16 probability rounding and hi + lo source split) and against the
warp-MMA kernel (noise_value_pass) on the same inputs.

Stated tolerance: 2e-3 of the largest |reference| of the output (bf16 probabilities; the two GPU kernels round the
exponent argument differently, so single probabilities can differ by one bf16 ulp). At the credit benchmark's full
size (rows 128, T 2048, window 2048) the size-independent property: with lse taken over the same window every
receiver's probabilities sum to one, so sum_t out[t] = sum_s source[s] for each row and channel."""
import sys

import pytest
import torch

from conftest import GOLDEN
from oracle import credit

sys.path.insert(0, str(GOLDEN))
from credit_inputs import credit_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None
TOL = 2e-3


def rel(a, r):
    return ((a.double().cpu() - r.double().cpu()).abs().max() / r.double().abs().max()).item()


@pytest.fixture(scope='module')
def mk():
    import noise_b200.moment_kernels as m
    return m


def run(mk, b, lse, source, window, **kw):
    out = mk.value_pass(b['qp'], b['kp'], lse, source, window, **kw)
    return out


# windows below, at and above one tile; T = 384 has an odd number of key tiles (the last pair has one tile)
@pytest.mark.parametrize('rows,t,window', [(3, 384, 0), (3, 384, 1), (3, 384, 127), (3, 384, 200), (3, 384, 1000),
                                           (2, 256, 128), (1, 128, 64), (2, 512, 320)])
def test_against_oracle_and_warp_kernel(mk, rows, t, window):
    from noise_b200 import _lib
    x = credit_inputs(rows, t, seed=rows * 1000 + window)
    b = {k: x[k].to(DEV).bfloat16() for k in ('qp', 'kp')}
    bd = {k: x[k].bfloat16().double() for k in ('qp', 'kp')}
    lse = credit.implicit_key_context(bd['qp'], bd['kp'], bd['qp'], bd['qp'], window)[0]
    lse = lse.float().to(DEV)
    src = x['hub'].to(DEV)
    got = run(mk, b, lse, src, window)
    torch.cuda.synchronize()
    assert _lib.read_status(got._noise_workspace) == 0
    ref = credit.value_pass(bd['qp'], bd['kp'], lse.cpu(), x['hub'], window, emulate=True)
    assert rel(got, ref) < TOL
    warp = run(mk, b, lse, src, window, tc=False)
    assert not hasattr(warp, '_noise_workspace')
    assert rel(got, warp) < TOL


def test_more_items_than_sms_and_strided_views(mk):
    """600 work items on 148 SMs (persistent loop, both O buffers reused); the source read and the output written
    through by-token views (rows // 2, T, 2 * 64), as terminal_value_credits_into does."""
    rows, t, window, heads = 300, 512, 512, 2
    g = torch.Generator().manual_seed(5)
    q = torch.nn.functional.rms_norm(torch.randn(rows, t, 64, generator=g), (64,)).to(DEV).bfloat16()
    k = torch.nn.functional.rms_norm(torch.randn(rows, t, 64, generator=g), (64,)).to(DEV).bfloat16()
    lse = (torch.randn(rows, t, generator=g) * 0.3 + 5.0).to(DEV)
    src = (torch.randn(rows // heads, t, heads * 64, generator=g) * 0.1).to(DEV)
    got = mk.value_pass(q, k, lse, src, window, heads, heads)
    warp = mk.value_pass(q, k, lse, src, window, heads, heads, tc=False)
    torch.cuda.synchronize()
    from noise_b200 import _lib
    assert _lib.read_status(got._noise_workspace) == 0
    assert rel(got, warp) < TOL


def test_full_size_sum_property(mk):
    """rows 128 (16 x 8 heads), T 2048, window 2048: sum over keys of the credits equals the source's sum over
    receivers (probabilities normalised by the same window's lse), and the two GPU kernels agree."""
    rows, t, window = 128, 2048, 2048
    x = credit_inputs(rows, t, seed=3)
    b = {k: x[k].to(DEV).bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    lse, _ = mk.implicit_key_context_edges(b['qp'], b['kp'], b['values'], b['hub'], window)
    src = x['values'].to(DEV)
    got = mk.value_pass(b['qp'], b['kp'], lse, src, window)
    warp = mk.value_pass(b['qp'], b['kp'], lse, src, window, tc=False)
    torch.cuda.synchronize()
    from noise_b200 import _lib
    assert _lib.read_status(got._noise_workspace) == 0
    assert rel(got, warp) < TOL
    s_out, s_src = got.double().sum(1), src.double().sum(1)
    assert ((s_out - s_src).abs().max() / s_src.abs().max()).item() < 1e-2
