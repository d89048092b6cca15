"""The tcgen05 identity-phase GEMMs (noise_b200.id_kernels) against the reference's Triton kernels (tests/golden/
id_kernels.pt) and, at larger shapes taking the other tile width, against the CPU oracle (oracle/idk.py).

Stated tolerance: as tests/test_id_kernels_oracle.py (one bf16 ulp, two for hidden_credits, or 2^-16 of the largest
|output| near zero; at most 2% of the outputs differ)."""
import sys

import pytest
import torch

from conftest import GOLDEN
from oracle import idk
from test_id_kernels_oracle import check

sys.path.insert(0, str(GOLDEN))
from id_inputs import at_b_inputs, hidden_inputs, square_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None


@pytest.fixture(scope='module')
def ik():
    import noise_b200.id_kernels as m
    return m


def dev(ts):
    return [t.to(DEV) for t in ts]


def status_ok(out):
    from noise_b200 import _lib
    return _lib.read_status(out._noise_workspace) == 0


def test_against_reference_kernels(ik, golden):
    g = golden('id_kernels.pt')
    us, steps, credb, w_out_t = hidden_inputs()
    got = ik.hidden_credits_fused(dev(us), steps.to(DEV), credb.to(DEV), w_out_t.to(DEV))
    assert status_ok(got)
    check(got.cpu(), g['hidden'], 2.0)
    As, Bs = at_b_inputs()
    out = torch.empty(8, As[0].shape[-1], Bs[0].shape[-1], dtype=torch.bfloat16, device=DEV)
    ik.at_b_layers(dev(As), dev(Bs), out)
    assert status_ok(out)
    check(out.cpu(), g['at_b'])
    n1s, got2 = square_inputs()
    d = n1s[0].shape[1]
    out = torch.empty(3 * len(n1s), d, d, dtype=torch.bfloat16, device=DEV)
    ik.square_credit_grads(dev(n1s), got2.to(DEV), out)
    assert status_ok(out)
    check(out.cpu(), g['square'])


@pytest.mark.parametrize('m,n,k', [(512, 384, 256), (256, 2048, 512)])
def test_hidden_credits_larger(ik, m, n, k):
    us, steps, credb, w_out_t = hidden_inputs(m=m, n=n, k=k, seed=m + n + k)
    got = ik.hidden_credits_fused(dev(us), steps.to(DEV), credb.to(DEV), w_out_t.to(DEV))
    assert status_ok(got)
    check(got.cpu(), idk.hidden_credits(us, steps, credb, w_out_t), 2.0)


@pytest.mark.parametrize('k,p,q', [(1024, 256, 512), (4096, 128, 384)])
def test_at_b_layers_larger(ik, k, p, q):
    As, Bs = at_b_inputs(k=k, p=p, q=q, seed=k + p + q)
    out = torch.empty(8, p, q, dtype=torch.bfloat16, device=DEV)
    ik.at_b_layers(dev(As), dev(Bs), out)
    assert status_ok(out)
    check(out.cpu(), idk.at_b_layers(As, Bs))


@pytest.mark.parametrize('world,m', [(4, 256), (8, 192)])
def test_square_credit_grads_larger(ik, world, m):
    """world 4 (d = 256: 256-wide tiles, each of 4 column chunks from a different got2 plane) and world 8 (d = 512),
    written into a slice of a wider gradient buffer as run.py's gsq[:3 L]."""
    n1s, got2 = square_inputs(world=world, m=m, seed=world * m)
    d = world * 64
    buf = torch.zeros(32, d, d, dtype=torch.bfloat16, device=DEV)
    out = buf[:24]
    ik.square_credit_grads(dev(n1s), got2.to(DEV), out)
    assert status_ok(out)
    check(out.cpu(), idk.square_credit_grads(n1s, got2))
    assert buf[24:].abs().sum().item() == 0
