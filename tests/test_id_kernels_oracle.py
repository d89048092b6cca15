"""The identity-phase GEMM oracle (oracle/idk.py) against the reference's own Triton kernels (tests/golden/
id_kernels.pt, made by running speedrun/id_kernels.py under the patched interpreter).

Stated tolerance: bf16 outputs within one bf16 ulp of the reference (fp64 vs fp32 accumulation before the bf16
rounding) or, for outputs near zero (cancelling sums), within 2^-16 of the matrix's largest |output|; at most 2% of
the outputs differ at all. hidden_credits rounds the product to bf16 before scaling it by the slope (up to 2 |u|),
so a one-ulp difference there can become two in the output: two ulps there."""
import sys

import torch

from conftest import GOLDEN
from oracle import idk

sys.path.insert(0, str(GOLDEN))
from id_inputs import at_b_inputs, hidden_inputs, square_inputs  # noqa: E402


def ulps(got, ref):
    """|got - ref| in units of max(ref's bf16 ulp (2^(exponent - 7)), 2^-16 max |ref|), elementwise."""
    g, r = got.float(), ref.float()
    e = torch.floor(torch.log2(r.abs().clamp(min=2.0 ** -126)))
    return (g - r).abs() / torch.maximum(torch.pow(2.0, e - 7), r.abs().max() * 2.0 ** -16)


def check(got, ref, max_ulps=1.0):
    u = ulps(got, ref)
    assert u.max().item() <= max_ulps, u.max().item()
    assert (u > 0).float().mean().item() <= 0.02


def test_hidden_credits(golden):
    g = golden('id_kernels.pt')
    check(idk.hidden_credits(*hidden_inputs()), g['hidden'], 2.0)


def test_at_b_layers(golden):
    g = golden('id_kernels.pt')
    check(idk.at_b_layers(*at_b_inputs()), g['at_b'])


def test_square_credit_grads(golden):
    g = golden('id_kernels.pt')
    check(idk.square_credit_grads(*square_inputs()), g['square'])
