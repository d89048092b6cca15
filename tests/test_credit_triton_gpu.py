"""BASELINE config 3 on the B200: the tcgen05 credit kernels against the reference's own Triton kernels
(train/speedrun/moment_kernels.py with KEY_IMPL = VALUE_IMPL = None, JIT-compiled for sm_100 on this GPU, loaded
from the reference install in baseline/_ref) at full size: rows = 16 x 8 heads, T = 2048, windows 2048 and 1024,
the same seeded inputs (bench.credit_config3).

Both arms read the same key context (the reference's lse / center) downstream, so each kernel is compared on equal
inputs. Tolerances, of the largest |reference| output: lse / center 1e-5 (fp32 softmax statistics of bf16 dots);
value pass 2e-3 (bf16 probabilities; one exponent rounding apart moves single probabilities by one bf16 ulp); key
scan 5e-3 (tf32 logits and scores); query moments 1e-2 (the outputs are bf16); key moments 5e-3 and their value
sums 2e-3 — the tolerances the oracle comparisons of these kernels use."""
import sys

import pytest
import torch

from conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None


def rel(a, r):
    return ((a.double() - r.double()).abs().max() / r.double().abs().max()).item()


@pytest.fixture(scope='module')
def arms():
    if not bench.REFERENCE_MOMENT_KERNELS.exists():
        pytest.skip('the reference install (baseline/_ref) is absent: pip install the reference into baseline/_ref')
    import noise_b200.moment_kernels as ours
    return ours, bench.reference_moment_kernels(), bench.credit_config3(DEV)


@pytest.mark.parametrize('window', [2048, 1024])
def test_credit_kernels_match_reference_triton_at_config3(arms, window):
    ours, ref, x = arms
    lse, center = ref.implicit_key_context_edges(*x['b16'], window)
    my_lse, my_center = ours.implicit_key_context_edges(*x['b16'], window)
    torch.cuda.synchronize()
    errors = {'lse': rel(my_lse, lse), 'center': rel(my_center, center)}
    mine = bench.credit_calls(ours, x, window, lse, center)
    theirs = bench.credit_calls(ref, x, window, lse, center)
    for name in ('value_pass', 'key_scan', 'moment_query_scores', 'moment_key_scores'):
        if name not in mine:
            continue
        got = mine[name]()
        want = theirs[name]()
        torch.cuda.synchronize()
        if name == 'moment_key_scores':
            errors['key_moments'] = rel(got[0], want[0])
            errors['key_moment_values'] = rel(got[1], want[1])
        else:
            errors[name] = rel(got.float(), want.float())
    print(f'window {window}: ' + ', '.join(f'{k} {v:.2e}' for k, v in errors.items()))
    limits = {'lse': 1e-5, 'center': 1e-5, 'value_pass': 2e-3, 'key_scan': 5e-3, 'moment_query_scores': 1e-2,
              'key_moments': 5e-3, 'key_moment_values': 2e-3}
    for k, v in errors.items():
        assert v < limits[k], (k, v)
