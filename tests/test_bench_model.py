"""bench.py's algorithmic work model (CPU): the FLOPs and bytes its roofline fractions divide by.

A population forward call launches, per block, norm<BLOCK>, the QKV GEMM, attention, the c_proj GEMM, norm<MID>, the
c_fc GEMM and the mlp.c_proj GEMM; then norm<FINAL> and the LM-head GEMM once. Summed over one call, the per-launch
FLOPs must give the forward's 68.3 MFLOP per member-token (linears 2 x 27.26 M MAC, attention 2 x 6.82 M MAC at the
[S, S, S, L] x 2 windows, low-rank terms ~0.16 MFLOP)."""
import importlib.util

import pytest

from conftest import ROOT


@pytest.fixture(scope='module')
def bench():
    spec = importlib.util.spec_from_file_location('bench_model', ROOT / 'bench.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_visible_pairs_counts_the_window(bench):
    for length, window in ((256, 64), (384, 128), (512, 511), (128, 2048)):
        brute = sum(1 for t in range(length) for s in range(length) if 0 <= t - s <= window)
        assert bench.visible_pairs(length, window) == brute


def test_flops_per_call_match_the_forward(bench):
    members, length = 4, 2048
    per_block = ('gemm_qkv', 'attention', 'gemm_cproj', 'gemm_cfc', 'gemm_mproj')
    flops = sum(8 * bench.kernel_work(k, members, length)[0] for k in per_block)
    flops += bench.kernel_work('gemm_head_ce', members, length)[0]
    per_token = flops / (members * length)
    # everything but the low-rank terms, which no kernel kind counts
    assert per_token == pytest.approx(bench.FLOP_PER_MEMBER_TOKEN - 0.16e6, rel=2e-3)


def test_norm_bytes_per_row(bench):
    rows = 3 * 2048
    assert bench.kernel_work('norm_mix', 3, 2048) == (None, 5168.0 * rows)
    assert bench.kernel_work('norm_mid', 3, 2048) == (None, 3088.0 * rows)
    assert bench.kernel_work('gemm_cfc', 3, 2048)[1] is None
