"""The head-sharding oracle (oracle/heads.py) against the reference's own kernels (tests/golden/heads.pt: run.py's
pack_heads_kernel, head_prep_fused and id_head_scores under the patched Triton interpreter)."""
import sys
from pathlib import Path

import torch

from oracle import heads

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from heads_inputs import got_inputs, pack_inputs, rotary  # noqa: E402


def _rel(a, r):
    return ((a.double() - r.double()).abs().max() / r.double().abs().max()).item()


def _close_bf16(a, r):
    """Every element within one bf16 unit of the reference (2^-7 relative) plus 1e-6 absolute: fp32 arithmetic in
    another order (FMA contraction, rsqrt rounding) moves values near zero (cancellation in the RoPE rotation) by more
    units in the last place than values away from it."""
    a, r = a.cpu().float(), r.cpu().float()
    return bool(((a - r).abs() <= 2.0 ** -7 * r.abs() + 1e-6).all())


def test_pack_heads_bit_exact(golden):
    g = golden('heads.pt')
    p = pack_inputs()
    out = heads.pack_heads(p['qs'], p['ks'], p['vals'], p['outs'], p['targets'], p['lses'])
    assert torch.equal(out.view(torch.int16), g['pack'])


def test_head_prep_matches_reference(golden):
    g = golden('heads.pt')
    got, b = got_inputs()
    cos, sin = rotary(g['t'])
    mine = heads.head_prep(got, cos, sin, b, g['t'])
    ref = g['prep']
    for name in ('v16', 'hub16', 'lse'):  # copies
        assert torch.equal(mine[name].view(-1), ref[name].reshape(-1)), name
    for name in ('q16', 'k16', 'f2', 'f4', 'xy'):  # bf16 of fp32 arithmetic: at most one rounding flip
        assert _close_bf16(mine[name], ref[name]), name
        assert (mine[name] != ref[name]).float().mean() < 0.01, name
    for name in ('q32', 'sq_q', 'sq_k', 'steps_q', 'steps_k', 'hub_out'):
        assert _rel(mine[name], ref[name]) < 1e-6, name


def test_id_head_scores_matches_reference(golden):
    g = golden('heads.pt')
    got, b = got_inputs()
    cos, sin = rotary(g['t'])
    back = heads.id_head_scores(got, cos, sin, b, g['t'])
    ref = g['back'].double()
    mine = back.float().bfloat16().double()  # the reference stores bf16
    for slot, tol in ((0, 1e-2), (1, 1e-2), (2, 1e-2)):
        assert _rel(mine[:, :, slot], ref[:, :, slot]) < tol, slot
