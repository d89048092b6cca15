"""Parity of the identity phase's head-sharding kernels (noise_b200.heads: run.py's pack_heads_kernel,
head_prep_fused, id_head_scores) with the reference's own outputs (tests/golden/heads.pt) and with the CPU oracle
at larger sizes.

Tolerances: the pack is a byte copy (bit-exact). head_prep's bf16 outputs are roundings of fp32 arithmetic done in
another order (sums of squares, rsqrt, FMA contraction): within one bf16 unit plus 1e-6, on under 1% of elements; its fp32 outputs within
REL_F32. The credits are bf16 results of the moment kernels (tf32/bf16 tensor-core dots): max |diff| within
CREDIT_REL of max |ref| (one bf16 rounding flip on the largest element is 0.4%)."""
import sys
from pathlib import Path

import pytest
import torch

from oracle import heads as oracle_heads

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from heads_inputs import got_inputs, pack_inputs, rotary  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None
REL_F32 = 2e-6
CREDIT_REL = 1e-2


def _rel(a, r):
    a, r = a.double().cpu(), r.double().cpu()
    return ((a - r).abs().max() / r.abs().max()).item()


def _close_bf16(a, r):
    """Every element within one bf16 unit of the reference (2^-7 relative) plus 1e-6 absolute: fp32 arithmetic in
    another order (FMA contraction, rsqrt rounding) moves values near zero (cancellation in the RoPE rotation) by more
    units in the last place than values away from it."""
    a, r = a.cpu().float(), r.cpu().float()
    return bool(((a - r).abs() <= 2.0 ** -7 * r.abs() + 1e-6).all())


def _dev(p):
    return {k: [z.to(DEV) for z in v] for k, v in p.items()}


def test_pack_heads_matches_reference(golden):
    from noise_b200 import heads
    g = golden('heads.pt')
    p = _dev(pack_inputs())
    out = heads.pack_heads_kernel(p['qs'], p['ks'], p['vals'], p['outs'], p['targets'], p['lses'])
    torch.cuda.synchronize()
    assert torch.equal(out.cpu().view(torch.int16), g['pack'])


def test_pack_heads_full_layers():
    """Eight layers of 2048 tokens in rows of 1024 (the identity phase's shape on one rank): bit-exact."""
    from noise_b200 import heads
    p = pack_inputs(layers=8, n=2048, t=1024, seed=3)
    out = heads.pack_heads_kernel(*(_dev(p)[k] for k in ('qs', 'ks', 'vals', 'outs', 'targets', 'lses')))
    ref = oracle_heads.pack_heads(p['qs'], p['ks'], p['vals'], p['outs'], p['targets'], p['lses'])
    torch.cuda.synchronize()
    assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))


def _check_prep(mine, ref):
    for name in ('v16', 'hub16', 'lse'):
        assert torch.equal(mine[name].cpu().reshape(-1), ref[name].reshape(-1)), name
    for name in ('q16', 'k16', 'f2', 'f4', 'xy'):
        assert _close_bf16(mine[name], ref[name]), name
        assert (mine[name].cpu() != ref[name]).float().mean() < 0.01, name
    for name in ('q32', 'sq_q', 'sq_k', 'steps_q', 'steps_k', 'hub_out'):
        assert _rel(mine[name], ref[name]) < REL_F32, name


def _prep(got, b, t):
    from noise_b200 import heads
    cos, sin = rotary(t)
    names = ('q16', 'k16', 'v16', 'hub16', 'q32', 'pairs', 'lse', 'hub_out', 'sq_q', 'sq_k', 'steps_q', 'steps_k')
    out = dict(zip(names, heads.head_prep_fused(got.to(DEV), cos.to(DEV), sin.to(DEV), b, t)))
    out['f2'], out['f4'], out['xy'] = out.pop('pairs')
    torch.cuda.synchronize()
    return out


def test_head_prep_matches_reference(golden):
    g = golden('heads.pt')
    got, b = got_inputs()
    _check_prep(_prep(got, b, g['t']), g['prep'])


def test_head_prep_matches_oracle_larger():
    got, b = got_inputs(world=8, layers=3, n=512, t=256, seed=21)
    cos, sin = rotary(256)
    _check_prep(_prep(got, b, 256), oracle_heads.head_prep(got, cos, sin, b, 256))


def _scores(got, b, t):
    from noise_b200 import heads
    cos, sin = rotary(t)
    w, layers, n, _ = got.shape
    back = torch.full((w, layers, 3, n, 64), float('nan'), dtype=torch.bfloat16, device=DEV)
    heads.id_head_scores(got.to(DEV), (cos.to(DEV), sin.to(DEV)), back, b, t)
    torch.cuda.synchronize()
    return back.cpu()


def test_id_head_scores_matches_reference(golden):
    g = golden('heads.pt')
    got, b = got_inputs()
    back = _scores(got, b, g['t'])
    assert not back.isnan().any()
    for slot in range(3):
        assert _rel(back[:, :, slot], g['back'][:, :, slot]) < CREDIT_REL, slot


def test_id_head_scores_matches_oracle_larger():
    got, b = got_inputs(world=8, layers=2, n=256, t=256, seed=5)
    back = _scores(got, b, 256)
    cos, sin = rotary(256)
    ref = oracle_heads.id_head_scores(got, cos, sin, b, 256)
    assert not back.isnan().any()
    for slot in range(3):
        assert _rel(back[:, :, slot], ref[:, :, slot].float().bfloat16()) < CREDIT_REL, slot
