"""The Dust block-rerun oracle (oracle/dust.py) against the reference's own block_forward (tests/golden/dust.pt)."""
import sys
from pathlib import Path

from oracle import dust

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from dust_inputs import dust_inputs  # noqa: E402


def _rel(a, r):
    return ((a.double() - r.double()).abs().max() / r.double().abs().max()).item()


def test_block_forward_fp32(golden):
    g, x = golden('dust.pt'), dust_inputs()
    gated = dust.block_forward(x['x'], x['w'], x['ve'], x['cos'], x['sin'], x['windows'][0], autocast=False,
                               **x['jitter'])
    plain = dust.block_forward(x['x'], x['plain'], None, x['cos'], x['sin'], x['windows'][1], autocast=False)
    assert _rel(gated, g['gated']) < 1e-5 and _rel(plain, g['plain']) < 1e-5


def test_head_error(golden):
    from dust_inputs import head_error_inputs
    h = head_error_inputs()
    n = 16
    noises = [h['noise'](n * 2, 128, 256) for _ in range(h['draws'] // n)]
    err = dust.head_error(h['raw'], h['y'], h['clean_loss'], noises, h['sigma'])
    ref = golden('dust.pt')['head_error']
    touched = ref.shape[-1]
    assert not err[..., touched:].any()
    assert _rel(err[..., :touched], ref) < 1e-2 and (err[..., :touched] != ref).float().mean() < 0.02
