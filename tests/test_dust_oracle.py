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
