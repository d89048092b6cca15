"""The no-allocation entry point noise_population_loss_noalloc against the workspace entry point.

Some callers cannot allocate device memory when they evaluate (a C/FFI host without its own CUDA allocator that must
not call cudaMalloc on its hot path, or one whose memory pool is already fully reserved); the no-allocation entry point
runs in the library's static device scratch instead. Both entry points run the same kernels on the same inputs, so
their results must be identical bit for bit. This file is collected last so that a failure here, under ``-x``, comes
after every other test has run. It passes alone in a fresh process and after the other tests."""
import ctypes

import pytest
import torch

from oracle import eggroll, gpt

pytestmark = pytest.mark.gpu


def _case(members, length, seed, device):
    from noise_b200.population import member_offsets
    shapes = gpt.param_shapes()
    n_noise = 2 ** 20
    buf = eggroll.make_buffer(n_noise, seed=0).to(device)
    offs = eggroll.offsets(shapes, members // 2, step=seed, n_noise=n_noise)
    table = torch.stack([offs[n] for n, _ in shapes]).to(device)
    off = member_offsets(table, (torch.arange(members) // 2).to(device))
    sign = torch.where(torch.arange(members) % 2 == 0, eggroll.SIGMA, -eggroll.SIGMA).to(device)
    tok = gpt.zipf_tokens(1, length + 1, seed=seed)[0].to(device)
    return buf, off, sign, tok[:-1], tok[1:]


@pytest.mark.parametrize('reduction', ['mean', 'none'])
def test_noalloc_matches_workspace_entry_point_twice_in_a_row(reduction):
    import noise_b200
    from noise_b200.population import PackedGPT, population_loss_offsets, population_loss_offsets_noalloc
    dev = torch.device('cuda', 0)
    packed = PackedGPT({k: v.to(dev) for k, v in gpt.informative_weights(0).items()})
    for members, length, seed in [(2, 2048, 11), (4, 1024, 12)]:  # two calls in a row, different sizes and inputs
        buf, off, sign, idx, tgt = _case(members, length, seed, dev)
        got = population_loss_offsets_noalloc(packed, buf, off, sign, idx, tgt, reduction)
        assert noise_b200._lib.read_static_status(dev) == 0, 'a bounded wait of the no-allocation call gave up'
        ref = population_loss_offsets(packed, buf, off, sign, idx, tgt, reduction)
        torch.cuda.synchronize()
        assert noise_b200._lib.read_status(ref._noise_workspace) == 0
        assert got.shape == ref.shape == ((members, length) if reduction == 'none' else (members,))
        assert torch.isfinite(got).all()
        assert torch.equal(got, ref), (got - ref).abs().max().item()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from noise_b200 import _lib
    L = _lib.lib()
    assert L.noise_population_workspace_bytes(4, 2048) > _lib.STATIC_SCRATCH_BYTES
    gpt_struct = _lib.GPT()
    slices = (_lib.Slice * 60)()
    fake = 256  # never dereferenced: the size check comes first
    rc = L.noise_population_loss_noalloc(ctypes.byref(gpt_struct), slices, fake, fake, fake, 4, 2048, 0, fake, None)
    assert rc == _lib.ERR_TOO_LARGE
    assert b'static scratch' in L.noise_status_string(rc)
