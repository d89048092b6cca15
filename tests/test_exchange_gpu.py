"""The identity phase's peer-memory exchange (noise_b200.heads.HeadExchange: the pack fused with the heads-in
all_to_all, the heads-out all_to_all, the epoch-flag waits).

On one GPU (world 1, every send lands in the rank's own buffer): got equals pack_heads_kernel's send buffer and got2
equals back bit for bit over several epochs, calls out of the step order raise, and a wait for an epoch nobody sends
gives up after its limit with the timeout status (the context stays usable). On 2, 4 and 8 GPUs
(tests/exchange_ranks.py under torchrun, each skipped with fewer GPUs): got and got2 equal NCCL's all_to_all_single of
the same buffers bit for bit."""
import ctypes
import os
import subprocess
import sys

import pytest
import torch

from conftest import GOLDEN, ROOT

sys.path.insert(0, str(GOLDEN))
from heads_inputs import pack_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None


def pieces_on_device(seed):
    p = pack_inputs(layers=2, n=64, t=32, seed=seed)
    return {k: [x.to(DEV) for x in v] for k, v in p.items()}


def test_world1_round_trips_and_order():
    from noise_b200 import heads
    ex = heads.HeadExchange(layers=2, tokens=64, seq_len=32)
    try:
        for step in range(3):
            p = pieces_on_device(100 + step)
            args = (p['qs'], p['ks'], p['vals'], p['outs'], p['targets'], p['lses'])
            ref = heads.pack_heads_kernel(*args)
            ex.send_heads(*args)
            got = ex.wait_heads()
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
            with pytest.raises(RuntimeError):
                ex.wait_heads()
            back = torch.randn(1, 2, 3, 64, 64, device=DEV).bfloat16()
            ex.send_back(back)
            got2 = ex.wait_back()
            assert torch.equal(got2.view(torch.int16), back.view(torch.int16))
            assert ex.read_status() == 0
        assert ex.epoch == [3, 3]
    finally:
        ex.close()


def test_wait_gives_up_with_timeout_status():
    """A flag nobody sets: the wait kernel stops after 50 ms with NOISE_DEVICE_TIMEOUT in the status word."""
    from noise_b200 import _lib, heads
    ex = heads.HeadExchange(layers=1, tokens=16, seq_len=16)
    try:
        ws = torch.zeros(_lib.STATUS_BYTES, dtype=torch.uint8, device=DEV)
        rc = _lib.lib().noise_exchange_wait(ctypes.byref(ex.peers), 0, 7, 50_000_000, ws.data_ptr(),
                                            _lib.stream_handle(DEV))
        assert rc == 0
        assert _lib.read_status(ws) == 1
        assert torch.ones(4, device=DEV).sum().item() == 4  # the context is still usable
    finally:
        ex.close()


@pytest.mark.parametrize('world', [2, 4, 8])
def test_ranks_match_nccl_all_to_all(world):
    """world ranks (one GPU each; skipped when the box has fewer): the exchange against all_to_all_single."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f'needs {world} GPUs')
    env = dict(os.environ, NCCL_NVLS_ENABLE='0', PYTHONPATH=str(ROOT))
    cmd = ['timeout', '-k', '30', '240', sys.executable, '-m', 'torch.distributed.run', '--nnodes=1',
           '--nproc-per-node', str(world), '--master-addr', '127.0.0.1', '--master-port', str(29530 + world),
           str(ROOT / 'tests' / 'exchange_ranks.py')]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count('exchange ok') == world, r.stdout
