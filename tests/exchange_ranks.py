"""Rank program of tests/test_exchange_gpu.py's two-GPU case (launched by torchrun, one process per GPU): the
peer-memory exchange against NCCL's all_to_all_single on the same buffers, three steps, bit for bit."""
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / 'tests' / 'golden'))


def main():
    from heads_inputs import pack_inputs
    from noise_b200 import heads
    rank, world = int(os.environ['RANK']), int(os.environ['WORLD_SIZE'])
    dev = torch.device('cuda', int(os.environ['LOCAL_RANK']))
    torch.cuda.set_device(dev)
    dist.init_process_group('nccl', device_id=dev, timeout=timedelta(seconds=60))
    layers, n, t = 2, 64, 32
    ex = heads.HeadExchange(layers, n, t, wait_seconds=20.0)
    try:
        for step in range(3):
            p = pack_inputs(layers=layers, n=n, t=t, seed=1000 * step + rank)
            p = {k: [x.to(dev) for x in v] for k, v in p.items()}
            args = (p['qs'], p['ks'], p['vals'], p['outs'], p['targets'], p['lses'])
            send = heads.pack_heads_kernel(*args)
            ref = torch.empty_like(send)
            dist.all_to_all_single(ref, send)
            ex.send_heads(*args)
            got = ex.wait_heads()
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), f'rank {rank} step {step}: got'
            g = torch.Generator(device=dev).manual_seed(77 + 10 * step + rank)
            back = torch.randn(world, layers, 3, n, 64, device=dev, generator=g).bfloat16()
            ref2 = torch.empty_like(back)
            dist.all_to_all_single(ref2, back)
            ex.send_back(back)
            got2 = ex.wait_back()
            assert torch.equal(got2.view(torch.int16), ref2.view(torch.int16)), f'rank {rank} step {step}: got2'
        assert ex.read_status() == 0
        print(f'exchange ok rank {rank}', flush=True)
    finally:
        ex.close()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
