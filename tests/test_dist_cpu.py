"""The multi-rank host logic on CPU ranks (gloo, world size 2): the loss all-gather gives every rank the same fitness
weights, and the update rebuilt on each rank's pair shard and all-reduced equals the single-rank rebuild. The
per-shard rebuild uses the CPU oracle here; on the GPU the same shards run on the tcgen05 rebuild."""
import os
import sys

import torch
import torch.multiprocessing as mp

from conftest import ROOT


def _worker(rank, world, port, result):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist
    from noise_b200.train import fitness_weights, pair_shard
    from oracle import eggroll as oe, gpt
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    pairs, n_noise = 6, 2 ** 16
    shapes = [s for s in gpt.param_shapes() if s[0] in ('resid_lambdas', 'transformer.h.1.attn.ve_gate.weight',
                                                         'transformer.h.0.attn.c_q.weight')]
    members = 2 * pairs
    per_rank = members // world
    # this rank's member losses (a deterministic stand-in for the forward), then the all-gather of eggroll.py:147-150
    all_losses = torch.linspace(8.0, 9.0, members) + 0.01 * torch.sin(torch.arange(members, dtype=torch.float32))
    local = all_losses[rank * per_rank:(rank + 1) * per_rank].clone()
    gathered = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(gathered, local)
    losses = torch.cat(gathered)
    weight, count = fitness_weights(losses, pairs)
    buf = oe.make_buffer(n_noise, seed=0)
    offs = oe.offsets(shapes, pairs, step=1, n_noise=n_noise)
    start, stop = pair_shard(pairs, rank, world)
    part_w = torch.zeros(pairs)
    part_w[start:stop] = weight[start:stop]
    part = oe.rebuild_update(buf, offs, part_w, count, shapes)
    flat = torch.cat([part[n].flatten() for n, _ in shapes])
    dist.all_reduce(flat)
    full = oe.rebuild_update(buf, offs, weight, count, shapes)
    ref = torch.cat([full[n].flatten() for n, _ in shapes])
    result[rank] = (float((flat - ref).abs().max()), float(ref.abs().max()), bool(torch.equal(losses, all_losses)))
    dist.destroy_process_group()


def test_two_rank_gather_and_sharded_update():
    world = 2
    port = 29500 + os.getpid() % 1000
    with mp.Manager() as m:
        result = m.dict()
        mp.spawn(_worker, args=(world, port, result), nprocs=world, join=True)
        for rank in range(world):
            err, scale, same = result[rank]
            assert same
            assert err <= 1e-5 * scale, (err, scale)


def test_pair_shards_partition_the_pairs():
    from noise_b200.train import pair_shard
    for pairs in (1, 7, 12288):
        for world in (1, 2, 3, 8):
            shards = [pair_shard(pairs, r, world) for r in range(world)]
            covered = [j for a, b in shards for j in range(a, b)]
            assert covered == list(range(pairs))
