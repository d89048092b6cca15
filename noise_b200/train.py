"""One EGGROLL update end to end on the CUDA path (reference archive/10M/train/val/eggroll.py:131-167).

``EggrollTrainer.step(tokens, step)``:
1. offsets of the step (eggroll.py:117-120) and this rank's share of the population forward (``Population``);
2. NCCL all-gather of the losses, fitness l(-) - l(+) z-scored and summed per pair (eggroll.py:147-154);
3. the seed-rebuilt update G_P = -(1 / count) sum_j w_j a_j b_j^T over this rank's shard of the pairs: a GEMM with
   K = pairs on the tcgen05 core at tf32 (the reference's fp32 matmul at 'high' precision, eggroll.py:184) for every
   matrix, a direct kernel for the small ones (eggroll.py:155-163); the
   partial updates are summed with one NCCL all-reduce of the flat gradient (the reference rebuilds the whole update
   on every rank instead; ``shard_update=False`` does that);
4. AdamW on the flat fp32 parameters (eggroll.py:164-167) and a re-pack of the bf16 weights.
"""
import ctypes
import math

import torch

from . import _lib
from .eggroll import NOISE, SIGMA, Population, member_layout, noise_buffer, step_offsets
from .population import PARAMS

GEMM_N = 32  # the GEMM's N granularity (columns of a stored chunk)
GEMM_MIN_ROWS = 128  # smaller matrices (the [8, 32] value-embedding gates) take the direct kernel


def fitness_weights(losses, pairs):
    """Antithetic fitness l[odd] - l[even], z-scored, summed per pair (eggroll.py:151-154); (weight [pairs], count)."""
    fitness = losses[1::2] - losses[0::2]
    fitness = fitness / (fitness.std() + 1e-8)
    weight = torch.zeros(pairs, device=losses.device, dtype=fitness.dtype)
    weight.index_add_(0, torch.arange(len(fitness), device=losses.device) % pairs, fitness)
    return weight, len(fitness)


def pair_shard(pairs, rank, world):
    """[start, stop) of the pairs whose update terms rank `rank` of `world` rebuilds."""
    per = -(-pairs // world)
    start = min(pairs, rank * per)
    return start, min(pairs, start + per)


class FlatParams:
    """The 60 parameters as views of one flat fp32 buffer (named_parameters order), so an update is one all-reduce and
    one AdamW launch."""

    def __init__(self, params, device):
        sizes = [math.prod(shape) for _, shape in PARAMS]
        self.flat = torch.empty(sum(sizes), device=device, dtype=torch.float32)
        self.offsets, off = [], 0
        for n in sizes:
            self.offsets.append(off)
            off += n
        self.views = {}
        for (name, shape), o, n in zip(PARAMS, self.offsets, sizes):
            v = self.flat[o:o + n].view(shape)
            v.copy_(params[name].detach().float())
            self.views[name] = v

    def like(self):
        return {name: self.flat.new_empty(0) for name in self.views}


def rebuild_update(buffer, offsets, weight, count, shard, grad_flat, fp):
    """Write into grad_flat (fp32, FlatParams layout) the update terms of the pairs shard = (start, stop):
    G_P = -(1 / count) sum_j w_j a_j b_j^T. offsets: int64 [60, pairs]; weight: fp32 [pairs].
    Returns (device status word, number of the library's kernels enqueued)."""
    start, stop = shard
    pairs = offsets.shape[1] if offsets.dim() == 2 else -1
    if offsets.dtype != torch.int64 or tuple(offsets.shape) != (len(PARAMS), pairs) or tuple(weight.shape) != (pairs,):
        raise ValueError(f'offsets int64 [{len(PARAMS)}, pairs] and weight [pairs]: got {offsets.dtype} '
                         f'{tuple(offsets.shape)}, {tuple(weight.shape)}')
    if not 0 <= start <= stop <= pairs:
        raise ValueError(f'shard {shard} outside the {pairs} pairs')
    if buffer.dtype != torch.float32 or buffer.dim() != 1:
        raise ValueError('buffer: a 1-D fp32 tensor')
    if grad_flat.dtype != torch.float32 or grad_flat.shape != fp.flat.shape or not grad_flat.is_contiguous():
        raise ValueError(f'grad_flat: contiguous fp32 {tuple(fp.flat.shape)}')
    _lib.require_cuda(buffer, offsets, weight, grad_flat)
    L = _lib.lib()
    stream = _lib.stream_handle(buffer.device)
    n = stop - start
    scale = -1.0 / count
    status = torch.zeros(_lib.STATUS_BYTES // 4, dtype=torch.int32, device=buffer.device)
    w = weight[start:stop].float().contiguous()
    launches = 0
    for k, (name, shape) in enumerate(PARAMS):
        g = grad_flat[fp.offsets[k]:fp.offsets[k] + math.prod(shape)]
        if n == 0:
            g.zero_()
            continue
        off = offsets[k, start:stop].contiguous()
        if len(shape) == 2 and shape[0] >= GEMM_MIN_ROWS and shape[1] % GEMM_N == 0:
            out, inn = shape
            kp = -(-n // 4) * 4  # whole 16-byte rows of fp32; the GEMM reads zeros past them
            a = torch.empty((out, kp), dtype=torch.float32, device=buffer.device)
            b = torch.empty((inn, kp), dtype=torch.float32, device=buffer.device)
            _lib.check(L.noise_rank1_operands_f32(buffer.data_ptr(), off.data_ptr(), w.data_ptr(), scale, 0, out, n,
                                                  kp, a.data_ptr(), stream), 'noise_rank1_operands_f32')
            _lib.check(L.noise_rank1_operands_f32(buffer.data_ptr(), off.data_ptr(), None, 1.0, out, inn, n, kp,
                                                  b.data_ptr(), stream), 'noise_rank1_operands_f32')
            _lib.check(L.noise_gemm_tf32_tn(a.data_ptr(), b.data_ptr(), g.data_ptr(), out, inn, kp,
                                            status.data_ptr(), stream), 'noise_gemm_tf32_tn')
            launches += 3
        else:
            one_d = len(shape) == 1
            n_out, n_in = (1, shape[0]) if one_d else shape
            _lib.check(L.noise_rank1_small(buffer.data_ptr(), off.data_ptr(), w.data_ptr(), scale, n_out, n_in,
                                           int(one_d), n, g.data_ptr(), stream), 'noise_rank1_small')
            launches += 1
    return status, launches


class AdamW:
    """torch.optim.AdamW(lr, betas, eps, weight_decay=0) over a flat fp32 tensor, on the library's kernel."""

    def __init__(self, flat, lr=1e-3, betas=(0.5, 0.95), eps=1e-8):
        self.flat, self.lr, self.betas, self.eps = flat, lr, betas, eps
        self.exp_avg = torch.zeros_like(flat)
        self.exp_avg_sq = torch.zeros_like(flat)
        self.t = 0

    def step(self, grad, lr=None):
        if grad.dtype != torch.float32 or grad.shape != self.flat.shape or not grad.is_contiguous():
            raise ValueError(f'grad: contiguous fp32 {tuple(self.flat.shape)}')
        _lib.require_cuda(self.flat, grad)
        self.t += 1
        _lib.check(_lib.lib().noise_adam_step(self.flat.data_ptr(), self.exp_avg.data_ptr(),
                                              self.exp_avg_sq.data_ptr(), grad.data_ptr(), self.flat.numel(),
                                              float(self.lr if lr is None else lr), float(self.betas[0]),
                                              float(self.betas[1]), float(self.eps), self.t,
                                              _lib.stream_handle(self.flat.device)), 'noise_adam_step')


class EggrollTrainer:
    """EGGROLL with AdamW on the CUDA path; ranks of a torch.distributed group share the population."""

    def __init__(self, params, pairs, rows, sigma=SIGMA, lr=1e-3, betas=(0.5, 0.95), seed=0, rank=0, world=1,
                 buffer=None, noise_size=NOISE, shard_update=True):
        self.device = params['lm_head.weight'].device
        self.pairs, self.rows, self.seed, self.rank, self.world = pairs, rows, seed, rank, world
        self.fp = FlatParams(params, self.device)
        self.params = self.fp.views
        buffer = noise_buffer(self.device, seed, noise_size) if buffer is None else buffer
        self.pop = Population(self.params, pairs, sigma, seed, rank, world, buffer=buffer)
        self.buffer = buffer
        self.grad = torch.zeros_like(self.fp.flat)
        self.opt = AdamW(self.fp.flat, lr, betas)
        self.shard_update = shard_update
        members = member_layout(pairs, rows)[0]
        if members % world:
            raise ValueError('every rank must evaluate the same number of members')

    PHASES = ('forward', 'fitness', 'rebuild', 'all_reduce', 'adamw')

    def step(self, tokens, step, lr=None, timer=None):
        """tokens: int64 [rows, T + 1] on the device. Returns the population's mean loss (a device scalar).

        timer: optional list; CUDA events recorded on the current stream at the start and after each phase are
        appended to it as (phase, event) pairs (phases: PHASES; 'forward' includes the re-pack of the bf16 weights
        after the previous update). ``launches`` holds the number of the library's kernels the step enqueued."""
        def mark(name):
            if timer is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                timer.append((name, ev))

        mark('start')
        offsets = step_offsets(self.pairs, step, self.device, self.seed, self.buffer.numel())
        packs = self.pop.packed.refresh().packs
        _, losses = self.pop.evaluate(tokens, step, offsets=offsets)
        mark('forward')
        weight, count = fitness_weights(losses, self.pairs)
        mark('fitness')
        shard = pair_shard(self.pairs, self.rank, self.world) if self.shard_update else (0, self.pairs)
        self.status, rebuilt = rebuild_update(self.buffer, offsets, weight, count, shard, self.grad, self.fp)
        mark('rebuild')
        if self.shard_update and self.world > 1:
            torch.distributed.all_reduce(self.grad)
        mark('all_reduce')
        self.opt.step(self.grad, lr)
        self.pop.packed.invalidate()
        mark('adamw')
        self.launches = packs + self.pop.launches + rebuilt + 1
        return losses.mean()


def phase_ms(timer):
    """Milliseconds per phase from the (phase, event) list ``EggrollTrainer.step(timer=...)`` filled (after a
    synchronize), summed over the steps it covers."""
    out = {}
    for (_, e0), (name, e1) in zip(timer, timer[1:]):
        if name == 'start':
            continue
        out[name] = out.get(name, 0.0) + e0.elapsed_time(e1)
    return out
