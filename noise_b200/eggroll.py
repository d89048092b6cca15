"""EGGROLL bookkeeping around the CUDA population forward (reference archive/10M/train/val/eggroll.py).

- ``make_params``: the reference's ``make_model`` weights (eggroll.py:38-53 over utils/model.py:149-175), drawn with
  the same torch calls in the same order on the given device, so on CUDA they equal the reference's bit for bit.
- ``noise_buffer`` / ``step_offsets``: the fixed N(0, 1) buffer and the per-step slice offsets (eggroll.py:114-120).
- ``member_layout``: members, per-sequence and per-rank counts, each member's direction, sign and row (:134-143).
- ``Population``: one rank's share of a population evaluated through ``population_loss_offsets``, its fitness
  all-gathered over NCCL (eggroll.py:147-150).
"""
import torch

from .population import NAMES, PARAMS, PackedGPT, has_ve, member_offsets, population_loss_offsets, N_LAYER, N_EMBD

NOISE = 2 ** 28
SIGMA = 0.002


@torch.no_grad()
def make_params(device, seed=0):
    """name -> fp32 tensor on ``device``: init_weights (utils/model.py:149-175), the CUDA bf16 round trip of wte and the
    value embeddings (:171-175), then the c_proj re-draw U(+-1.5 sqrt(3 / fan_in)) (eggroll.py:45-49)."""
    device = torch.device(device)
    torch.manual_seed(seed)
    p = {name: torch.empty(shape, device=device) for name, shape in PARAMS}
    s = 3 ** 0.5 * N_EMBD ** -0.5
    torch.nn.init.normal_(p['transformer.wte.weight'], mean=0.0, std=1.0)
    torch.nn.init.normal_(p['lm_head.weight'], mean=0.0, std=0.001)
    for i in range(N_LAYER):
        pre = f'transformer.h.{i}.'
        for n in ('attn.c_q', 'attn.c_k', 'attn.c_v'):
            torch.nn.init.uniform_(p[pre + n + '.weight'], -s, s)
        torch.nn.init.zeros_(p[pre + 'attn.c_proj.weight'])
        torch.nn.init.uniform_(p[pre + 'mlp.c_fc.weight'], -s, s)
        torch.nn.init.zeros_(p[pre + 'mlp.c_proj.weight'])
    p['resid_lambdas'].fill_(1.0)
    p['x0_lambdas'].fill_(0.1)
    for i in range(N_LAYER):
        if has_ve(i):
            torch.nn.init.uniform_(p[f'value_embeds.{i}.weight'], -s, s)
    for i in range(N_LAYER):
        if has_ve(i):
            torch.nn.init.zeros_(p[f'transformer.h.{i}.attn.ve_gate.weight'])
    if device.type == 'cuda':
        for name in p:
            if name == 'transformer.wte.weight' or name.startswith('value_embeds.'):
                p[name] = p[name].bfloat16().float()
    for i in range(N_LAYER):
        for name in (f'transformer.h.{i}.attn.c_proj.weight', f'transformer.h.{i}.mlp.c_proj.weight'):
            scale = 1.5 * (3 / p[name].shape[1]) ** 0.5
            torch.nn.init.uniform_(p[name], -scale, scale)
    return p


def noise_buffer(device, seed=0, size=NOISE):
    """eggroll.py:114."""
    return torch.randn(size, device=device, generator=torch.Generator(device).manual_seed(seed))


def step_offsets(pairs, step, device, seed=0, size=NOISE):
    """int64 [60, pairs]: row P = offsets of parameter P (named_parameters order) for this step, drawn exactly as
    eggroll.py:117-120 draws them (one generator seeded 1_000_003 * seed + step, parameters in order)."""
    g = torch.Generator(device).manual_seed(1_000_003 * seed + step)
    return torch.stack([torch.randint(0, size - sum(shape), (pairs,), device=device, generator=g)
                        for _, shape in PARAMS])


def member_layout(pairs, rows, world=1, rank=0, device='cpu'):
    """(members, per_seq, per_rank, directions [members], signs +-1 [members], row [members]) (eggroll.py:134-143)."""
    members = max(2 * pairs, 2 * rows)
    per_seq, per_rank = members // rows, members // world
    i = torch.arange(members, device=device)
    sign = torch.where(i % 2 == 0, 1.0, -1.0)
    return members, per_seq, per_rank, (i % (2 * pairs)) // 2, sign, i // per_seq


class Population:
    """One rank's population evaluation: members [rank * per_rank, (rank + 1) * per_rank) of a population of
    ``2 * pairs`` antithetic members, each member scored on its rows of ``tokens`` (eggroll.py:131-150).

    ``evaluate(tokens, step)`` returns this rank's per-member losses (mean or summed over tokens, and over the rows of
    ``rows_per_member`` when every member reads several rows) and, with ``gather``, the all-gathered population
    losses; ``launches`` counts the CUDA kernels of the library issued by the last call."""

    def __init__(self, params, pairs, sigma=SIGMA, seed=0, rank=0, world=1, chunk=512, buffer=None):
        self.p, self.pairs, self.sigma, self.seed, self.rank, self.world = params, pairs, sigma, seed, rank, world
        self.device = params['lm_head.weight'].device
        self.packed = PackedGPT(params)
        self.buffer = noise_buffer(self.device, seed) if buffer is None else buffer
        self.chunk = chunk
        self.launches = 0

    def evaluate(self, tokens, step, rows_per_member=1, reduction='mean', gather=True, offsets=None):
        """tokens: int64 [rows, T + 1] on the device. With rows_per_member == 1 the reference layout holds (members
        split evenly over the rows); with rows_per_member == rows every member reads every row and its losses add up
        over the rows (each member scores 8 x 2048 tokens)."""
        from . import _lib
        rows = tokens.shape[0]
        members, per_seq, per_rank, directions, signs, row_of = member_layout(
            self.pairs, rows if rows_per_member == 1 else 1, self.world, self.rank, self.device)
        if offsets is None:
            offsets = step_offsets(self.pairs, step, self.device, self.seed, self.buffer.numel())
        first = self.rank * per_rank
        losses = torch.zeros(per_rank, device=self.device)
        self.launches = 0
        chunk = self.chunk
        if rows_per_member == 1:  # a launch shares one token row: chunks may not straddle rows (eggroll.py:143)
            while per_seq % chunk or per_rank % chunk:
                chunk //= 2
        for start in range(first, first + per_rank, chunk):
            sel = slice(start, min(start + chunk, first + per_rank))
            off = member_offsets(offsets, directions[sel])
            sign = signs[sel] * self.sigma
            row_list = [int(row_of[sel.start])] if rows_per_member == 1 else range(rows)
            for r in row_list:
                idx, tgt = tokens[r, :-1], tokens[r, 1:]
                out = population_loss_offsets(self.packed, self.buffer, off, sign, idx, tgt, reduction)
                self.launches += _lib.launches()
                losses[sel.start - first:sel.stop - first] += out
        if gather and self.world > 1:
            gathered = [torch.empty_like(losses) for _ in range(self.world)]
            torch.distributed.all_gather(gathered, losses)
            return losses, torch.cat(gathered)
        return losses, losses
