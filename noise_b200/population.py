"""Drop-in population-perturbed forward (the hot path of EGGROLL, reference archive/10M/train/val/eggroll.py).

``population_loss(model, p, noise, sign, idx, targets)`` has the reference's signature and meaning
(eggroll.py:66-103): the cross-entropy of m rank-1-perturbed copies of the fixed GPT on one token row, one value per
member, computed as under ``torch.autocast('cuda', torch.bfloat16)``. The work runs in libnoise_b200.so
(tcgen05 GEMMs with the rank-1 term fused into their epilogues, windowed attention, LM head fused with the softcap and
cross-entropy); this module only packs the weights, describes the noise slices and calls the C ABI.

``population_loss_offsets`` is the same forward fed straight from EGGROLL's fixed noise buffer and per-step offsets
(eggroll.py:114-128): member j of parameter P reads buffer[offsets[P, direction_j] : ... + out + in] in place, so the
reference's ``noise()`` gather and ``repeat_interleave`` copies (eggroll.py:141-142) disappear.
"""
import ctypes

import torch

from . import _lib

N_LAYER, N_HEAD, HEAD_DIM, N_EMBD, VOCAB = 8, 8, 64, 512, 4096
WINDOWS = [1024, 1024, 1024, 2048, 1024, 1024, 1024, 2048]


def has_ve(i):
    return i % 2 == (N_LAYER - 1) % 2


def param_shapes():
    """(name, shape) in the reference GPT's named_parameters() order (utils/model.py:123-147)."""
    out = [('resid_lambdas', (N_LAYER,)), ('x0_lambdas', (N_LAYER,)), ('transformer.wte.weight', (VOCAB, N_EMBD))]
    for i in range(N_LAYER):
        pre = f'transformer.h.{i}.'
        out += [(pre + f'attn.{n}.weight', (N_EMBD, N_EMBD)) for n in ('c_q', 'c_k', 'c_v', 'c_proj')]
        if has_ve(i):
            out.append((pre + 'attn.ve_gate.weight', (N_HEAD, 32)))
        out += [(pre + 'mlp.c_fc.weight', (4 * N_EMBD, N_EMBD)), (pre + 'mlp.c_proj.weight', (N_EMBD, 4 * N_EMBD))]
    out.append(('lm_head.weight', (VOCAB, N_EMBD)))
    out += [(f'value_embeds.{i}.weight', (VOCAB, N_EMBD)) for i in range(N_LAYER) if has_ve(i)]
    return out


PARAMS = param_shapes()
NAMES = [n for n, _ in PARAMS]
INDEX = {n: i for i, n in enumerate(NAMES)}


def rotary_tables(length, device, base=10000):
    """bf16 cos, sin [length, 32] as utils/model.py:177-183 computes them on ``device``."""
    inv_freq = 1.0 / base ** (torch.arange(0, HEAD_DIM, 2, dtype=torch.float32, device=device) / HEAD_DIM)
    t = torch.arange(length, dtype=torch.float32, device=device)
    freqs = torch.outer(t, inv_freq)
    return freqs.cos().bfloat16().contiguous(), freqs.sin().bfloat16().contiguous()


class PackedGPT:
    """The weights as the C ABI consumes them (noise_gpt_t): matrices packed to bf16 once, embeddings fp32.

    ``refresh()`` re-packs only when a source tensor changed (new storage or an in-place update)."""

    def __init__(self, params, device=None, cos=None, sin=None):
        self.params = params
        head = params.get('lm_head.weight')  # a missing one is reported by refresh's shape check
        self.device = torch.device(device) if device is not None else (head.device if head is not None else None)
        self._key = None
        self._cos, self._sin = cos, sin
        self.refresh()

    def invalidate(self):
        """Force a re-pack at the next refresh (after the weights were written in place by a raw kernel, which does
        not bump torch's version counter)."""
        self._key = None

    def _source_key(self):
        return tuple((t.data_ptr(), t._version) for t in (self.params[n] for n in NAMES))

    def _pack(self, dst, src):
        self.packs += 1
        src = src.detach().float().contiguous()
        _lib.check(_lib.lib().noise_pack_bf16(src.data_ptr(), dst.data_ptr(), src.numel(),
                                              _lib.stream_handle(self.device)), 'noise_pack_bf16')

    def refresh(self):
        """Re-pack if a source changed; ``packs`` = the pack kernels this call launched."""
        p = self.params
        for name, shape in PARAMS:  # each is packed into a slot of exactly this size
            if name not in p or tuple(p[name].shape) != shape:
                raise ValueError(f'{name}: expected shape {shape}, got '
                                 f'{tuple(p[name].shape) if name in p else "nothing"}')
        key = self._source_key()
        self.packs = 0
        if key == self._key:
            return self
        dev = self.device
        for t in p.values():
            _lib.require_cuda(t)
        if self._cos is not None:
            for z in (self._cos, self._sin):
                if z.dtype != torch.bfloat16 or z.dim() != 2 or z.shape[1] != HEAD_DIM // 2:
                    raise ValueError(f'RoPE tables: bf16 [positions, {HEAD_DIM // 2}], got {z.dtype} {tuple(z.shape)}')
            _lib.require_cuda(self._cos, self._sin)
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.wqkv, self.wproj, self.wfc, self.wmproj, self.wgate, self.ve = [], [], [], [], [], []
        for i in range(N_LAYER):
            pre = f'transformer.h.{i}.'
            qkv = torch.empty((3 * N_EMBD, N_EMBD), **bf)
            for k, n in enumerate(('c_q', 'c_k', 'c_v')):
                self._pack(qkv[k * N_EMBD:(k + 1) * N_EMBD], p[pre + f'attn.{n}.weight'])
            proj = torch.empty((N_EMBD, N_EMBD), **bf)
            self._pack(proj, p[pre + 'attn.c_proj.weight'])
            fc = torch.empty((4 * N_EMBD, N_EMBD), **bf)
            self._pack(fc, p[pre + 'mlp.c_fc.weight'])
            mproj = torch.empty((N_EMBD, 4 * N_EMBD), **bf)
            self._pack(mproj, p[pre + 'mlp.c_proj.weight'])
            self.wqkv.append(qkv)
            self.wproj.append(proj)
            self.wfc.append(fc)
            self.wmproj.append(mproj)
            self.wgate.append(p[pre + 'attn.ve_gate.weight'].detach().float().contiguous() if has_ve(i) else None)
            self.ve.append(p[f'value_embeds.{i}.weight'].detach().float().contiguous() if has_ve(i) else None)
        self.whead = torch.empty((VOCAB, N_EMBD), **bf)
        self._pack(self.whead, p['lm_head.weight'])
        self.wte = p['transformer.wte.weight'].detach().float().contiguous()
        self.resid = p['resid_lambdas'].detach().float().contiguous()
        self.x0 = p['x0_lambdas'].detach().float().contiguous()
        if self._cos is None:
            self._cos, self._sin = rotary_tables(2048, dev)
        s = _lib.GPT()
        for i in range(N_LAYER):
            s.wqkv[i], s.wproj[i] = self.wqkv[i].data_ptr(), self.wproj[i].data_ptr()
            s.wfc[i], s.wmproj[i] = self.wfc[i].data_ptr(), self.wmproj[i].data_ptr()
            s.wgate[i] = self.wgate[i].data_ptr() if self.wgate[i] is not None else None
            s.ve[i] = self.ve[i].data_ptr() if self.ve[i] is not None else None
        s.whead, s.wte = self.whead.data_ptr(), self.wte.data_ptr()
        s.resid_lambdas, s.x0_lambdas = self.resid.data_ptr(), self.x0.data_ptr()
        s.cos, s.sin = self._cos.data_ptr(), self._sin.data_ptr()
        self.struct = s
        self._key = key
        return self

    def check_length(self, length):
        """The RoPE tables cover positions 0 .. length - 1 (the kernels read one row per position)."""
        if self._cos.shape[0] < length or self._sin.shape[0] < length:
            raise ValueError(f'the RoPE tables hold {self._cos.shape[0]} positions, the rows {length}')


_packed = {}


def _packed_for(model, p):
    key = id(p)
    cached = _packed.get(key)
    if cached is None or cached.params is not p:
        cos = sin = None
        if model is not None and hasattr(model, 'cos'):
            cos = model.cos.reshape(-1, HEAD_DIM // 2)[:2048].contiguous()
            sin = model.sin.reshape(-1, HEAD_DIM // 2)[:2048].contiguous()
        _packed.clear()
        cached = _packed[key] = PackedGPT(p, cos=cos, sin=sin)
    return cached.refresh()


def _row_args(sign, idx, targets, reduction):
    """sign fp32 [m], idx / targets int64 [T] as contiguous CUDA tensors, after the checks every entry makes."""
    sign = sign.detach().float().contiguous()
    idx = idx.detach().long().contiguous()
    targets = targets.detach().long().contiguous()
    _lib.require_cuda(sign, idx, targets)
    if sign.dim() != 1 or idx.dim() != 1 or targets.shape != idx.shape:
        raise ValueError('sign must be [m]; idx and targets [T] of the same length')
    if reduction not in _lib.REDUCTION:
        raise ValueError(f'reduction must be one of {sorted(_lib.REDUCTION)}')
    return sign, idx, targets


def _run(packed, slices, keep, sign, idx, targets, reduction):
    dev = packed.device
    sign, idx, targets = _row_args(sign, idx, targets, reduction)
    m, length = sign.shape[0], idx.shape[0]
    packed.check_length(length)
    L = _lib.lib()
    nbytes = L.noise_population_workspace_bytes(m, length)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    losses = torch.empty((m, length) if reduction == 'none' else (m,), dtype=torch.float32, device=dev)
    arr = (_lib.Slice * len(NAMES))(*slices)
    rc = L.noise_population_loss(ctypes.byref(packed.struct), arr, sign.data_ptr(), idx.data_ptr(),
                                 targets.data_ptr(), m, length, _lib.REDUCTION[reduction], losses.data_ptr(),
                                 ws.data_ptr(), nbytes, _lib.stream_handle(dev))
    _lib.check(rc, 'noise_population_loss')
    losses._noise_workspace = ws  # keeps the scratch (and its status word) alive with the result
    del keep
    return losses


def population_loss(model, p, noise, sign, idx, targets, reduction='mean'):
    """Mean (or summed) cross-entropy [m] of m perturbed models on one sequence (eggroll.py:66-103); with
    reduction='none' the per-token losses [m, T] the reference averages (eggroll.py:101-102).

    model: the reference GPT module (its RoPE tables are used when present) or None; p: parameter name -> tensor;
    noise: name -> (a [m, out], b [m, in]) for matrices and embeddings, eps [m, numel] for the mixing scalars;
    sign [m] (+-sigma); idx, targets [T] int64 with T % 128 == 0."""
    packed = _packed_for(model, p)
    m = sign.shape[0] if sign.dim() == 1 else -1
    slices, keep = [], []
    for name, shape in PARAMS:
        v = noise[name]
        if isinstance(v, (tuple, list)):
            a, b = (t.detach().float() for t in v)
            if a.stride(-1) != 1 or b.stride(-1) != 1:
                a, b = a.contiguous(), b.contiguous()
            if len(shape) != 2 or tuple(a.shape) != (m, shape[0]) or tuple(b.shape) != (m, shape[1]):
                raise ValueError(f'{name}: a [m, out] and b [m, in] for m = {m} members of a {shape} parameter, got '
                                 f'{tuple(a.shape)}, {tuple(b.shape)}')
            _lib.require_cuda(a, b)
            keep += [a, b]
            slices.append(_lib.Slice(a.data_ptr(), b.data_ptr(), None, a.stride(0), b.stride(0)))
        else:
            e = v.detach().float()
            if e.stride(-1) != 1:
                e = e.contiguous()
            if len(shape) != 1 or tuple(e.shape) != (m, shape[0]):
                raise ValueError(f'{name}: eps [m, {shape[0]}] for m = {m} members, got {tuple(e.shape)}')
            _lib.require_cuda(e)
            keep.append(e)
            slices.append(_lib.Slice(e.data_ptr(), e.data_ptr(), None, e.stride(0), e.stride(0)))
    return _run(packed, slices, keep, sign, idx, targets, reduction)


def member_offsets(offsets, directions):
    """int64 [60, m]: offsets [60, pairs] (one row per parameter, named_parameters order) gathered at the members'
    directions."""
    return offsets.index_select(1, directions.to(offsets.device)).contiguous()


def _offset_slices(packed, buffer, member_off, members):
    """The 60 noise_slice_t of the in-place noise path (checked: fp32 CUDA buffer, int64 CUDA offsets [60, m])."""
    _lib.require_cuda(buffer, member_off)
    if buffer.dtype != torch.float32 or buffer.dim() != 1:
        raise ValueError('buffer must be a 1-D fp32 tensor')
    if member_off.dtype != torch.int64 or member_off.dim() != 2 or member_off.shape != (len(NAMES), members):
        raise ValueError(f'member_off must be int64 [{len(NAMES)}, m] with m = len(sign)')
    if buffer.device != packed.device or member_off.device != packed.device:
        raise ValueError('buffer and member_off must be on the weights\' device')
    member_off = member_off.contiguous()
    base = buffer.data_ptr()
    slices = []
    for k, (name, shape) in enumerate(PARAMS):
        off = member_off[k].data_ptr()
        out = shape[0] if len(shape) == 2 else 0
        slices.append(_lib.Slice(base, base + 4 * out, off, 0, 0))
    return slices, member_off


def population_loss_offsets(packed, buffer, member_off, sign, idx, targets, reduction='mean'):
    """population_loss with every member's (a, b) read in place from the fixed noise buffer: member j of parameter P
    uses a = buffer[off : off + out], b = buffer[off + out : off + out + in] with off = member_off[P, j]
    (eggroll.py:122-128). member_off: int64 [60, m] device tensor (``member_offsets``)."""
    packed = packed.refresh()
    slices, member_off = _offset_slices(packed, buffer, member_off, sign.shape[0])
    return _run(packed, slices, [member_off, buffer], sign, idx, targets, reduction)


def population_loss_offsets_noalloc(packed, buffer, member_off, sign, idx, targets, reduction='mean'):
    """``population_loss_offsets`` through ``noise_population_loss_noalloc``, for callers that cannot allocate device
    memory while they evaluate: the C entry point takes no workspace and runs in the library's static device scratch
    (48 MiB per GPU: members x tokens up to about 4,400 rows). Only the returned loss vector is allocated here, by
    torch. The call runs with the weights' device current, on that device's current stream. Calls that overlap on the
    GPU race on the shared scratch. Its device status word is read with ``_lib.read_static_status(device)``."""
    packed = packed.refresh()
    slices, member_off = _offset_slices(packed, buffer, member_off, sign.shape[0])
    sign, idx, targets = _row_args(sign, idx, targets, reduction)
    m, length = sign.shape[0], idx.shape[0]
    packed.check_length(length)
    dev = packed.device
    losses = torch.empty((m, length) if reduction == 'none' else (m,), dtype=torch.float32, device=dev)
    arr = (_lib.Slice * len(NAMES))(*slices)
    with torch.cuda.device(dev):
        rc = _lib.lib().noise_population_loss_noalloc(ctypes.byref(packed.struct), arr, sign.data_ptr(),
                                                      idx.data_ptr(), targets.data_ptr(), m, length,
                                                      _lib.REDUCTION[reduction], losses.data_ptr(),
                                                      _lib.stream_handle(dev))
    _lib.check(rc, 'noise_population_loss_noalloc')
    return losses


def gpt_loss(model, p, idx, targets, loss_reduction='mean'):
    """GPT.forward(idx, targets, loss_reduction) (utils/model.py:193-209) of the un-perturbed model on B distinct
    rows: softcap 15, cross-entropy with ignore_index -1; 'mean' and 'sum' give a 0-d tensor, 'none' [B * T].

    The numerics are the population forward's (bf16 tensor-core linears, fp32 accumulation, fp32 residual stream and
    embeddings), i.e. the reference run under ``torch.autocast('cuda', torch.bfloat16)`` with EGGROLL's fp32
    embeddings. model: the reference GPT module (for its RoPE tables) or None; p: parameter name -> tensor;
    idx, targets int64 [B, T] with T % 128 == 0, T <= 2048."""
    packed = _packed_for(model, p)
    dev = packed.device
    idx = idx.detach().long().contiguous()
    targets = targets.detach().long().contiguous()
    _lib.require_cuda(idx, targets)
    if idx.dim() != 2 or targets.shape != idx.shape:
        raise ValueError('idx and targets must be [B, T] of the same shape')
    rows, length = idx.shape
    packed.check_length(length)
    if loss_reduction not in _lib.REDUCTION:
        raise ValueError(f'loss_reduction must be one of {sorted(_lib.REDUCTION)}')
    L = _lib.lib()
    nbytes = L.noise_gpt_workspace_bytes(rows, length)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    out = torch.empty((rows * length,) if loss_reduction == 'none' else (), dtype=torch.float32, device=dev)
    rc = L.noise_gpt_loss(ctypes.byref(packed.struct), idx.data_ptr(), targets.data_ptr(), rows, length,
                          _lib.REDUCTION[loss_reduction], out.data_ptr(), ws.data_ptr(), nbytes,
                          _lib.stream_handle(dev))
    _lib.check(rc, 'noise_gpt_loss')
    out._noise_workspace = ws
    return out


def head_loss(x, weight, targets, vocab=VOCAB):
    """dust.head_loss (train/val/dust.py:94-99): norm(x), the LM head, softcap 15 and per-token cross-entropy
    (ignore_index -1, reduction 'none') -> fp32 [N * T]. x [N, T, 512] (fp32; other dtypes are widened), weight
    [>= vocab, 512] (bf16, or fp32 rounded to bf16 as autocast does), targets [N, T]; vocab must be 4096 and N * T a
    multiple of 128."""
    if vocab != VOCAB:
        raise ValueError(f'vocab must be {VOCAB}')
    dev = x.device
    xs = x.detach().reshape(-1, N_EMBD).float().contiguous()
    w = weight.detach()[:VOCAB]
    if tuple(w.shape) != (VOCAB, N_EMBD):
        raise ValueError(f'weight: [>= {VOCAB}, {N_EMBD}], got {tuple(weight.shape)}')
    w = (w if w.dtype == torch.bfloat16 else w.bfloat16()).contiguous()
    tg = targets.detach().reshape(-1).long().contiguous()
    _lib.require_cuda(xs, w, tg)
    rows = xs.shape[0]
    if tg.shape[0] != rows:
        raise ValueError('targets must hold one id per row of x')
    L = _lib.lib()
    nbytes = L.noise_head_loss_workspace_bytes(rows)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
    out = torch.empty(rows, dtype=torch.float32, device=dev)
    rc = L.noise_head_loss(xs.data_ptr(), w.data_ptr(), tg.data_ptr(), rows, out.data_ptr(), ws.data_ptr(), nbytes,
                           _lib.stream_handle(dev))
    _lib.check(rc, 'noise_head_loss')
    out._noise_workspace = ws
    return out
