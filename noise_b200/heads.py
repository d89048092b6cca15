"""The identity phase's head-sharding kernels (reference train/speedrun/run.py:3694-3804) on libnoise_b200.so.

Same names, arguments and results as the reference's functions:

- ``pack_heads_kernel(qs, ks, vals, outs, targets, lses)`` -> the (H, L, n, PACK) bf16 all_to_all send buffer
  (run.py:3718-3731): every head's q, k, v, attention-output and target pieces and its lse's fp32 bits.
- ``head_prep_fused(got, cos, sin, b, t)`` -> the received heads' RoPE'd and normed queries and keys, values, hubs,
  fp32 queries, the keys' pair features, lse, hub . o, square norms and steps (run.py:3781-3796).
- ``id_head_scores(got, rope32, back, b, t)``: head_prep, then the query- and key-moment credits into
  back (W, L, 3, N, 64) bf16 (run.py:3799-3803), in one library call.
"""
import ctypes

import torch

from . import _lib

H, HD, PACK = 8, 64, 5 * 64 + 2
KEY_SIGMA, NORM_EPS = 0.003, 1e-6  # run.py's KEY_SIGMA and NORM_EPS


def _two_byte(t, what):
    if t.element_size() != 2 or t.stride(-1) != 1:
        raise ValueError(f'{what}: a 16-bit tensor with a unit last stride')
    return t


def _pieces(qs, ks, vals, outs, targets, lses):
    """noise_head_pieces_t per layer from each layer's (tokens, D) pieces and its lse (rows, H, t); returns (pieces,
    tensors to keep alive, n, t, layers)."""
    n, t = qs[0].shape[0], lses[0].shape[-1]
    layers = len(qs)
    if not len(ks) == len(vals) == len(outs) == len(targets) == len(lses) == layers:
        raise ValueError('q, k, v, o, target and lse: one piece of each per layer')
    if t < 1 or n % t:
        raise ValueError(f'{n} tokens are not whole sequences of lse\'s {t}')
    checked = []
    for i, group in enumerate(zip(qs, ks, vals, outs, targets, lses)):
        *mats, lse = group
        mats = [_two_byte(m.detach(), 'q, k, v, o, target') for m in mats]
        if any(tuple(m.shape) != (n, H * HD) for m in mats):
            raise ValueError(f'layer {i}: q, k, v, o, target must be ({n}, {H * HD})')
        lse = lse.detach().float().contiguous()
        if tuple(lse.shape) != (n // t, H, t):
            raise ValueError(f'layer {i}: lse {tuple(lse.shape)}, expected {(n // t, H, t)}')
        checked.append((mats, lse))
    _lib.require_cuda(*(z for mats, lse in checked for z in mats + [lse]))
    pieces = (_lib.HeadPieces * layers)()
    keep = []
    for i, (mats, lse) in enumerate(checked):
        keep += mats + [lse]
        p = pieces[i]
        p.q, p.k, p.v, p.o, p.target = (m.data_ptr() for m in mats)
        p.q_stride, p.k_stride, p.v_stride, p.o_stride, p.target_stride = (m.stride(0) for m in mats)
        p.lse = lse.data_ptr()
    return pieces, keep, n, t, layers


def pack_heads_kernel(qs, ks, vals, outs, targets, lses):
    """identity_grad's (H, L, n, PACK) all_to_all send buffer from each layer's (tokens, D) pieces and its lse
    (rows, H, t) (run.py:3718-3731)."""
    pieces, keep, n, t, layers = _pieces(qs, ks, vals, outs, targets, lses)
    dev = qs[0].device
    out = torch.empty(H, layers, n, PACK, device=dev, dtype=torch.bfloat16)
    _lib.check(_lib.lib().noise_pack_heads(pieces, layers, n, t, out.data_ptr(), _lib.stream_handle(dev)),
               'noise_pack_heads')
    return out


def _prep_struct(got, b, t, keep_k32):
    w, layers, n, _ = got.shape
    rows = layers * b
    dev = got.device
    new = lambda *s, dtype=torch.float32: torch.empty(*s, device=dev, dtype=dtype)
    bf = torch.bfloat16
    q16, k16, v16, hub16 = (new(rows, t, HD, dtype=bf) for _ in range(4))
    q32 = new(rows, t, HD)
    k32 = new(rows, t, HD) if keep_k32 else None
    pairs = (new(rows, t, HD, dtype=bf), new(rows, t, 2 * HD, dtype=bf), new(rows, t, HD // 2, dtype=bf))
    lse, hub_out, sq_q, sq_k, steps_q, steps_k = (new(rows, t) for _ in range(6))
    s = _lib.HeadPrep()
    s.q16, s.k16, s.v16, s.hub16, s.q32 = (z.data_ptr() for z in (q16, k16, v16, hub16, q32))
    s.k32 = k32.data_ptr() if k32 is not None else None
    s.f2, s.f4, s.xy = (z.data_ptr() for z in pairs)
    s.lse, s.hub_out, s.sq_q, s.sq_k, s.steps_q, s.steps_k = (z.data_ptr() for z in
                                                             (lse, hub_out, sq_q, sq_k, steps_q, steps_k))
    return s, (q16, k16, v16, hub16, q32, pairs, lse, hub_out, sq_q, sq_k, steps_q, steps_k), k32


def _got(got, b, t):
    got = _two_byte(got.detach(), 'got')
    if got.dim() != 4 or got.shape[-1] != PACK or not got.is_contiguous():
        raise ValueError(f'got: contiguous (W, L, N, {PACK})')
    w, _, n, _ = got.shape
    if w * n != b * t:
        raise ValueError('got holds W * N = b * t tokens per layer')
    _lib.require_cuda(got)
    return got


def _rope(cos, sin, t):
    """fp32 contiguous RoPE tables with at least t rows of HD / 2 on the device (the kernels read rows 0 .. t - 1)."""
    cos, sin = (z.detach().float().contiguous() for z in (cos, sin))
    for z in (cos, sin):
        if z.dim() != 2 or z.shape[0] < t or z.shape[1] != HD // 2:
            raise ValueError(f'cos / sin: ({t} or more, {HD // 2}), got {tuple(z.shape)}')
    _lib.require_cuda(cos, sin)
    return cos, sin


def head_prep_fused(got, cos, sin, b: int, t: int):
    """The received heads' RoPE'd queries and keys, values, hubs, lse and square norms and steps from got (W, L, N,
    PACK), in one kernel pass (run.py:3781-3796). Returns (q16, k16, v16, hub16, q32, (f2, f4, xy), lse, hub_out,
    sq_q, sq_k, steps_q, steps_k)."""
    got = _got(got, b, t)
    w, layers, n, _ = got.shape
    cos, sin = _rope(cos, sin, t)
    s, result, _ = _prep_struct(got, b, t, keep_k32=False)
    _lib.check(_lib.lib().noise_head_prep(got.data_ptr(), w, layers, n, cos.data_ptr(), sin.data_ptr(), t, KEY_SIGMA,
                                          NORM_EPS, ctypes.byref(s), _lib.stream_handle(got.device)),
               'noise_head_prep')
    return result


def id_head_scores(got, rope32, back, b, t):
    """head_prep_fused, then the query credits into back[:, :, 0] and the key credits and value sums into
    back[:, :, 1], back[:, :, 2] (run.py:3799-3803); back: bf16 (W, L, 3, N, 64), written in place."""
    got = _got(got, b, t)
    w, layers, n, _ = got.shape
    if back.dtype != torch.bfloat16 or tuple(back.shape) != (w, layers, 3, n, HD) or not back.is_contiguous():
        raise ValueError('back: contiguous bf16 (W, L, 3, N, 64)')
    cos, sin = _rope(*rope32, t)
    _lib.require_cuda(back)
    L = _lib.lib()
    nbytes = L.noise_id_head_scores_workspace_bytes(w, layers, n)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=got.device)
    _lib.check(L.noise_id_head_scores(got.data_ptr(), w, layers, n, cos.data_ptr(), sin.data_ptr(), t, KEY_SIGMA,
                                      NORM_EPS, back.data_ptr(), ws.data_ptr(), nbytes,
                                      _lib.stream_handle(got.device)), 'noise_id_head_scores')


class _DeviceArray:
    """A device allocation of the library, seen by torch through the CUDA array interface (no copy)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {'shape': tuple(shape), 'typestr': typestr, 'data': (ptr, False),
                                         'version': 3, 'strides': None}


class HeadExchange:
    """identity_grad's two all_to_all_single exchanges (run.py:3887-3888 heads in, :3905-3906 heads out) over peer
    memory: the pack writes every head's rows straight into the owning rank's buffer over NVLink, the heads-out
    credits are stored the same way, and a bounded wait on per-source epoch flags replaces heads_in.wait() /
    heads_out.wait() (run.py:3902, 3912). One buffer per rank, shared with CUDA IPC (no multicast).

    ``send_heads(qs, ks, vals, outs, targets, lses)`` + ``wait_heads()`` -> got, the (H, L, n, PACK) bf16 buffer
    dist.all_to_all_single(got, pack_heads_kernel(...)) fills (with world 8: (W, L, N, PACK)); ``send_back(back)``
    + ``wait_back()`` -> got2 = all_to_all_single of back (W, L, 3, n, 64). Per step the order is send_heads,
    wait_heads, send_back, wait_back (what the reference does): a rank sends the next step's heads only after it has
    the previous step's credits back, which is also what tells it every peer has finished reading its buffer.
    Construct and ``close()`` collectively on every rank of ``group``."""

    def __init__(self, layers, tokens, seq_len, group=None, wait_seconds=60.0, device=None):
        import torch.distributed as dist
        self.dist = dist if dist.is_available() and dist.is_initialized() else None
        self.group = group
        self.world = self.dist.get_world_size(group) if self.dist else 1
        self.rank = self.dist.get_rank(group) if self.dist else 0
        if H % self.world or self.world > 8:
            raise ValueError('the exchange needs a world size dividing 8')
        self.layers, self.n, self.t = layers, tokens, seq_len
        self.device = torch.device('cuda', torch.cuda.current_device()) if device is None else device
        self.limit_ns = int(wait_seconds * 1e9)
        got_bytes = H * layers * tokens * PACK * 2
        back_bytes = self.world * layers * 3 * tokens * HD * 2
        self.got_offset = 1024
        self.got2_offset = (self.got_offset + got_bytes + 255) // 256 * 256
        L = _lib.lib()
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            _lib.check(L.noise_exchange_alloc(self.got2_offset + back_bytes, ctypes.byref(ptr), handle),
                       'noise_exchange_alloc')
        self.ptr = ptr.value
        handles = [handle.raw]
        if self.dist:
            handles = [None] * self.world
            self.dist.all_gather_object(handles, handle.raw, group=group)
        self.opened = []
        self.peers = _lib.Peers()
        self.peers.rank, self.peers.world = self.rank, self.world
        for w in range(self.world):
            if w == self.rank:
                self.peers.base[w] = self.ptr
                continue
            p = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                _lib.check(L.noise_exchange_open(ctypes.create_string_buffer(handles[w], 64), ctypes.byref(p)),
                           'noise_exchange_open')
            self.opened.append(p.value)
            self.peers.base[w] = p.value
        as_bf16 = lambda off, shape: torch.as_tensor(_DeviceArray(self.ptr + off, shape, '<i2'),
                                                     device=self.device).view(torch.bfloat16)
        self.got = as_bf16(self.got_offset, (H, layers, tokens, PACK))
        self.got2 = as_bf16(self.got2_offset, (self.world, layers, 3, tokens, HD))
        self.status = torch.zeros(_lib.STATUS_BYTES, dtype=torch.uint8, device=self.device)
        self.epoch = [0, 0]
        self.phase = 'send_heads'

    def _step(self, want, nxt):
        if self.phase != want:
            raise RuntimeError(f'HeadExchange: {want} called out of order (expected {self.phase})')
        self.phase = nxt

    def send_heads(self, qs, ks, vals, outs, targets, lses):
        """pack_heads_kernel + the heads-in all_to_all_single, one kernel (run.py:3885-3888)."""
        self._step('send_heads', 'wait_heads')
        pieces, keep, n, t, layers = _pieces(qs, ks, vals, outs, targets, lses)
        if (n, t, layers) != (self.n, self.t, self.layers):
            raise ValueError('send_heads: pieces do not match the exchange\'s layers / tokens / seq_len')
        self.epoch[0] += 1
        _lib.check(_lib.lib().noise_pack_heads_peer(pieces, layers, n, t, ctypes.byref(self.peers), self.got_offset,
                                                    0, self.epoch[0], _lib.stream_handle(self.device)),
                   'noise_pack_heads_peer')
        self._keep = keep

    def wait_heads(self):
        """heads_in.wait() (run.py:3902): the stream waits until every rank's heads have landed; returns got."""
        self._step('wait_heads', 'send_back')
        _lib.check(_lib.lib().noise_exchange_wait(ctypes.byref(self.peers), 0, self.epoch[0], self.limit_ns,
                                                  self.status.data_ptr(), _lib.stream_handle(self.device)),
                   'noise_exchange_wait')
        return self.got

    def send_back(self, back):
        """The heads-out all_to_all_single of back (W, L, 3, n, 64) bf16 (run.py:3905-3906)."""
        self._step('send_back', 'wait_back')
        if back.dtype != torch.bfloat16 or tuple(back.shape) != tuple(self.got2.shape) or not back.is_contiguous():
            raise ValueError('back: contiguous bf16 (W, L, 3, n, 64)')
        _lib.require_cuda(back)
        self.epoch[1] += 1
        _lib.check(_lib.lib().noise_alltoall_peer(back.data_ptr(), back[0].numel() * 2, ctypes.byref(self.peers),
                                                  self.got2_offset, 1, self.epoch[1],
                                                  _lib.stream_handle(self.device)), 'noise_alltoall_peer')
        self._keep_back = back

    def wait_back(self):
        """heads_out.wait() (run.py:3912); returns got2."""
        self._step('wait_back', 'send_heads')
        _lib.check(_lib.lib().noise_exchange_wait(ctypes.byref(self.peers), 1, self.epoch[1], self.limit_ns,
                                                  self.status.data_ptr(), _lib.stream_handle(self.device)),
                   'noise_exchange_wait')
        return self.got2

    def read_status(self):
        """The device status word of the waits (0, or NOISE_DEVICE_TIMEOUT); synchronises the stream."""
        return _lib.read_status(self.status)

    def close(self):
        """Unmap the peers' buffers and free this rank's (collective: every rank calls it)."""
        torch.cuda.synchronize(self.device)
        L = _lib.lib()
        for p in self.opened:
            _lib.check(L.noise_exchange_close(p), 'noise_exchange_close')
        self.opened = []
        if self.dist:
            self.dist.barrier(group=self.group)
        if self.ptr:
            self.got = self.got2 = None
            _lib.check(L.noise_exchange_free(self.ptr), 'noise_exchange_free')
            self.ptr = None
