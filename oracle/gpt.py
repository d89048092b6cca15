"""CPU restatement of Noise's fixed GPT (reference ``utils/model.py``) — test infrastructure only.

The weights live in a plain ``dict`` name -> tensor with the reference's ``named_parameters()`` names and order
(``resid_lambdas``, ``x0_lambdas``, ``transformer.wte.weight``, the blocks, ``lm_head.weight``,
``value_embeds.{1,3,5,7}.weight``), so they can be handed to the reference, to this oracle and to the CUDA path alike.

The forward uses a dense masked softmax instead of flex attention; the arithmetic is the reference's:
- ``norm``: RMS norm without weight, eps = finfo(dtype).eps (model.py:46-47, ``F.rms_norm`` with ``eps=None``).
- ``apply_rotary_emb``: half-split rotation with bf16 cos/sin tables, base 1e4 (model.py:55-58, 177-183).
- attention: key s visible to query t iff 0 <= t - s <= window, scale 1/sqrt(64) (model.py:17-31).
- value embeddings on blocks 1, 3, 5, 7 gated by 2 sigmoid(W_g x[:32]) (model.py:50-52, 87-90).
- ReLU^2 MLP (model.py:100-107); mixing resid * x + x0l * x0 (model.py:198-199); softcap 15 tanh(z / 15) and
  cross-entropy (model.py:202-209).
"""
import math

import torch
from torch.nn import functional as F

N_LAYER, N_HEAD, N_EMBD, VOCAB, SEQ = 8, 8, 512, 4096, 2048
HEAD_DIM = N_EMBD // N_HEAD
VE_GATE_CHANNELS = 32
WINDOWS = [1024, 1024, 1024, 2048, 1024, 1024, 1024, 2048]  # model.py:185-191, pattern SSSL, last block L
ROTARY_LEN = SEQ * 10


def has_ve(i, n_layer=N_LAYER):
    """Value embeddings on every other block counting back from the last (model.py:50-52)."""
    return i % 2 == (n_layer - 1) % 2


def param_shapes():
    """(name, shape) in the reference's ``named_parameters()`` order (60 tensors, 37,749,776 values)."""
    out = [('resid_lambdas', (N_LAYER,)), ('x0_lambdas', (N_LAYER,)), ('transformer.wte.weight', (VOCAB, N_EMBD))]
    for i in range(N_LAYER):
        pre = f'transformer.h.{i}.'
        out += [(pre + 'attn.c_q.weight', (N_EMBD, N_EMBD)), (pre + 'attn.c_k.weight', (N_EMBD, N_EMBD)),
                (pre + 'attn.c_v.weight', (N_EMBD, N_EMBD)), (pre + 'attn.c_proj.weight', (N_EMBD, N_EMBD))]
        if has_ve(i):
            out.append((pre + 'attn.ve_gate.weight', (N_HEAD, VE_GATE_CHANNELS)))
        out += [(pre + 'mlp.c_fc.weight', (4 * N_EMBD, N_EMBD)), (pre + 'mlp.c_proj.weight', (N_EMBD, 4 * N_EMBD))]
    out.append(('lm_head.weight', (VOCAB, N_EMBD)))
    out += [(f'value_embeds.{i}.weight', (VOCAB, N_EMBD)) for i in range(N_LAYER) if has_ve(i)]
    return out


def _construction_draws():
    """Consume the CPU generator exactly as ``GPT(GPTConfig())`` does when it is built on the CPU: nn.Embedding's
    normal init, nn.Linear's kaiming-uniform init, in module-construction order (model.py:124-147)."""
    torch.nn.Embedding(VOCAB, N_EMBD)
    for i in range(N_LAYER):
        for _ in range(4):
            torch.nn.Linear(N_EMBD, N_EMBD, bias=False)
        if has_ve(i):
            torch.nn.Linear(VE_GATE_CHANNELS, N_HEAD, bias=False)
        torch.nn.Linear(N_EMBD, 4 * N_EMBD, bias=False)
        torch.nn.Linear(4 * N_EMBD, N_EMBD, bias=False)
    torch.nn.Linear(N_EMBD, VOCAB, bias=False)
    for i in range(N_LAYER):
        if has_ve(i):
            torch.nn.Embedding(VOCAB, N_EMBD)


def init_weights(seed=0, constructed=True, eggroll=False, cuda_embeddings=False):
    """The reference's weights as a dict.

    constructed=True reproduces ``torch.manual_seed(seed); GPT(GPTConfig()); init_weights()`` on the CPU (the
    constructor's own draws come first). eggroll=True reproduces EGGROLL's ``make_model`` (eggroll.py:38-53): built on
    the meta device (no constructor draws), ``init_weights`` (model.py:149-175), then every ``c_proj`` re-drawn
    U(+-1.5 sqrt(3 / fan_in)) in ``named_modules`` order. cuda_embeddings=True applies the bf16 round trip that
    ``init_weights`` gives wte and the value embeddings on a CUDA device (model.py:171-175) before make_model turns
    them back to fp32.
    """
    torch.manual_seed(seed)
    if constructed and not eggroll:
        _construction_draws()
    w = {name: torch.empty(shape) for name, shape in param_shapes()}
    s = 3 ** 0.5 * N_EMBD ** -0.5
    torch.nn.init.normal_(w['transformer.wte.weight'], mean=0.0, std=1.0)
    torch.nn.init.normal_(w['lm_head.weight'], mean=0.0, std=0.001)
    for i in range(N_LAYER):
        pre = f'transformer.h.{i}.'
        torch.nn.init.uniform_(w[pre + 'attn.c_q.weight'], -s, s)
        torch.nn.init.uniform_(w[pre + 'attn.c_k.weight'], -s, s)
        torch.nn.init.uniform_(w[pre + 'attn.c_v.weight'], -s, s)
        torch.nn.init.zeros_(w[pre + 'attn.c_proj.weight'])
        torch.nn.init.uniform_(w[pre + 'mlp.c_fc.weight'], -s, s)
        torch.nn.init.zeros_(w[pre + 'mlp.c_proj.weight'])
    w['resid_lambdas'].fill_(1.0)
    w['x0_lambdas'].fill_(0.1)
    for i in range(N_LAYER):
        if has_ve(i):
            torch.nn.init.uniform_(w[f'value_embeds.{i}.weight'], -s, s)
    for i in range(N_LAYER):
        if has_ve(i):
            torch.nn.init.zeros_(w[f'transformer.h.{i}.attn.ve_gate.weight'])
    if cuda_embeddings:
        for name in w:
            if name == 'transformer.wte.weight' or name.startswith('value_embeds.'):
                w[name] = w[name].bfloat16().float()
    if eggroll:
        for i in range(N_LAYER):
            for name in (f'transformer.h.{i}.attn.c_proj.weight', f'transformer.h.{i}.mlp.c_proj.weight'):
                scale = 1.5 * (3 / w[name].shape[1]) ** 0.5
                torch.nn.init.uniform_(w[name], -scale, scale)
    return w


def informative_weights(seed=0):
    """EGGROLL's make_model weights with the parts that are inert at initialisation made active, for parity tests:
    at init the LM head has std 1e-3, so every loss sits at ln 4096 whatever the body computes, and the value-embedding
    gates are zero. Here the LM head is N(0, 2 / sqrt(512)) (logits of std ~2), the ve gates N(0, 0.5) and the mixing
    scalars spread around their init, so per-member losses depend on every block."""
    w = init_weights(seed, eggroll=True)
    g = torch.Generator().manual_seed(10_000 + seed)
    w['lm_head.weight'] = torch.randn(VOCAB, N_EMBD, generator=g) * (2 / N_EMBD ** 0.5)
    for i in range(N_LAYER):
        if has_ve(i):
            w[f'transformer.h.{i}.attn.ve_gate.weight'] = torch.randn(N_HEAD, VE_GATE_CHANNELS, generator=g) * 0.5
    w['resid_lambdas'] = 1 + 0.2 * torch.randn(N_LAYER, generator=g)
    w['x0_lambdas'] = 0.1 + 0.2 * torch.randn(N_LAYER, generator=g)
    return w


def rotary(seq_len=ROTARY_LEN, head_dim=HEAD_DIM, base=10000):
    """bf16 cos, sin tables [seq_len, head_dim / 2] (model.py:177-183)."""
    inv_freq = 1.0 / base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)
    t = torch.arange(seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return freqs.cos().bfloat16(), freqs.sin().bfloat16()


def norm(x):
    """model.py:46-47."""
    return F.rms_norm(x, (x.size(-1),))


def apply_rotary_emb(x, cos, sin):
    """x [..., T, H, D] with cos/sin [T, D/2] (model.py:55-58)."""
    d = x.shape[-1] // 2
    cos, sin = cos[:, None, :], sin[:, None, :]
    x1, x2 = x[..., :d], x[..., d:]
    return torch.cat([x1 * cos + x2 * sin, x1 * -sin + x2 * cos], -1)


def window_allowed(length, window, device=None):
    """[T, T] bool: query t sees key s iff 0 <= t - s <= window (model.py:17-21)."""
    t = torch.arange(length, device=device)
    lag = t[:, None] - t[None, :]
    return (lag >= 0) & (lag <= window)


def attention(q, k, v, window):
    """Dense restatement of model.py:24-31 on [B, T, H, D] tensors (fp32 or fp64)."""
    qh, kh, vh = (z.transpose(1, 2) for z in (q, k, v))
    scores = (qh @ kh.transpose(-1, -2)) * HEAD_DIM ** -0.5
    scores = scores.masked_fill(~window_allowed(q.shape[1], window, q.device), float('-inf'))
    return (scores.softmax(-1) @ vh).transpose(1, 2)


def attention_autocast(q, k, v, window):
    """model.py:24-31 as it runs under ``torch.autocast(..., torch.bfloat16)``: flex attention's autocast rule
    (torch._higher_order_ops.flex_attention, ``_flex_attention_autocast_impl`` in the torch of this build, 2.11)
    casts q, k and v to bf16 before attending; the scores of the bf16 values are formed in fp32, softmax in fp32,
    the probabilities rounded to bf16 for the product with v, and the output is bf16."""
    qh, kh, vh = (z.transpose(1, 2).bfloat16() for z in (q, k, v))
    scores = (qh.float() @ kh.float().transpose(-1, -2)) * HEAD_DIM ** -0.5
    scores = scores.masked_fill(~window_allowed(q.shape[1], window, q.device), float('-inf'))
    p = scores.softmax(-1).bfloat16()
    return (p.float() @ vh.float()).bfloat16().float().transpose(1, 2)


def forward(w, idx, targets=None, loss_reduction='mean', dtype=torch.float32):
    """GPT.forward (model.py:193-209) in ``dtype`` on the CPU. idx [B, T] int64."""
    B, T = idx.shape
    w = {k: v.to(dtype) for k, v in w.items()}
    cos, sin = (z[:T].to(dtype) for z in rotary())
    x = x0 = norm(w['transformer.wte.weight'][idx])
    for i in range(N_LAYER):
        pre = f'transformer.h.{i}.'
        x = w['resid_lambdas'][i] * x + w['x0_lambdas'][i] * x0
        h = norm(x)
        q = (h @ w[pre + 'attn.c_q.weight'].t()).view(B, T, N_HEAD, HEAD_DIM)
        k = (h @ w[pre + 'attn.c_k.weight'].t()).view(B, T, N_HEAD, HEAD_DIM)
        v = (h @ w[pre + 'attn.c_v.weight'].t()).view(B, T, N_HEAD, HEAD_DIM)
        if has_ve(i):
            ve = w[f'value_embeds.{i}.weight'][idx].view(B, T, N_HEAD, HEAD_DIM)
            gate = 2 * torch.sigmoid(h[..., :VE_GATE_CHANNELS] @ w[pre + 'attn.ve_gate.weight'].t())
            v = v + gate.unsqueeze(-1) * ve
        q, k = norm(apply_rotary_emb(q, cos, sin)), norm(apply_rotary_emb(k, cos, sin))
        y = torch.stack([attention(q[b:b + 1], k[b:b + 1], v[b:b + 1], WINDOWS[i]) for b in range(B)]).view(B, T, -1)
        x = x + y @ w[pre + 'attn.c_proj.weight'].t()
        x = x + F.relu(norm(x) @ w[pre + 'mlp.c_fc.weight'].t()).square() @ w[pre + 'mlp.c_proj.weight'].t()
    logits = (norm(x) @ w['lm_head.weight'].t())[..., :VOCAB]
    logits = 15 * torch.tanh(logits / 15)
    if targets is None:
        return logits
    return F.cross_entropy(logits.reshape(-1, VOCAB), targets.reshape(-1), ignore_index=-1, reduction=loss_reduction)


def zipf_tokens(rows, length, seed=0, s=1.1, vocab=VOCAB):
    """Synthetic stand-in for the FineWeb rows: ids ~ Zipf(s) over ranks 1..vocab mapped to ids 0..vocab-1, drawn
    with ``torch.multinomial`` from a CPU generator seeded ``seed``; int64 [rows, length]."""
    p = torch.arange(1, vocab + 1, dtype=torch.float64) ** -s
    g = torch.Generator().manual_seed(seed)
    return torch.multinomial((p / p.sum()).float(), rows * length, replacement=True, generator=g).view(rows, length)


def param_count():
    return sum(math.prod(s) for _, s in param_shapes())
