"""Generate the golden fixtures under tests/golden/ by running the reference itself on the CPU.

Runs only where the reference checkout is readable (pass its path as argv[1] or set NOISE_REFERENCE); the GPU box
never runs this script, it only reads the committed ``*.pt`` files. Reference files used:

- ``utils/model.py``: GPT(GPTConfig()), init_weights, forward (config 1 of the benchmark plan).
- ``archive/10M/train/val/eggroll.py``: make_model, lowrank, lowrank_embed, population_loss, Eggroll.offsets/noise
  and one Eggroll.step (member layout, fitness, seed-rebuilt gradient).
- ``train/speedrun/moment_kernels.py``: _implicit_key_context under TRITON_INTERPRET=1 (its dots are fp32 tf32 dots,
  which the interpreter evaluates in fp32), then every credit kernel (lse/center on bf16 inputs, value pass, key
  scan, query moments, key moments) under the interpreter with its bf16 dot and bf16 rounding fixed
  (patch_triton_interpreter: a fix of the tool's arithmetic; the reference kernels run unmodified).

Compiled flex attention does not lower on the CPU, so ``utils.model.flex`` is switched to the eager
``flex_attention`` (same function, no compilation). The noise buffer is shrunk from 2**28 to 2**20 values
(``eggroll.NOISE``) and the chunk from 256 to 2 pairs (``eggroll.CHUNK``) so one step finishes in seconds.

- ``utils/model.py`` and ``eggroll.py`` again on weights whose blocks are all active (``informative.pt``): GPT.forward
  and population_loss (fp32 and CPU autocast) with oracle.gpt.informative_weights loaded by load_state_dict.

- ``train/speedrun/run.py``: pack_heads_kernel, head_prep_fused and id_head_scores (the identity phase's head
  sharding) under the same patched interpreter, on tests/golden/heads_inputs.py's seeded inputs.

- ``train/val/run.py`` (its `recipe` section): the track-1 readout scorers' ops noise_record::future_scores,
  ::future_query_response (CPU paths) and ::key_response, ::routed_response (Triton kernels, patched interpreter).

- ``train/val/run.py`` (its `readout` section, through the file's own section loader): the true-path readout's
  scorer kernels stats_kernel, staged_kernel, readout_kernel (patched interpreter).

- ``train/speedrun/run.py``: the identity phase's readout cycle top_credit and coordinate_change (compiled helpers
  as their original functions, the Triton weights kernel under the patched interpreter).

- ``train/val/dust.py``: block_forward (its compiled function as the original) with jitter at every site.

- ``train/speedrun/id_kernels.py``: hidden_credits_fused, at_b_layers, square_credit_grads (their Triton kernels
  under the patched interpreter) on id_inputs.py's seeded inputs.

Usage: python tests/golden/make_golden.py /path/to/reference [fixture,...]
"""
import importlib.util
import os
import sys
from pathlib import Path

os.environ.setdefault('TRITON_INTERPRET', '1')  # read when triton is first imported; only the credit fixture uses it
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from credit_inputs import credit_inputs  # noqa: E402
SMALL_NOISE = 2 ** 20


def load_reference(root):
    sys.path.insert(0, str(root))
    import utils.model as model
    from torch.nn.attention.flex_attention import flex_attention
    model.flex = flex_attention
    spec = importlib.util.spec_from_file_location('ref_eggroll', root / 'archive/10M/train/val/eggroll.py')
    eggroll = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(eggroll)
    return model, eggroll


def checksums(sd):
    """Per tensor: (sum, sum |x|, first 8 values) — enough to pin an init draw for draw."""
    return {k: (float(v.double().sum()), float(v.double().abs().sum()), v.flatten()[:8].clone())
            for k, v in sd.items()}


def zipf(rows, length, seed=0):
    p = torch.arange(1, 4097, dtype=torch.float64) ** -1.1
    g = torch.Generator().manual_seed(seed)
    return torch.multinomial((p / p.sum()).float(), rows * length, replacement=True, generator=g).view(rows, length)


def golden_forward(model):
    """Config 1: torch.manual_seed(0); GPT(GPTConfig()); init_weights(); fp32 eval forward on Zipf rows."""
    torch.manual_seed(0)
    gpt = model.GPT(model.GPTConfig())
    gpt.init_weights()
    gpt.eval()
    tokens = zipf(4, 2049, seed=0)
    with torch.no_grad():
        ce = gpt(tokens[:, :-1], tokens[:, 1:].contiguous(), loss_reduction='none').view(4, 2048)
    torch.save(dict(tokens=tokens.short(), ce=ce, loss_sum=ce.double().sum(),
                    weights=checksums(dict(gpt.named_parameters()))), HERE / 'gpt_forward.pt')
    print('gpt_forward: sum CE', float(ce.double().sum()))


def golden_population(eggroll, length=2048, pairs=2, sigma=0.002):
    """population_loss on 2 antithetic pairs (4 members) of EGGROLL's make_model weights, fp32 (native CPU) and
    under CPU bf16 autocast, plus the noise map pieces (offsets, gathered slices)."""
    eggroll.NOISE = SMALL_NOISE
    model = eggroll.make_model(torch.device('cpu'), 0)
    es = eggroll.Eggroll(model, pairs)
    offsets = es.offsets(step=1)
    directions = torch.tensor([0, 0, 1, 1])
    nz = es.noise(offsets, directions)
    sign = torch.tensor([sigma, -sigma]).repeat(pairs)
    tokens = zipf(1, length + 1, seed=1)[0]
    idx, tgt = tokens[:-1], tokens[1:].contiguous()
    with torch.no_grad():
        fp32 = eggroll.population_loss(model, es.params, nz, sign, idx, tgt)
        with torch.autocast('cpu', dtype=torch.bfloat16):
            bf16 = eggroll.population_loss(model, es.params, nz, sign, idx, tgt)
    gathered = {k: (tuple(t[:, :4].clone() for t in v) if isinstance(v, tuple) else v[:, :4].clone())
                for k, v in nz.items()}
    torch.save(dict(length=length, pairs=pairs, sigma=sigma, noise_size=SMALL_NOISE, buffer_sum=es.buffer.double().sum(),
                    buffer_head=es.buffer[:16].clone(), offsets={k: v.clone() for k, v in offsets.items()},
                    directions=directions, tokens=tokens.short(), loss_fp32=fp32, loss_autocast=bf16.float(),
                    gathered=gathered, weights=checksums(es.params)), HERE / f'population_T{length}.pt')
    print(f'population T={length}: fp32', fp32.tolist(), 'autocast', bf16.float().tolist())


def golden_informative(model, eggroll):
    """The reference's GPT.forward and population_loss on weights whose every block matters: EGGROLL's make_model
    weights with an active LM head, value-embedding gates and mixing scalars (oracle.gpt.informative_weights, the
    parity tests' weights), loaded into the reference's own modules with load_state_dict (strict). At the reference's
    initialisation the LM head (std 1e-3) puts every loss at ln 4096 and GPT(GPTConfig())'s zero c_proj makes every
    block inert, so these fixtures are the ones that pin attention, MLP, norms and value embeddings.

    - forward: GPT(GPTConfig()) fp32 eval forward, loss_reduction='none', on 2 Zipf rows x 2048 (seed 3).
    - population_T256: 16 antithetic pairs (32 members), one Zipf row of 256 (seed 1), step 1 offsets.
    - population_T2048: 4 pairs (8 members), one Zipf row of 2048 (seed 1), step 1 offsets.
    Each population case runs fp32 (the CPU's native arithmetic) and under CPU bf16 autocast."""
    sys.path.insert(0, str(HERE.parents[1]))
    from oracle.gpt import informative_weights  # the input generator only; outputs come from the reference
    w = informative_weights(0)
    out = dict(weights=checksums(w))
    torch.manual_seed(0)
    gpt = model.GPT(model.GPTConfig())
    gpt.load_state_dict(w, strict=True)
    gpt.eval()
    tokens = zipf(2, 2049, seed=3)
    with torch.no_grad():
        ce = gpt(tokens[:, :-1], tokens[:, 1:].contiguous(), loss_reduction='none').view(2, 2048)
    out['forward'] = dict(tokens=tokens.short(), ce=ce.clone())
    print('informative forward: mean CE', float(ce.mean()))
    eggroll.NOISE = SMALL_NOISE
    for length, pairs in ((256, 16), (2048, 4)):
        net = eggroll.make_model(torch.device('cpu'), 0)
        net.load_state_dict(w, strict=True)
        es = eggroll.Eggroll(net, pairs)
        offsets = es.offsets(step=1)
        directions = torch.arange(2 * pairs) // 2
        nz = es.noise(offsets, directions)
        sign = torch.tensor([eggroll.SIGMA, -eggroll.SIGMA]).repeat(pairs)
        row = zipf(1, length + 1, seed=1)[0]
        idx, tgt = row[:-1], row[1:].contiguous()
        with torch.no_grad():
            fp32 = eggroll.population_loss(net, es.params, nz, sign, idx, tgt)
            with torch.autocast('cpu', dtype=torch.bfloat16):
                bf16 = eggroll.population_loss(net, es.params, nz, sign, idx, tgt).float()
        out[f'population_T{length}'] = dict(length=length, pairs=pairs, sigma=eggroll.SIGMA, noise_size=SMALL_NOISE,
                                             step=1, directions=directions, tokens=row.short(), loss_fp32=fp32,
                                             loss_autocast=bf16)
        fit32, fit16 = fp32[1::2] - fp32[0::2], bf16[1::2] - bf16[0::2]
        print(f'informative population T={length}: mean loss {float(fp32.mean()):.4f}; autocast-vs-fp32 fitness '
              f'gap {float((fit16 - fit32).abs().max() / fit32.std()):.4f} of the fitness std')
    torch.save(out, HERE / 'informative.pt')


def golden_step(eggroll, length=256, pairs=4, rows=2):
    """One Eggroll.step with CHUNK = 2 pairs: member layout, losses, fitness weights and the rebuilt gradient."""
    eggroll.NOISE = SMALL_NOISE
    eggroll.CHUNK = 2
    model = eggroll.make_model(torch.device('cpu'), 0)
    es = eggroll.Eggroll(model, pairs)
    es.loss = eggroll.population_loss
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, betas=(0.5, 0.95), eps=1e-8, weight_decay=0.0)
    tokens = zipf(rows, length + 1, seed=2)
    grads = {}
    orig = opt.step

    def capture(*a, **k):
        for n, p in model.named_parameters():
            grads[n] = p.grad.clone()
        return orig(*a, **k)

    opt.step = capture
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter('ignore')
        mean_loss = es.step(tokens[:, :-1].contiguous(), tokens[:, 1:].contiguous(), opt, step=3)
    small = {n: g for n, g in grads.items() if g.numel() <= 4096}
    corner = {n: g[:8, :8].clone() for n, g in grads.items() if g.dim() == 2}
    torch.save(dict(length=length, pairs=pairs, rows=rows, chunk=2, step=3, noise_size=SMALL_NOISE,
                    tokens=tokens.short(), mean_loss=mean_loss, grad_small=small, grad_corner=corner,
                    grad_sums={n: float(g.double().sum()) for n, g in grads.items()},
                    grad_abs={n: float(g.double().abs().sum()) for n, g in grads.items()}),
               HERE / 'eggroll_step.pt')
    print('eggroll step: mean loss', mean_loss)


def golden_implicit(root):
    """lse and center from the reference Triton kernel under the interpreter (fp32 inputs, tf32 dots evaluated in
    fp32), rows = 2, T = 256, window 128 and 256. Inputs are regenerated from the CPU generator seed by the test:
    q, k, v = randn / 8 and hub = randn, drawn in that order."""
    spec = importlib.util.spec_from_file_location('ref_moments', root / 'train/speedrun/moment_kernels.py')
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    g = torch.Generator().manual_seed(5)
    rows, t = 2, 256
    q, k, v, hub = (torch.randn(rows, t, 64, generator=g) / 8 for _ in range(4))
    hub = hub * 8
    out = {}
    for window in (128, 256):
        lse, center = mk._implicit_key_context(q, k, v, hub, window, edges=True)
        out[window] = (lse.clone(), center.clone())
    torch.save(dict(seed=5, rows=rows, length=t, out=out), HERE / 'implicit_key_context.pt')
    print('implicit_key_context: ok')


def patch_triton_interpreter():
    """Make the Triton interpreter compute what the GPU computes (a fix of the tool, not of the reference kernels).

    The interpreter stores bf16 tensors as raw uint16 bits. Its tl.dot multiplies those bits as integers, and its
    fp32 -> bf16 cast truncates, where the hardware rounds to nearest even. Patched: bf16 dot operands are widened to
    fp32 before the numpy matmul (bf16 products are exact in fp32; accumulation is fp32 as on the tensor cores) and
    fp32 <-> bf16 casts go through torch's round-to-nearest-even conversion."""
    import numpy as np
    import triton.language as tl
    from triton.runtime import interpreter as ti

    def widen(h):
        if h.dtype.scalar != tl.bfloat16:
            return h
        return ti.TensorHandle((h.data.astype(np.uint32) << 16).view(np.float32), tl.float32)

    def narrow(data):
        t = torch.from_numpy(np.ascontiguousarray(data, dtype=np.float32))
        return t.bfloat16().view(torch.int16).numpy().view(np.uint16).reshape(np.shape(data))

    dot = ti.InterpreterBuilder.create_dot
    cast = ti.InterpreterBuilder.cast_impl
    fp_to_fp = ti.InterpreterBuilder.create_fp_to_fp

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        return dot(self, widen(a), widen(b), d, input_precision, max_num_imprecise_acc)

    def cast_impl(self, src, dst_type):
        s, d = src.dtype.scalar, dst_type.scalar
        if s == tl.float32 and d == tl.bfloat16:
            return ti.TensorHandle(narrow(src.data), d)
        if s == tl.bfloat16 and d == tl.float32:
            return ti.TensorHandle(widen(src).data, d)
        return cast(self, src, dst_type)

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        if src.dtype.scalar in (tl.float32, tl.bfloat16) and dst_type.scalar in (tl.float32, tl.bfloat16):
            return cast_impl(self, src, dst_type)
        return fp_to_fp(self, src, dst_type, rounding_mode)

    ti.InterpreterBuilder.create_dot = create_dot
    ti.InterpreterBuilder.cast_impl = cast_impl
    ti.InterpreterBuilder.create_fp_to_fp = create_fp_to_fp


def interpreter_libdevice():
    """numpy float32 versions of the libdevice functions the credit kernels call (log1p, expm1, rsqrt); the interpreter
    has no libdevice of its own. Installed as the interpreted module's ``libdevice`` global."""
    import types

    import numpy as np
    import triton.language as tl
    from triton.runtime import interpreter as ti

    def unary(fn):
        def f(x, *args, **kwargs):
            data = fn(np.asarray(x.handle.data, dtype=np.float32)).astype(np.float32)
            return tl.core.tensor(ti.TensorHandle(data, x.handle.dtype.scalar), x.type)
        return f

    return types.SimpleNamespace(log1p=unary(np.log1p), expm1=unary(np.expm1),
                                 rsqrt=unary(lambda v: np.float32(1.0) / np.sqrt(v)))


def golden_credit(root, rows=2, t=256):
    """Every credit kernel of the reference (moment_kernels.py) on Cut-like inputs, through the patched interpreter:
    implicit_key_context (bf16 inputs), the value pass, the key scan (with and without the value credit), query
    moments and the identity phase's key moments. Inputs are regenerated by credit_inputs(rows, t, seed)."""
    patch_triton_interpreter()
    spec = importlib.util.spec_from_file_location('ref_moments_patched', root / 'train/speedrun/moment_kernels.py')
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    mk.libdevice = interpreter_libdevice()
    x = credit_inputs(rows, t)
    b16 = lambda z: z.bfloat16().contiguous()
    q16, k16, v16, h16 = b16(x['qp']), b16(x['kp']), b16(x['values']), b16(x['hub'])
    out = {}
    for window in (128, t):
        lse, center = mk._implicit_key_context(q16, k16, v16, h16, window, edges=True)
        raw_value = mk._value_pass(q16, k16, lse, x['hub'], window)
        key = mk._key_scan(x['qp'], x['kp'], x['k_raw'], lse, x['values'], x['hub'], center, x['cos'], x['sin'],
                           window, 0.003, False)[0]
        key_v, raw_v = mk._key_scan(x['qp'], x['kp'], x['k_raw'], lse, x['values'], x['hub'], center, x['cos'],
                                    x['sin'], window, 0.003, True)
        sq = x['q_raw'].square().sum(-1)
        steps = 0.01 * (sq / 64).sqrt().clamp(min=1e-6)
        qs = torch.empty(1, rows, t, 64, dtype=torch.bfloat16)
        mk._moment_query_scores(q16, k16, v16, h16, x['q_raw'].unsqueeze(0).contiguous(), sq, x['kp'], x['cos'],
                                x['sin'], lse, center, steps, qs, 4, window)
        out[window] = dict(lse=lse.clone(), center=center.clone(), raw_value=raw_value.clone(), key=key.clone(),
                           key_v=key_v.clone(), raw_v=raw_v.clone(), query=qs[0].float().clone(), sq=sq, steps=steps)
    # identity phase: full causal key moments (receivers s >= t), lse / hub_out of the full causal context
    lse, center = mk._implicit_key_context(q16, k16, v16, h16, t, edges=True)
    sqk = x['k_raw'].square().sum(-1)
    stepsk = 0.01 * (sqk / 64).sqrt().clamp(min=1e-6)
    ko = torch.empty(1, rows, t, 64)
    kv = torch.empty(1, rows, t, 64)
    mk._moment_key_scores(q16, k16, v16, h16, x['k_raw'].unsqueeze(0).contiguous(), sqk, x['qp'], x['cos'], x['sin'],
                          lse, center, stepsk, ko, kv, 2)
    out['keys'] = dict(lse=lse.clone(), center=center.clone(), sq=sqk, steps=stepsk, out=ko[0].clone(),
                       values=kv[0].clone())
    torch.save(dict(rows=rows, length=t, seed=7, out=out), HERE / 'credit_kernels.pt')
    print('credit kernels: ok')


def golden_heads(root):
    """The identity phase's pack_heads_kernel, head_prep_fused and id_head_scores (speedrun/run.py:3694-3804) under
    the patched interpreter, on heads_inputs' seeded inputs: world 8 (one head per rank), 2 layers, N = 64 tokens per
    rank, t = 64 (b = 8 rows per layer); the pack on 2 layers of 64 tokens (t = 32)."""
    patch_triton_interpreter()
    sys.path.insert(0, str(root / 'train/speedrun'))
    spec = importlib.util.spec_from_file_location('ref_run', root / 'train/speedrun/run.py')
    run = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(run)
    run.moment_kernels.libdevice = interpreter_libdevice()
    from heads_inputs import got_inputs, pack_inputs, rotary
    p = pack_inputs()
    packed = run.pack_heads_kernel(p['qs'], p['ks'], p['vals'], p['outs'], p['targets'], p['lses'])
    got, b = got_inputs()
    t = 64
    cos, sin = rotary(t)
    assert torch.equal(cos, run.rotary(t, 'cpu')[0]) and torch.equal(sin, run.rotary(t, 'cpu')[1])
    prep = run.head_prep_fused(got, cos, sin, b, t)
    names = ('q16', 'k16', 'v16', 'hub16', 'q32', 'pairs', 'lse', 'hub_out', 'sq_q', 'sq_k', 'steps_q', 'steps_k')
    prep = dict(zip(names, prep))
    prep['f2'], prep['f4'], prep['xy'] = prep.pop('pairs')
    back = torch.empty(got.shape[0], got.shape[1], 3, got.shape[2], 64, dtype=torch.bfloat16)
    run.id_head_scores(got, (cos, sin), back, b, t)
    torch.save(dict(pack=packed.view(torch.int16).clone(), prep={k: v.clone() for k, v in prep.items()},
                    back=back.clone(), b=b, t=t), HERE / 'heads.pt')
    print('heads: ok')


def load_recipe(root):
    """train/val/run.py keeps its modules as `# ==== module <name>` sections behind a loader; this loads the `recipe`
    section (the record's ops) the same way, compiled at its own line numbers."""
    import types
    file = root / 'train/val/run.py'
    mark = '# ' + '=' * 40 + ' module '
    lines = file.read_text().splitlines(keepends=True)
    starts = [(i, line[len(mark):].strip()) for i, line in enumerate(lines) if line.startswith(mark)]
    spans = {n: (i + 1, j) for (i, n), (j, _) in zip(starts, starts[1:] + [(len(lines), '')])}
    a, b = spans['recipe']
    module = types.ModuleType('recipe')
    module.__file__ = str(file)
    sys.modules['recipe'] = module
    exec(compile('\n' * a + ''.join(lines[a:b]), str(file), 'exec'), module.__dict__)
    return module


def golden_readout(root):
    """The track-1 readout scorers' record ops on readout_inputs' seeded inputs: future_scores and
    future_query_response through the ops themselves (CPU tensors take their dense paths), key_response and
    routed_response through their Triton kernels under the patched interpreter (launched with the ops' arguments)."""
    import triton
    import triton.language as tl
    patch_triton_interpreter()
    R = load_recipe(root)
    # the interpreter runs a kernel's source against its module's globals (the factories' local imports are not
    # seen): give the recipe module the names the kernels use, libdevice as interpreter_libdevice's numpy versions
    for name, value in (('libdevice', interpreter_libdevice()), ('tl', tl), ('triton', triton)):
        if not hasattr(R, name) or name == 'libdevice':
            setattr(R, name, value)
    from readout_inputs import future_inputs, key_inputs, query_inputs, routed_inputs
    out = {}
    f = future_inputs()
    out['future'] = R.fused_scores(f['q'], f['target'], f['dk'], f['dv'], f['a'], f['contrast'], f['source_start'],
                                   f['window'])
    qi = query_inputs()
    out['query'] = R.query_response(qi['dq'], qi['keys'], qi['values'], qi['probabilities'], qi['base'])
    routed, key_kernel = R.finite_attention_kernels()
    k = key_inputs()
    heads, probes, sources, width = k['dk'].shape
    key_out = torch.empty(heads, probes, sources)
    key_kernel[(triton.cdiv(probes * sources, 64), heads)](
        k['q'], k['dk'].contiguous(), k['A'], k['C'], key_out, heads, k['q'].shape[1], sources, probes, width,
        *k['q'].stride(), *k['A'].stride(), *k['C'].stride(), k['source_start'], k['query_start'], k['window'], 64, 64)
    out['key'] = key_out
    r = routed_inputs()
    m, probes, heads, width = r['dq'].shape
    count = r['keys'].shape[2]
    routed_out = torch.empty(m, probes, heads, width)
    routed[(triton.cdiv(probes, 32), m * heads)](
        r['dq'].contiguous(), r['keys'].contiguous(), r['values'].contiguous(), r['probabilities'].contiguous(),
        r['rest'].contiguous(), routed_out, probes, heads, count, width, 32, max(16, triton.next_power_of_2(count)))
    out['routed'] = routed_out
    torch.save({k: v.clone() for k, v in out.items()}, HERE / 'readout.pt')
    print('readout: ok', {k: tuple(v.shape) for k, v in out.items()})


def golden_scorer(root):
    """The true-path readout's scorer kernels (train/val/run.py `readout` section: stats_kernel, staged_kernel,
    readout_kernel) under the patched interpreter on scorer_inputs' seeded inputs, gated, with the exact diagonal
    and the self-edge. The section is imported through the file's own section loader (its bootstrap, run here)."""
    import triton
    patch_triton_interpreter()
    file = root / 'train/val/run.py'
    text = file.read_text()
    boot = text[:text.index('LOADER = Sections()')] + 'LOADER = Sections()\n'
    env = {'__name__': 'ref_val_boot', '__file__': str(file)}
    exec(compile(boot, str(file), 'exec'), env)
    sys.path.insert(0, str(root))
    sys.meta_path.insert(0, env['LOADER'])
    import readout as RO
    RO.libdevice = interpreter_libdevice()
    from scorer_inputs import scorer_inputs
    x = scorer_inputs()
    m, n, d_rows, start, nc = x['m'], x['n'], x['d_rows'], x['start'], x['nc']
    db = torch.empty(m, n, 512, dtype=torch.bfloat16)
    st = torch.empty(m, n, 2)
    RO.stats_kernel[(triton.cdiv(n, 16), m)](x['delta'], x['X'], x['SQX'], db, st, start, n, d_rows, 512, 16, x['eps'])
    out_s = torch.empty(m, n)
    se_s = torch.zeros(m, d_rows, 512, dtype=torch.bfloat16)
    RO.staged_kernel[(triton.cdiv(n, 64), m)](
        x['UP'], st, x['R0'], x['VC'], x['GZ'], x['VE'], x['CS'], x['SN'], x['U'], x['W'], x['M1'], x['M2'], x['QD'],
        x['GD'], x['AD'], x['CD'], x['VT'], x['OT'], out_s, se_s, start, n, d_rows, 512, 8, 64, True, True, True, 64,
        nc)
    tok = slice(start, start + m)
    cs, sn = x['CS'][tok], x['SN'][tok]
    out_d = torch.empty(m, n)
    se_d = torch.zeros(m, n, 512, dtype=torch.bfloat16)
    RO.readout_kernel[(m, triton.cdiv(n, RO.BPR))](
        x['PJ'], x['R0'][tok].contiguous(), cs, sn, x['GC'], x['VE'][tok].contiguous(), x['U'], x['W'], x['M1'],
        x['M2'], x['QD'], x['GD'], x['AD'], x['CD'], x['VT'], x['OT'], out_d, se_d, start, n, *cs.stride(),
        *sn.stride(), 8, 64, True, True, True, RO.BPR)
    torch.save(dict(db=db, st=st, staged=out_s, staged_se=se_s, direct=out_d, direct_se=se_d), HERE / 'scorer.pt')
    print('scorer: ok')


def golden_cycle(root):
    """The identity phase's readout cycle (train/speedrun/run.py top_credit, coordinate_change) on cycle_inputs'
    seeded inputs: its torch.compile'd helpers called as their original functions, its Triton weights kernel under the
    patched interpreter (libdevice tanh / exp as numpy's)."""
    import types
    import numpy as np
    patch_triton_interpreter()
    sys.path.insert(0, str(root / 'train/speedrun'))
    spec = importlib.util.spec_from_file_location('ref_run_cycle', root / 'train/speedrun/run.py')
    run = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(run)
    for name in ('coordinate_change', 'cycle_scales', 'cycle_finish', 'cycle_powers'):
        fn = getattr(run, name)
        setattr(run, name, getattr(fn, '_torchdynamo_orig_callable', fn))
    lib = interpreter_libdevice()
    base = vars(lib)
    from triton.runtime import interpreter as ti
    import triton.language as tl

    def unary(fn):
        def f(x, *args, **kwargs):
            data = fn(np.asarray(x.handle.data, dtype=np.float32)).astype(np.float32)
            return tl.core.tensor(ti.TensorHandle(data, x.handle.dtype.scalar), x.type)
        return f
    run.libdevice = types.SimpleNamespace(**base, tanh=unary(np.tanh), exp=unary(np.exp))
    from cycle_inputs import cycle_inputs
    x = cycle_inputs()
    model = types.SimpleNamespace(H=x['H'], step_t=x['step_t'], lm_head=x['lm_head'])
    credit = run.top_credit(model, x['x'], x['y'])
    coords = run.coordinate_change(x['raw'], x['y'])
    signs = run.step_signs(x['step_t'], 'cpu')
    torch.save(dict(credit=credit.clone(), coords=coords.clone(), signs=signs.clone()), HERE / 'cycle.pt')
    print('cycle: ok', tuple(credit.shape), tuple(coords.shape))


def chunk_size_ref(draws, cap):
    return next(n for n in range(min(cap, draws), 0, -1) if draws % n == 0)


def golden_dust(root):
    """Dust's block_forward (train/val/dust.py, its compiled function called as the original, eager flex attention)
    on dust_inputs' seeded inputs, fp32 on the CPU: a value-embedding block with jitter at all four sites, and a plain
    block with none."""
    import utils.model as model
    from torch.nn.attention.flex_attention import flex_attention
    model.flex = flex_attention
    spec = importlib.util.spec_from_file_location('ref_dust', root / 'train/val/dust.py')
    dust = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(dust)
    bf = getattr(dust.block_forward, '_torchdynamo_orig_callable', dust.block_forward)
    from dust_inputs import dust_inputs
    x = dust_inputs()
    cos, sin = x['cos'][None, :, None, :], x['sin'][None, :, None, :]
    with torch.no_grad():
        gated = bf(x['x'], x['w'], x['ve'], cos, sin, x['windows'][0], **x['jitter'])
        plain = bf(x['x'], x['plain'], None, cos, sin, x['windows'][1])
    # DUST.head_error, run as the class's own method on a stand-in instance (the attributes it reads)
    import types
    from dust_inputs import head_error_inputs
    h = head_error_inputs()
    b, t = h['y'].shape
    inst = types.SimpleNamespace(outputs={'lm_head': h['raw']}, y=h['y'], clean_loss=h['clean_loss'], batch=b,
                                 length=t, dtype=torch.bfloat16, device=torch.device('cpu'),
                                 recipe=types.SimpleNamespace(nrep=h['nrep']),
                                 model=types.SimpleNamespace(config=types.SimpleNamespace(vocab_size=4096)))
    inst.noise = lambda *shape, dtype=None: h['noise'](*shape)
    error = dust.DUST.head_error(inst, h['draws'], h['sigma'])
    touched = h['draws'] // chunk_size_ref(h['draws'], h['nrep']) * 256  # the slabs the chunks jittered
    assert not error[..., touched:].any()
    torch.save(dict(gated=gated.clone(), plain=plain.clone(), head_error=error[..., :touched].clone()),
               HERE / 'dust.pt')
    print('dust: ok', tuple(gated.shape), tuple(error.shape))


def golden_id_kernels(root):
    """The identity phase's batched GEMMs (speedrun/id_kernels.py: hidden_credits_fused, at_b_layers,
    square_credit_grads) through their Triton kernels under the patched interpreter, on id_inputs' seeded inputs."""
    patch_triton_interpreter()
    spec = importlib.util.spec_from_file_location('ref_id_kernels', root / 'train/speedrun/id_kernels.py')
    idk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(idk)
    from id_inputs import at_b_inputs, hidden_inputs, square_inputs
    us, steps, credb, w_out_t = hidden_inputs()
    hidden = idk.hidden_credits_fused(us, steps, credb, w_out_t)
    As, Bs = at_b_inputs()
    at_b = torch.empty(8, As[0].shape[-1], Bs[0].shape[-1], dtype=torch.bfloat16)
    idk.at_b_layers(As, Bs, at_b)
    n1s, got2 = square_inputs()
    d = n1s[0].shape[1]
    square = torch.empty(3 * len(n1s), d, d, dtype=torch.bfloat16)
    idk.square_credit_grads(n1s, got2, square)
    torch.save(dict(hidden=hidden.clone(), at_b=at_b.clone(), square=square.clone()), HERE / 'id_kernels.pt')
    print('id_kernels: ok')


def main():
    root = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get('NOISE_REFERENCE', ''))
    assert (root / 'utils/model.py').exists(), 'pass the reference checkout as argv[1]'
    only = set(sys.argv[2].split(',')) if len(sys.argv) > 2 else None  # e.g. "heads": regenerate that fixture only
    want = lambda name: only is None or name in only
    torch.set_num_threads(os.cpu_count())
    model, eggroll = load_reference(root)
    if want('forward'):
        golden_forward(model)
    if want('population'):
        golden_population(eggroll, length=256)
        golden_population(eggroll, length=2048)
    if want('step'):
        golden_step(eggroll)
    if want('informative'):
        golden_informative(model, eggroll)
    if want('implicit'):
        golden_implicit(root)
    if want('credit'):
        golden_credit(root)
    if want('heads'):
        golden_heads(root)
    if want('readout'):
        golden_readout(root)
    if want('scorer'):
        golden_scorer(root)
    if want('cycle'):
        golden_cycle(root)
    if want('dust'):
        golden_dust(root)
    if want('id_kernels'):
        golden_id_kernels(root)


if __name__ == '__main__':
    main()
