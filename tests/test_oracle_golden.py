"""The CPU oracle against the reference's own outputs (tests/golden/, made by tests/golden/make_golden.py from the
reference checkout). These pin the restatement before it is used to check the CUDA path."""
import pytest
import torch

from oracle import credit, eggroll, gpt


def _check_weights(w, sums):
    for name, (s, a, head) in sums.items():
        assert torch.equal(w[name].flatten()[:8], head), name
        assert abs(float(w[name].double().sum()) - s) <= 1e-9 * max(1.0, abs(a)), name
        assert abs(float(w[name].double().abs().sum()) - a) <= 1e-9 * max(1.0, a), name


def test_param_order_and_count():
    names = [n for n, _ in gpt.param_shapes()]
    assert len(names) == 60 and names[:3] == ['resid_lambdas', 'x0_lambdas', 'transformer.wte.weight']
    assert gpt.param_count() == 37_749_776


def test_init_matches_reference_constructor(golden):
    _check_weights(gpt.init_weights(0), golden('gpt_forward.pt')['weights'])


def test_init_matches_reference_make_model(golden):
    _check_weights(gpt.init_weights(0, eggroll=True), golden('population_T256.pt')['weights'])


def test_zipf_tokens_match_fixture(golden):
    g = golden('gpt_forward.pt')
    assert torch.equal(gpt.zipf_tokens(4, 2049, seed=0), g['tokens'].long())


@pytest.mark.parametrize('rows', [1])
def test_forward_fp32_matches_reference(golden, rows):
    """Config 1 (one of its four rows, to keep the CPU suite short): the oracle's dense-attention forward against the
    reference's flex-attention forward, fp32, per-token CE."""
    g = golden('gpt_forward.pt')
    tokens = g['tokens'].long()[:rows]
    ce = gpt.forward(gpt.init_weights(0), tokens[:, :-1], tokens[:, 1:], loss_reduction='none').view(rows, -1)
    torch.testing.assert_close(ce, g['ce'][:rows], rtol=1e-5, atol=1e-5)


def test_forward_rows_matches_reference(golden):
    """The oracle of the un-perturbed forward on distinct rows (population_loss at sign 0, per row) against the
    reference's GPT.forward, fp32, per-token CE, with ignore_index -1 on two targets."""
    g = golden('gpt_forward.pt')
    tokens = g['tokens'].long()[:1]
    targets = tokens[:, 1:].clone()
    targets[0, 7] = targets[0, 2000] = -1
    ce = eggroll.forward_rows(gpt.init_weights(0), tokens[:, :-1], targets, autocast=False, loss_reduction='none')
    want = g['ce'][0].clone()
    want[7] = want[2000] = 0
    torch.testing.assert_close(ce, want, rtol=1e-5, atol=1e-5)


def _population_case(g):
    buf = eggroll.make_buffer(g['noise_size'], seed=0)
    assert torch.equal(buf[:16], g['buffer_head'])
    assert abs(float(buf.double().sum()) - float(g['buffer_sum'])) < 1e-6
    shapes = gpt.param_shapes()
    offs = eggroll.offsets(shapes, g['pairs'], step=1, n_noise=g['noise_size'])
    for name in offs:
        assert torch.equal(offs[name], g['offsets'][name]), name
    nz = eggroll.noise(buf, offs, g['directions'], shapes)
    for name, ref in g['gathered'].items():
        got = nz[name]
        if isinstance(ref, tuple):
            assert all(torch.equal(x[:, :4], y) for x, y in zip(got, ref)), name
        else:
            assert torch.equal(got[:, :4], ref), name
    sign = torch.tensor([g['sigma'], -g['sigma']]).repeat(g['pairs'])
    tokens = g['tokens'].long()
    return nz, sign, tokens[:-1], tokens[1:]


def test_noise_map_bit_exact(golden):
    _population_case(golden('population_T256.pt'))


@pytest.mark.parametrize('length', [256, 2048])
def test_population_loss_fp32(golden, length):
    g = golden(f'population_T{length}.pt')
    nz, sign, idx, tgt = _population_case(g)
    w = gpt.init_weights(0, eggroll=True)
    got = eggroll.population_loss(w, nz, sign, idx, tgt)
    torch.testing.assert_close(got, g['loss_fp32'], rtol=2e-6, atol=0)


def test_population_loss_autocast(golden):
    """The oracle's bf16 rounding points against the reference run under CPU bf16 autocast."""
    g = golden('population_T256.pt')
    nz, sign, idx, tgt = _population_case(g)
    w = gpt.init_weights(0, eggroll=True)
    got = eggroll.population_loss(w, nz, sign, idx, tgt, autocast=True)
    torch.testing.assert_close(got, g['loss_autocast'], rtol=2e-5, atol=0)


def test_member_layout_and_update(golden):
    """One Eggroll.step: losses -> fitness -> seed-rebuilt gradient, against the reference step's gradients."""
    g = golden('eggroll_step.pt')
    pairs, rows, length, n = g['pairs'], g['rows'], g['length'], g['noise_size']
    shapes = gpt.param_shapes()
    members, per_seq, per_rank, directions, positive, row = eggroll.member_layout(pairs, rows)
    assert (members, per_seq, per_rank) == (2 * pairs, 2 * pairs // rows, 2 * pairs)
    buf = eggroll.make_buffer(n, seed=0)
    offs = eggroll.offsets(shapes, pairs, step=g['step'], n_noise=n)
    w = gpt.init_weights(0, eggroll=True)
    tokens = g['tokens'].long()
    losses = []
    chunk = 2 * g['chunk']
    for start in range(0, members, chunk):
        sel = torch.arange(start, start + chunk)
        nz = eggroll.noise(buf, offs, directions[sel], shapes)
        sign = torch.where(positive[sel], eggroll.SIGMA, -eggroll.SIGMA)
        r = int(row[start])
        losses.append(eggroll.population_loss(w, nz, sign, tokens[r, :-1], tokens[r, 1:]))
    losses = torch.cat(losses)
    assert abs(float(losses.mean()) - g['mean_loss']) < 1e-5
    weight, count = eggroll.fitness_weights(losses, pairs)
    grads = eggroll.rebuild_update(buf, offs, weight, count, shapes)
    for name, ref in g['grad_small'].items():
        torch.testing.assert_close(grads[name], ref, rtol=1e-4, atol=1e-6)
    for name, ref in g['grad_corner'].items():
        torch.testing.assert_close(grads[name][:8, :8], ref, rtol=1e-4, atol=1e-6)


def test_implicit_key_context_matches_reference_kernel(golden):
    g = golden('implicit_key_context.pt')
    gen = torch.Generator().manual_seed(g['seed'])
    q, k, v, hub = (torch.randn(g['rows'], g['length'], 64, generator=gen) / 8 for _ in range(4))
    hub = hub * 8
    for window, (lse, center) in g['out'].items():
        got_lse, got_center = credit.implicit_key_context(q, k, v, hub, window)
        torch.testing.assert_close(got_lse.float(), lse, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(got_center.float(), center, rtol=1e-4, atol=1e-5)


def _credit_case(golden):
    import sys
    from conftest import GOLDEN
    sys.path.insert(0, str(GOLDEN))
    from credit_inputs import credit_inputs
    g = golden('credit_kernels.pt')
    x = credit_inputs(g['rows'], g['length'], g['seed'])
    b16 = {k: x[k].bfloat16().double() for k in ('qp', 'kp', 'values', 'hub')}
    return g, x, b16


def _rel(a, r):
    return ((a.double() - r.double()).abs().max() / r.double().abs().max()).item()


@pytest.mark.parametrize('window', [128, 256])
def test_credit_oracle_matches_reference_kernels(golden, window):
    """The dense credit restatements (bf16 operand rounding emulated) against the reference Triton kernels run under
    the interpreter (its bf16 dot and rounding fixed, tests/golden/make_golden.py)."""
    g, x, b = _credit_case(golden)
    o = g['out'][window]
    lse, center = credit.implicit_key_context(b['qp'], b['kp'], b['values'], b['hub'], window)
    assert _rel(lse, o['lse']) < 1e-6 and _rel(center, o['center']) < 1e-6
    vp = credit.value_pass(b['qp'], b['kp'], o['lse'], x['hub'], window, emulate=True)
    assert _rel(vp, o['raw_value']) < 1e-4
    key = credit.key_scan(x['qp'], x['kp'], x['k_raw'], o['lse'], x['values'], x['hub'], o['center'], x['cos'],
                          x['sin'], window, 0.003, emulate=True)
    assert _rel(key, o['key']) < 1e-3
    assert torch.equal(o['key_v'], o['key'])
    qs = credit.moment_query_scores(b['qp'], b['kp'], b['values'], b['hub'], x['q_raw'], o['sq'], x['kp'], x['cos'],
                                    x['sin'], o['lse'], o['center'], o['steps'], window, emulate=True)
    qs = qs.float().bfloat16().float()  # the reference stores bf16
    assert (qs != o['query']).float().mean() < 0.01 and _rel(qs, o['query']) < 1e-3


def test_key_moment_oracle_matches_reference_kernel(golden):
    g, x, b = _credit_case(golden)
    o = g['out']['keys']
    out, values = credit.moment_key_scores(b['qp'], b['kp'], b['values'], b['hub'], x['k_raw'], o['sq'], x['qp'],
                                           x['cos'], x['sin'], o['lse'], o['center'], o['steps'], emulate=True)
    assert _rel(out, o['out']) < 1e-4 and _rel(values, o['values']) < 1e-4


# ------------------------------------------------------------------------------------------------------------------
# weights whose every block matters (tests/golden/informative.pt: the reference's modules loaded with
# oracle.gpt.informative_weights), so attention, MLP, norms and value embeddings are pinned, not only the embedding
# ------------------------------------------------------------------------------------------------------------------
def informative_case(p):
    """(noise, sign, idx, targets) of a population_T* entry of informative.pt."""
    shapes = gpt.param_shapes()
    buf = eggroll.make_buffer(p['noise_size'], seed=0)
    offs = eggroll.offsets(shapes, p['pairs'], step=p['step'], n_noise=p['noise_size'])
    nz = eggroll.noise(buf, offs, p['directions'], shapes)
    sign = torch.tensor([p['sigma'], -p['sigma']]).repeat(p['pairs'])
    tokens = p['tokens'].long()
    return nz, sign, tokens[:-1], tokens[1:]


def fitness_error(got, ref):
    """(max |fitness error| / max |fitness|, rms fitness error / std of the fitness) of per-member losses against a
    reference's, fitness = l(-) - l(+) per antithetic pair (eggroll.py:151); the std is what the update's z-scoring
    divides by (eggroll.py:152)."""
    fg, fr = got[1::2] - got[0::2], ref[1::2] - ref[0::2]
    err = (fg.double() - fr.double())
    return (err.abs().max() / fr.double().abs().max()).item(), (err.square().mean().sqrt() / fr.double().std()).item()


def test_informative_weights_match_fixture(golden):
    _check_weights(gpt.informative_weights(0), golden('informative.pt')['weights'])


def test_forward_informative_matches_reference(golden):
    """The oracle's dense-attention forward against the reference's GPT.forward, fp32, per token, on active weights
    (one of the fixture's two rows, to keep the CPU suite short)."""
    f = golden('informative.pt')['forward']
    tokens = f['tokens'].long()[:1]
    ce = gpt.forward(gpt.informative_weights(0), tokens[:, :-1], tokens[:, 1:], loss_reduction='none').view(1, -1)
    torch.testing.assert_close(ce, f['ce'][:1], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize('autocast', [False, True])
def test_population_informative_matches_reference(golden, autocast):
    """The oracle's population_loss against the reference's on active weights, 16 antithetic pairs x 256 tokens.

    fp32 against the reference's fp32 run: per-member losses within 2e-6 relative and the antithetic fitness within
    1e-3 of its scale, i.e. the same arithmetic. The autocast rounding points against the reference's CPU bf16
    autocast run: losses within 5e-4 relative and the fitness within 5% of its scale. That is the floor for any two
    bf16 implementations that sum their products in different orders: the CPU's bf16 GEMMs round about 1 output in
    10,000 to the other neighbouring bf16 value than an fp32-accumulated product does, and the same oracle with its
    products summed in fp64 moves the fitness by 2.5-2.9% of its scale (the reference's own autocast-vs-fp32 gap on
    these inputs is 2.7%)."""
    p = golden('informative.pt')['population_T256']
    nz, sign, idx, tgt = informative_case(p)
    got = eggroll.population_loss(gpt.informative_weights(0), nz, sign, idx, tgt, autocast=autocast)
    ref = p['loss_autocast'] if autocast else p['loss_fp32']
    torch.testing.assert_close(got, ref, rtol=5e-4 if autocast else 2e-6, atol=0)
    worst, rms = fitness_error(got, ref)
    assert worst <= (5e-2 if autocast else 1e-3), (worst, rms)
