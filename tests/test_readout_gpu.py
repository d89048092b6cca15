"""Parity of the track-1 readout scorers (noise_b200.readout) with the reference's own ops (tests/golden/readout.pt)
and with the fp64 oracle at larger sizes, and the install() seam.

Tolerances: fp32 arithmetic in another order than the reference's tf32x3 dots: max |diff| within REL of max |ref|;
routed_response rounds both dots' outputs to bf16, so a sum in another order flips an occasional rounding: ROUTED_REL,
with under 1% of elements off by more than 1e-3 of the scale."""
import sys
from pathlib import Path

import pytest
import torch

from oracle import readout as oracle

sys.path.insert(0, str(Path(__file__).resolve().parent / 'golden'))
from readout_inputs import future_inputs, key_inputs, query_inputs, routed_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None
REL = 2e-5
ROUTED_REL = 1e-2


def _rel(a, r):
    a, r = a.double().cpu(), r.double().cpu()
    return ((a - r).abs().max() / r.abs().max()).item()


def _routed_ok(got, ref):
    got, ref = got.cpu().float(), ref.cpu().float()
    return _rel(got, ref) < ROUTED_REL and (got - ref).abs().gt(1e-3 * ref.abs().max()).float().mean() < 0.01


def _dev(d):
    return {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}


def _future(f):
    from noise_b200 import readout
    return readout.future_scores(f['q'], f['target'], f['dk'], f['dv'], f['a'], f['contrast'], f['source_start'],
                                 f['window'])


def _key(k):
    from noise_b200 import readout
    return readout.key_response(k['q'], k['dk'], k['A'], k['C'], k['source_start'], k['query_start'], k['window'])


def _query(q):
    from noise_b200 import readout
    return readout.query_response(q['dq'], q['keys'], q['values'], q['probabilities'], q['base'])


def _routed(r):
    from noise_b200 import readout
    return readout.routed_response(r['dq'], r['keys'], r['values'], r['probabilities'], r['rest'])


def test_against_reference(golden):
    g = golden('readout.pt')
    assert _rel(_future(_dev(future_inputs())), g['future']) < REL
    assert _rel(_key(_dev(key_inputs())), g['key']) < REL
    assert _rel(_query(_dev(query_inputs())), g['query']) < REL
    assert _routed_ok(_routed(_dev(routed_inputs())), g['routed'])


def test_future_scores_larger():
    f = future_inputs(h=8, t=1024, p=8, m=128, source_start=256, window=512, seed=3)
    ref = oracle.future_scores(f['q'], f['target'], f['dk'], f['dv'], f['a'], f['contrast'], f['source_start'],
                               f['window'])
    assert _rel(_future(_dev(f)), ref) < REL


def test_key_response_larger():
    k = key_inputs(h=8, t=768, p=6, m=128, source_start=256, query_start=256, window=512, seed=5)
    ref = oracle.key_response(k['q'], k['dk'], k['A'], k['C'], k['source_start'], k['query_start'], k['window'])
    assert _rel(_key(_dev(k)), ref) < REL


def test_query_response_larger():
    q = query_inputs(m=5, p=72, h=8, t=1024, window=512, seed=7)
    ref = oracle.query_response(q['dq'], q['keys'], q['values'], q['probabilities'], q['base'])
    assert _rel(_query(_dev(q)), ref) < REL


@pytest.mark.parametrize('h,t,p,m,start,window', [(3, 300, 5, 100, 40, 96), (2, 1000, 3, 200, 0, 1000),
                                                   (2, 257, 1, 129, 250, 64), (1, 64, 2, 17, 10, 0)])
def test_column_scores_tc(h, t, p, m, start, window):
    """future_scores and key_response on tcgen05: column blocks of 128 spanning probes, sources past T, windows
    wider than T, an empty window, receivers off the 32-row tile; against the fp64 oracle and the CUDA-core kernels."""
    from noise_b200 import _lib, readout
    f = future_inputs(h=h, t=t, p=p, m=m, source_start=start, window=window, seed=41 + t)
    ref = oracle.future_scores(f['q'], f['target'], f['dk'], f['dv'], f['a'], f['contrast'], f['source_start'],
                               f['window'])
    d = _dev(f)
    args = (d['q'], d['target'], d['dk'], d['dv'], d['a'], d['contrast'], start, window)
    out = readout.future_scores_impl(*args, tc=True)
    assert _lib.read_status(out._noise_workspace) == 0
    scale = max(ref.abs().max().item(), 1e-30)
    assert (out.double().cpu() - ref).abs().max().item() <= REL * scale
    assert torch.allclose(out, readout.future_scores_impl(*args, tc=False), rtol=0, atol=REL * scale)
    k = key_inputs(h=h, t=t, p=p, m=m, source_start=start + 8, query_start=start, window=window, seed=43 + t)
    kref = oracle.key_response(k['q'], k['dk'], k['A'], k['C'], k['source_start'], k['query_start'], k['window'])
    e = _dev(k)
    kargs = (e['q'], e['dk'], e['A'], e['C'], start + 8, start, window)
    kout = readout.key_response_impl(*kargs, tc=True)
    assert _lib.read_status(kout._noise_workspace) == 0
    kscale = max(kref.abs().max().item(), 1e-30)
    assert (kout.double().cpu() - kref).abs().max().item() <= REL * kscale
    assert torch.allclose(kout, readout.key_response_impl(*kargs, tc=False), rtol=0, atol=REL * kscale)


def _query_case(m, p, h, t, window, seed, dead=None):
    """query_response inputs with token positions spread over the keys (sorted, as a row block's tokens are adjacent),
    a strided (T, H, 64) keys buffer seen as [H, T, 64], and optionally a band of keys with zero probability."""
    g = torch.Generator().manual_seed(seed)
    dq = torch.randn(m, p, h, 64, generator=g) * 0.3
    keys = torch.randn(t, h, 64, generator=g).permute(1, 0, 2)
    values = torch.randn(h, t, 64, generator=g)
    pos = torch.sort(torch.randint(0, t, (m,), generator=g)).values
    lag = pos[:, None] - torch.arange(t)[None]
    prob = torch.rand(h, m, t, generator=g) * ((lag >= 0) & (lag <= window))
    if dead is not None:
        prob[..., dead[0]:dead[1]] = 0
    prob = prob / prob.sum(-1, keepdim=True).clamp_min(1e-6)
    base = torch.randn(h, m, 64, generator=g)
    return dict(dq=dq, keys=keys, values=values, probabilities=prob, base=base)


def _query_tc(q, tc=True):
    from noise_b200 import readout
    return readout.query_response_impl(q['dq'], q['keys'], q['values'], q['probabilities'], q['base'], tc=tc)


def _query_status(out):
    from noise_b200 import _lib
    return _lib.read_status(out._noise_workspace)


@pytest.mark.parametrize('m,p,t,dead', [(5, 72, 1000, None), (3, 128, 64, None), (9, 16, 333, (100, 230)),
                                        (2, 200, 700, (64, 300))])
def test_query_response_tc_shapes(m, p, t, dead):
    """The tcgen05 kernel's 128-row blocks spanning 1 to 9 tokens (or part of one), key counts off the 64-key tile,
    live tiles with dead ones between them, and a strided keys view, against the fp64 oracle."""
    q = _query_case(m, p, 3, t, t // 2, seed=31 + m, dead=dead)
    ref = oracle.query_response(q['dq'], q['keys'], q['values'], q['probabilities'], q['base'])
    assert ref.abs().max() > 0
    out = _query_tc(_dev(q))
    assert _query_status(out) == 0
    assert _rel(out, ref) < REL


def test_query_response_ws_falls_through_past_32k_keys():
    """More keys than the tcgen05 kernel's live-tile list holds: the _ws entry runs the CUDA-core kernel, with its
    status word cleared and a status-only workspace."""
    from noise_b200 import _lib
    q = _query_case(2, 8, 1, 33000, 500, seed=77)
    assert _lib.lib().noise_query_response_workspace_bytes(2, 8, 1, 33000) == 256
    ref = oracle.query_response(q['dq'], q['keys'], q['values'], q['probabilities'], q['base'])
    out = _query_tc(_dev(q))
    assert _query_status(out) == 0
    assert _rel(out, ref) < REL


def test_query_response_tc_skips_dead_tiles_exactly():
    """A token whose probabilities are all zero gets exactly 0, even where e^(dq . k / 8) overflows (the reference
    skips its tiles; the dense form would give 0 * inf = nan), while the other token of its 128-row block is live."""
    q = _query_case(2, 64, 2, 256, 200, seed=5)
    q['probabilities'][:, 0] = 0
    q['dq'][0] *= 2000.0
    out = _query_tc(_dev(q)).cpu()
    assert torch.equal(out[0], torch.zeros_like(out[0]))
    ref = oracle.query_response(q['dq'][1:], q['keys'], q['values'], q['probabilities'][:, 1:], q['base'][:, 1:])
    assert _rel(out[1:], ref) < REL
    zero = dict(q, probabilities=torch.zeros_like(q['probabilities']))
    assert torch.equal(_query_tc(_dev(zero)).cpu(), torch.zeros(2, 64, 2, 64))


def test_query_response_tc_bench_shape():
    """The bench's shape (256 tokens x 64 probes x 8 heads over 2,048 keys, window 1,024; 1,024 CTAs, several waves):
    the tcgen05 kernel against the fp32 CUDA-core kernel over the whole output, and against the fp64 oracle on a sample
    of tokens. The probabilities are normalised per token, as attention's are: with unnormalised ones some tokens'
    1 + partition comes near zero and amplifies any rounding difference."""
    g = torch.Generator().manual_seed(9)
    mq, pq, h, t = 256, 64, 8, 2048
    dq, keys, vals = torch.randn(mq, pq, h, 64, generator=g) * 0.3, torch.randn(h, t, 64, generator=g), \
        torch.randn(h, t, 64, generator=g)
    pos = torch.arange(mq) * (t // mq) + t // mq - 1
    lag = pos[:, None] - torch.arange(t)[None]
    prob = torch.rand(h, mq, t, generator=g) * ((lag >= 0) & (lag <= 1024))
    prob = (prob / prob.sum(-1, keepdim=True)).contiguous()
    base = torch.randn(h, mq, 64, generator=g)
    q = dict(dq=dq, keys=keys, values=vals, probabilities=prob, base=base)
    qd = _dev(q)
    out = _query_tc(qd)
    assert _query_status(out) == 0
    assert _rel(out, _query_tc(qd, tc=False)) < REL
    pick = torch.tensor([0, 1, 127, 200, 255])
    ref = oracle.query_response(dq[pick], keys, vals, prob[:, pick], base[:, pick])
    assert _rel(out[pick.to(DEV)], ref) < REL


def test_expm1_against_fp64_and_cuda():
    """The scorers' own e^x - 1 (noise_expm1_f32: Cody-Waite reduction, degree-8 Taylor polynomial) over [-87,
    ln(FLT_MAX)] and tiny arguments of both signs: within 3.5e-7 relative of fp64 (about 3 ulp; CUDA's expm1f,
    torch.expm1 on the device, is held to the same bound here), +inf past the overflow, -1 far below, NaN kept."""
    from noise_b200 import _lib

    def run(xs):
        x = xs.float().to(DEV)
        out = torch.empty_like(x)
        _lib.check(_lib.lib().noise_expm1_f32(x.data_ptr(), out.data_ptr(), x.numel(), _lib.stream_handle(DEV)),
                   'noise_expm1_f32')
        return x, out

    tiny = torch.logspace(-30, 0, 300_001)
    xs = torch.cat([torch.linspace(-87, 88.7228, 4_000_001), tiny, -tiny, torch.tensor([0.0, 88.72283172607422])])
    x, out = run(xs)
    ref = torch.expm1(x.double().cpu())
    scale = ref.abs().clamp_min(1e-300)
    assert ((out.double().cpu() - ref).abs() / scale).max() < 3.5e-7
    assert ((torch.expm1(x).double().cpu() - ref).abs() / scale).max() < 3.5e-7
    assert torch.isfinite(out).all()
    _, sp = run(torch.tensor([88.72284, 100.0, float('inf'), -100.0, float('-inf'), float('nan')]))
    sp = sp.cpu()
    assert sp[:3].tolist() == [float('inf')] * 3 and sp[3:5].tolist() == [-1.0, -1.0] and sp[5].isnan()


@pytest.mark.parametrize('m,p,k', [(6, 70, 16), (5, 40, 100), (3, 64, 128), (4, 130, 129), (3, 20, 256), (1, 64, 32)])
def test_routed_response_tc(m, p, k):
    """The tcgen05 kernel: two items per 128-row tile (keys padded to 32 at most 128) or one (129..256 keys), an odd
    item count (the last tile's second slot repeats a real item), probe blocks of 64 with a partial last block,
    against the bf16-rounding oracle and the CUDA-core kernel."""
    from noise_b200 import _lib, readout
    r = routed_inputs(m=m, p=p, h=3, k=k, seed=13 + k)
    ref = oracle.routed_response(r['dq'], r['keys'], r['values'], r['probabilities'], r['rest'])
    d = _dev(r)
    out = readout.routed_response_impl(d['dq'], d['keys'], d['values'], d['probabilities'], d['rest'], tc=True)
    assert _lib.read_status(out._noise_workspace) == 0
    assert _routed_ok(out, ref)
    cc = readout.routed_response_impl(d['dq'], d['keys'], d['values'], d['probabilities'], d['rest'], tc=False)
    assert _routed_ok(out, cc)


@pytest.mark.parametrize('k', [16, 100, 256])
def test_routed_response_sizes(k):
    r = routed_inputs(m=6, p=70, h=8, k=k, seed=11)
    ref = oracle.routed_response(r['dq'], r['keys'], r['values'], r['probabilities'], r['rest'])
    assert _routed_ok(_routed(_dev(r)), ref)


def test_install_registers_cuda_kernels():
    """install(R) makes R's ops run these kernels on CUDA tensors, as the reference's fast_kernels.install does: here
    R is a stand-in module whose ops have only their dense default implementations."""
    import types
    from noise_b200 import readout

    @torch.library.custom_op('noise_b200_test_record::future_scores', mutates_args=())
    def fused_scores(q: torch.Tensor, target: torch.Tensor, dk: torch.Tensor, dv: torch.Tensor, a: torch.Tensor,
                     contrast: torch.Tensor, source_start: int, window: int) -> torch.Tensor:
        return oracle.future_scores(q.cpu(), target.cpu(), dk.cpu(), dv.cpu(), a.cpu(), contrast.cpu(), source_start,
                                    window).float().to(q.device)

    def stub(name):
        @torch.library.custom_op(f'noise_b200_test_record::{name}', mutates_args=())
        def op(x: torch.Tensor) -> torch.Tensor:
            return x.clone()
        return op

    R = types.SimpleNamespace(fused_scores=fused_scores, fused_key_response=stub('key_response'),
                              query_response=stub('future_query_response'), routed_response=stub('routed_response'))
    f = _dev(future_inputs())
    readout.install(R)
    out = R.fused_scores(f['q'], f['target'], f['dk'], f['dv'], f['a'], f['contrast'], f['source_start'],
                         f['window'])
    torch.cuda.synchronize()
    ref = oracle.future_scores(*(v.cpu() if torch.is_tensor(v) else v for v in future_inputs().values()))
    assert out.is_cuda and _rel(out, ref) < REL
