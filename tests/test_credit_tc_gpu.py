"""The tcgen05 credit kernels (bf16 operands, T % 128 == 0) against the dense CPU oracle (oracle/credit.py, with the
kernels' bf16 roundings) and against the warp-MMA kernels on the same inputs: the value pass (noise_value_pass_ws),
lse / center (noise_implicit_key_context_ws), the identity phase's key moments (noise_moment_key_scores_ws) and the
key scan (noise_key_scan_ws, tf32 logits and scores).

Value pass:
Stated tolerance: 2e-3 of the largest |reference| of the output (bf16 probabilities; the two GPU kernels round the
exponent argument differently, so single probabilities can differ by one bf16 ulp). At the credit benchmark's full
size (rows 128, T 2048, window 2048) the size-independent property: with lse taken over the same window every
receiver's probabilities sum to one, so sum_t out[t] = sum_s source[s] for each row and channel."""
import sys

import pytest
import torch

from conftest import GOLDEN
from oracle import credit

sys.path.insert(0, str(GOLDEN))
from credit_inputs import credit_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda', 0) if torch.cuda.is_available() else None
TOL = 2e-3


def rel(a, r):
    return ((a.double().cpu() - r.double().cpu()).abs().max() / r.double().abs().max()).item()


@pytest.fixture(scope='module')
def mk():
    import noise_b200.moment_kernels as m
    return m


def run(mk, b, lse, source, window, **kw):
    out = mk.value_pass(b['qp'], b['kp'], lse, source, window, **kw)
    return out


# windows below, at and above one tile; T = 384 has an odd number of key tiles (the last pair has one tile)
@pytest.mark.parametrize('rows,t,window', [(3, 384, 0), (3, 384, 1), (3, 384, 127), (3, 384, 200), (3, 384, 1000),
                                           (2, 256, 128), (1, 128, 64), (2, 512, 320)])
def test_against_oracle_and_warp_kernel(mk, rows, t, window):
    from noise_b200 import _lib
    x = credit_inputs(rows, t, seed=rows * 1000 + window)
    b = {k: x[k].to(DEV).bfloat16() for k in ('qp', 'kp')}
    bd = {k: x[k].bfloat16().double() for k in ('qp', 'kp')}
    lse = credit.implicit_key_context(bd['qp'], bd['kp'], bd['qp'], bd['qp'], window)[0]
    lse = lse.float().to(DEV)
    src = x['hub'].to(DEV)
    got = run(mk, b, lse, src, window)
    torch.cuda.synchronize()
    assert _lib.read_status(got._noise_workspace) == 0
    ref = credit.value_pass(bd['qp'], bd['kp'], lse.cpu(), x['hub'], window, emulate=True)
    assert rel(got, ref) < TOL
    warp = run(mk, b, lse, src, window, tc=False)
    assert not hasattr(warp, '_noise_workspace')
    assert rel(got, warp) < TOL


def test_more_items_than_sms_and_strided_views(mk):
    """600 work items on 148 SMs (persistent loop, both O buffers reused); the source read and the output written
    through by-token views (rows // 2, T, 2 * 64), as terminal_value_credits_into does."""
    rows, t, window, heads = 300, 512, 512, 2
    g = torch.Generator().manual_seed(5)
    q = torch.nn.functional.rms_norm(torch.randn(rows, t, 64, generator=g), (64,)).to(DEV).bfloat16()
    k = torch.nn.functional.rms_norm(torch.randn(rows, t, 64, generator=g), (64,)).to(DEV).bfloat16()
    lse = (torch.randn(rows, t, generator=g) * 0.3 + 5.0).to(DEV)
    src = (torch.randn(rows // heads, t, heads * 64, generator=g) * 0.1).to(DEV)
    got = mk.value_pass(q, k, lse, src, window, heads, heads)
    warp = mk.value_pass(q, k, lse, src, window, heads, heads, tc=False)
    torch.cuda.synchronize()
    from noise_b200 import _lib
    assert _lib.read_status(got._noise_workspace) == 0
    assert rel(got, warp) < TOL


def test_full_size_sum_property(mk):
    """rows 128 (16 x 8 heads), T 2048, window 2048: sum over keys of the credits equals the source's sum over
    receivers (probabilities normalised by the same window's lse), and the two GPU kernels agree."""
    rows, t, window = 128, 2048, 2048
    x = credit_inputs(rows, t, seed=3)
    b = {k: x[k].to(DEV).bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    lse, _ = mk.implicit_key_context_edges(b['qp'], b['kp'], b['values'], b['hub'], window)
    src = x['values'].to(DEV)
    got = mk.value_pass(b['qp'], b['kp'], lse, src, window)
    warp = mk.value_pass(b['qp'], b['kp'], lse, src, window, tc=False)
    torch.cuda.synchronize()
    from noise_b200 import _lib
    assert _lib.read_status(got._noise_workspace) == 0
    assert rel(got, warp) < TOL
    s_out, s_src = got.double().sum(1), src.double().sum(1)
    assert ((s_out - s_src).abs().max() / s_src.abs().max()).item() < 1e-2


# --- lse / center (noise_implicit_key_context_ws) --------------------------------------------------------------------

@pytest.mark.parametrize('rows,t,window', [(3, 384, 0), (3, 384, 64), (3, 384, 192), (2, 512, 512), (1, 128, 128),
                                           (2, 640, 2048)])
def test_context_against_oracle_and_warp_kernel(mk, rows, t, window):
    """lse and center within 1e-5 of max |ref| (as the warp kernel's own test), T = 384 / 640 with an odd number of
    query tiles (the last pair has one)."""
    from noise_b200 import _lib
    x = credit_inputs(rows, t, seed=7 * rows + window)
    b = {k: x[k].to(DEV).bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    bd = {k: x[k].bfloat16().double() for k in ('qp', 'kp', 'values', 'hub')}
    lse, center = mk.implicit_key_context_edges_impl(b['qp'], b['kp'], b['values'], b['hub'], window)
    torch.cuda.synchronize()
    assert _lib.read_status(lse._noise_workspace) == 0
    ref_lse, ref_center = credit.implicit_key_context(bd['qp'], bd['kp'], bd['values'], bd['hub'], window)
    assert rel(lse, ref_lse) < 1e-5 and rel(center, ref_center) < 1e-5
    wl, wc = mk.implicit_key_context_edges_impl(b['qp'], b['kp'], b['values'], b['hub'], window, tc=False)
    assert not hasattr(wl, '_noise_workspace')
    assert rel(lse, wl) < 1e-5 and rel(center, wc) < 1e-5


def test_context_full_size(mk):
    """rows 128, T 2048 (config 3) at windows 2048 and 1024: the tcgen05 and warp kernels agree within 1e-5, and
    every lse is at least the diagonal logit (the query's own key is always visible)."""
    from noise_b200 import _lib
    x = credit_inputs(128, 2048, seed=4)
    b = {k: x[k].to(DEV).bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    diag = (b['qp'].float() * b['kp'].float()).sum(-1) / 8
    for window in (2048, 1024):
        lse, center = mk.implicit_key_context_edges_impl(b['qp'], b['kp'], b['values'], b['hub'], window)
        wl, wc = mk.implicit_key_context_edges_impl(b['qp'], b['kp'], b['values'], b['hub'], window, tc=False)
        torch.cuda.synchronize()
        assert _lib.read_status(lse._noise_workspace) == 0
        assert rel(lse, wl) < 1e-5 and rel(center, wc) < 1e-5
        assert (lse >= diag - 1e-4).all()


# --- key moments (noise_moment_key_scores_ws) ------------------------------------------------------------------------

def key_moment_inputs(rows, t, seed):
    x = credit_inputs(rows, t, seed=seed)
    d = {k: v.to(DEV) for k, v in x.items()}
    b = {k: d[k].bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    sq = x['k_raw'].square().sum(-1)
    steps = 0.003 * (sq / 64).sqrt().clamp(min=1e-6)
    return x, d, b, sq, steps


@pytest.mark.parametrize('rows,t,out_dtype', [(2, 256, torch.float32), (3, 384, torch.bfloat16),
                                              (2, 512, torch.float32)])
def test_key_moments_against_oracle_and_warp_kernel(mk, rows, t, out_dtype):
    """Key credits within 5e-3 of max |ref| and value sums within 2e-3 (as the warp kernel's tests) for fp32 outputs;
    bf16 outputs add their own rounding (up to 2^-9 of an element: 8e-3 / 6e-3 against the fp64 oracle); T = 384 has
    an odd number of 128-key tiles."""
    x, d, b, sq, steps = key_moment_inputs(rows, t, seed=rows + t)
    lse, center = mk.implicit_key_context_edges_impl(b['qp'], b['kp'], b['values'], b['hub'], t)
    args = (b['qp'], b['kp'], b['values'], b['hub'], d['k_raw'].unsqueeze(0), sq.to(DEV), d['qp'], d['cos'], d['sin'],
            lse, center, steps.to(DEV))
    out = torch.empty(1, rows, t, 64, device=DEV, dtype=out_dtype)
    vals = torch.empty_like(out)
    ws = mk.moment_key_scores_impl(*args, out, vals)
    assert ws is not None
    from noise_b200 import _lib
    assert _lib.read_status(ws) == 0
    wout, wvals = torch.empty_like(out), torch.empty_like(out)
    assert mk.moment_key_scores_impl(*args, wout, wvals, tc=False) is None
    assert rel(out[0].float(), wout[0].float()) < 5e-3 and rel(vals[0].float(), wvals[0].float()) < 2e-3
    bd = {k: x[k].bfloat16().double() for k in ('qp', 'kp', 'values', 'hub')}
    ref, ref_vals = credit.moment_key_scores(bd['qp'], bd['kp'], bd['values'], bd['hub'], x['k_raw'], sq, x['qp'],
                                             x['cos'], x['sin'], lse.cpu(), center.cpu(), steps, emulate=True)
    tk, tv = (5e-3, 2e-3) if out_dtype == torch.float32 else (8e-3, 6e-3)
    assert rel(out[0].float(), ref) < tk and rel(vals[0].float(), ref_vals) < tv


def test_key_moments_full_size(mk):
    """rows 128, T 2048 (config 3): the tcgen05 and warp kernels agree (5e-3 / 2e-3 of max |ref|)."""
    x, d, b, sq, steps = key_moment_inputs(128, 2048, seed=9)
    lse, center = mk.implicit_key_context_edges_impl(b['qp'], b['kp'], b['values'], b['hub'], 2048)
    args = (b['qp'], b['kp'], b['values'], b['hub'], d['k_raw'].unsqueeze(0), sq.to(DEV), d['qp'], d['cos'], d['sin'],
            lse, center, steps.to(DEV))
    out = torch.empty(1, 128, 2048, 64, device=DEV)
    vals = torch.empty_like(out)
    ws = mk.moment_key_scores_impl(*args, out, vals)
    wout, wvals = torch.empty_like(out), torch.empty_like(out)
    mk.moment_key_scores_impl(*args, wout, wvals, tc=False)
    from noise_b200 import _lib
    assert _lib.read_status(ws) == 0
    assert rel(out, wout) < 5e-3 and rel(vals, wvals) < 2e-3


# --- key scan (noise_key_scan_ws) -------------------------------------------------------------------------------------

@pytest.mark.parametrize('rows,t,window,with_values', [(2, 256, 128, True), (3, 384, 320, False), (2, 512, 64, True),
                                                       (1, 384, 2048, True)])
def test_key_scan_against_oracle_and_warp_kernel(mk, rows, t, window, with_values):
    """Key credits within 8e-3 of max |ref| and raw value credits within 4e-3 of the warp kernel (the tcgen05 MMAs read
    the fp32 operands' tf32 part as they are, as the reference's Triton kernel does on this GPU; the warp kernel
    rounds them to nearest: observed 6e-3), windows below, across and beyond the tiles; against the fp64 oracle
    (exact logits) key credits within 5e-3 and value credits within 4e-3 (the tf32 logits' error averages over fewer
    receivers in a 64-wide window)."""
    from noise_b200 import _lib
    x = credit_inputs(rows, t, seed=31 * rows + window)
    d = {k: v.to(DEV) for k, v in x.items()}
    w_ctx = window if window % 64 == 0 else 512
    lse, center = mk.implicit_key_context_edges_impl(d['qp'], d['kp'], d['values'], d['hub'], w_ctx)
    args = (d['qp'], d['kp'], d['k_raw'], lse, d['values'], d['hub'], center, d['cos'], d['sin'], window, 0.003)
    key, val = mk.key_scan(*args, with_values=with_values)
    assert _lib.read_status(key._noise_workspace) == 0
    wkey, wval = mk.key_scan(*args, with_values=with_values, tc=False)
    assert rel(key, wkey) < 8e-3
    ref = credit.key_scan(x['qp'], x['kp'], x['k_raw'], lse.cpu(), x['values'], x['hub'], center.cpu(), x['cos'],
                          x['sin'], window, 0.003, with_values=with_values, emulate=True)
    if with_values:
        ref, ref_val = ref
        assert rel(val, wval) < 4e-3 and rel(val, ref_val) < 4e-3
    assert rel(key, ref) < 5e-3


def test_key_scan_full_size(mk):
    """rows 128, T 2048 (config 3) at windows 2048 and 1024, with the raw value credits (2-stage kernel) and without
    (3-stage kernel): the tcgen05 and warp kernels agree (8e-3 / 4e-3 of max |ref|: truncated against rounded tf32
    operands)."""
    from noise_b200 import _lib
    x = credit_inputs(128, 2048, seed=12)
    d = {k: v.to(DEV) for k, v in x.items()}
    for window in (2048, 1024):
        lse, center = mk.implicit_key_context_edges_impl(d['qp'], d['kp'], d['values'], d['hub'], window)
        args = (d['qp'], d['kp'], d['k_raw'], lse, d['values'], d['hub'], center, d['cos'], d['sin'], window, 0.003)
        key, val = mk.key_scan(*args, with_values=True)
        wkey, wval = mk.key_scan(*args, with_values=True, tc=False)
        assert _lib.read_status(key._noise_workspace) == 0
        assert rel(key, wkey) < 8e-3 and rel(val, wval) < 4e-3
        key_only, _ = mk.key_scan(*args, with_values=False)
        assert _lib.read_status(key_only._noise_workspace) == 0
        assert rel(key_only, key) < 1e-6


# --- query moments (noise_moment_query_scores_ws) ---------------------------------------------------------------------

@pytest.mark.parametrize('rows,t,window', [(2, 256, 256), (3, 384, 128), (2, 512, 320), (1, 384, 2048)])
def test_query_moments_against_oracle_and_warp_kernel(mk, rows, t, window):
    """Query credits within 1e-2 of max |ref| (bf16-rounded outputs, as the warp kernel's tests) against the oracle
    and the warp kernel, bf16 out (1, rows, T, 64); windows below and beyond the tiles."""
    x = credit_inputs(rows, t, seed=57 * rows + window)
    d = {k: v.to(DEV) for k, v in x.items()}
    b = {k: d[k].bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    w_ctx = window if window % 64 == 0 else 512
    lse, center = mk.implicit_key_context_edges_impl(b["qp"], b["kp"], b["values"], b["hub"], min(w_ctx, t))
    sq = x['q_raw'].square().sum(-1)
    steps = 0.01 * (sq / 64).sqrt().clamp(min=1e-6)
    args = (b['qp'], b['kp'], b['values'], b['hub'], d['q_raw'].unsqueeze(0), sq.to(DEV), d['kp'], d['cos'],
            d['sin'], lse, center, steps.to(DEV))
    out = torch.empty(1, rows, t, 64, dtype=torch.bfloat16, device=DEV)
    ws = mk.moment_query_scores_impl(*args, out, window)
    assert ws is not None
    from noise_b200 import _lib
    assert _lib.read_status(ws) == 0
    wout = torch.empty_like(out)
    assert mk.moment_query_scores_impl(*args, wout, window, tc=False) is None
    assert rel(out[0].float(), wout[0].float()) < 1e-2
    bd = {k: x[k].bfloat16().double() for k in ('qp', 'kp', 'values', 'hub')}
    ref = credit.moment_query_scores(bd['qp'], bd['kp'], bd['values'], bd['hub'], x['q_raw'], sq, x['kp'], x['cos'],
                                     x['sin'], lse.cpu(), center.cpu(), steps, window, emulate=True)
    assert rel(out[0].float(), ref) < 1e-2


def test_query_moments_full_size(mk):
    """rows 128, T 2048 (config 3), fp32 out: the tcgen05 and warp kernels agree within 1e-2 of max |ref|."""
    x = credit_inputs(128, 2048, seed=21)
    d = {k: v.to(DEV) for k, v in x.items()}
    b = {k: d[k].bfloat16() for k in ('qp', 'kp', 'values', 'hub')}
    lse, center = mk.implicit_key_context_edges_impl(b['qp'], b['kp'], b['values'], b['hub'], 2048)
    sq = d['q_raw'].square().sum(-1)
    steps = 0.01 * (sq / 64).sqrt().clamp(min=1e-6)
    args = (b['qp'], b['kp'], b['values'], b['hub'], d['q_raw'].unsqueeze(0), sq, d['kp'], d['cos'], d['sin'], lse,
            center, steps)
    out = torch.empty(1, 128, 2048, 64, device=DEV)
    wout = torch.empty_like(out)
    ws = mk.moment_query_scores_impl(*args, out, 2048)
    mk.moment_query_scores_impl(*args, wout, 2048, tc=False)
    from noise_b200 import _lib
    assert _lib.read_status(ws) == 0
    assert rel(out, wout) < 1e-2


def test_ws_fall_through_leaves_status_zero():
    """A _ws entry point that falls through to its warp-MMA kernel (here fp32 operands) still leaves its workspace's
    status word 0, as the header promises: the word starts as 0xFFFFFFFF."""
    import ctypes
    from noise_b200 import _lib
    dev = torch.device('cuda', 0)
    g = torch.Generator(device=dev).manual_seed(5)
    q, k, v, hub = (torch.randn(2, 128, 64, device=dev, generator=g) for _ in range(4))
    lse, center = torch.empty(2, 128, device=dev), torch.empty(2, 128, device=dev)
    ws = torch.full((_lib.STATUS_BYTES,), 255, dtype=torch.uint8, device=dev)
    rc = _lib.lib().noise_implicit_key_context_ws(q.data_ptr(), k.data_ptr(), v.data_ptr(), hub.data_ptr(), 0, 2, 128,
                                                  64, lse.data_ptr(), center.data_ptr(), ws.data_ptr(),
                                                  ctypes.c_size_t(_lib.STATUS_BYTES), _lib.stream_handle(dev))
    assert rc == 0
    assert _lib.read_status(ws) == 0
    assert torch.isfinite(lse).all() and torch.isfinite(center).all()
