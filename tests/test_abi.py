"""The C ABI without a GPU: the library loads, exports every entry point include/noise_b200.h declares, and rejects
bad arguments before touching the device."""
import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / 'include' / 'noise_b200.h'


def declared():
    text = HEADER.read_text()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    return sorted(set(re.findall(r'\b(noise_[a-z0-9_]+)\s*\(', text)))


@pytest.fixture(scope='module')
def L():
    from noise_b200 import _lib
    return _lib.lib()


def test_every_declared_symbol_is_exported(L):
    names = declared()
    assert 'noise_population_loss' in names
    for name in names:
        assert hasattr(L, name), name


def test_bindings_cover_header():
    from noise_b200 import _lib
    assert sorted(n for n, _, _ in _lib.SIGNATURES) == declared()


def test_param_index_matches_named_parameters(L):
    from noise_b200.population import INDEX, N_LAYER, has_ve
    kinds = {0: 'attn.c_q', 1: 'attn.c_k', 2: 'attn.c_v', 3: 'attn.c_proj', 4: 'attn.ve_gate', 5: 'mlp.c_fc',
             6: 'mlp.c_proj'}
    for block in range(N_LAYER):
        for which, kind in kinds.items():
            got = L.noise_param_index(block, which)
            name = f'transformer.h.{block}.{kind}.weight'
            assert got == INDEX.get(name, -1), (block, kind)
        assert L.noise_param_index(block, 7) == (INDEX[f'value_embeds.{block}.weight'] if has_ve(block) else -1)
    assert INDEX['lm_head.weight'] == 55 and INDEX['transformer.wte.weight'] == 2


def test_param_order_matches_oracle():
    from noise_b200.population import PARAMS
    from oracle import gpt
    assert PARAMS == gpt.param_shapes()


def test_workspace_size(L):
    small = L.noise_population_workspace_bytes(1, 128)
    big = L.noise_population_workspace_bytes(4, 2048)
    assert 0 < small < big
    assert L.noise_population_workspace_bytes(0, 128) == 0


def test_rejects_bad_shapes_before_launch(L):
    from noise_b200 import _lib
    gpt = _lib.GPT()
    slices = (_lib.Slice * 60)()
    fake = 256  # never dereferenced: validation fails first
    args = (ctypes.byref(gpt), slices, fake, fake, fake)
    assert L.noise_population_loss(*args, 4, 100, 0, fake, fake, 1 << 30, None) == 1   # T % 128
    assert L.noise_population_loss(*args, 4, 4096, 0, fake, fake, 1 << 30, None) == 1  # T > 2048
    assert L.noise_population_loss(*args, 0, 128, 0, fake, fake, 1 << 30, None) == 1   # no members
    assert L.noise_population_loss(*args, 4, 128, 7, fake, fake, 1 << 30, None) == 4   # reduction
    assert L.noise_population_loss(*args, 4, 128, 0, fake, fake, 16, None) == 3        # workspace too small
    assert L.noise_status_string(3) == b'workspace missing or too small'
    assert L.noise_population_loss(*args, 4, 128, 2, fake, fake, 16, None) == 3        # 'none' is a reduction
    # the un-perturbed forward and the head loss validate the same way
    assert L.noise_gpt_loss(ctypes.byref(gpt), fake, fake, 2, 100, 0, fake, fake, 1 << 30, None) == 1
    assert L.noise_gpt_loss(ctypes.byref(gpt), fake, fake, 2, 128, 3, fake, fake, 1 << 30, None) == 4
    assert L.noise_gpt_loss(ctypes.byref(gpt), fake, fake, 2, 128, 2, fake, fake, 16, None) == 3
    assert L.noise_gpt_loss(ctypes.byref(gpt), None, fake, 2, 128, 0, fake, fake, 1 << 30, None) == 4
    assert L.noise_gpt_workspace_bytes(2, 128) == L.noise_population_workspace_bytes(2, 128)
    assert L.noise_head_loss(fake, fake, fake, 100, fake, fake, 1 << 30, None) == 1     # rows % 128
    assert L.noise_head_loss(fake + 4, fake, fake, 128, fake, fake, 1 << 30, None) == 2  # x not 16-byte aligned
    assert L.noise_head_loss(fake, fake, fake, 128, fake, fake, 16, None) == 3
    assert 0 < L.noise_head_loss_workspace_bytes(128) < L.noise_head_loss_workspace_bytes(256)
    # head sharding: the reference's shape asserts
    pieces = (_lib.HeadPieces * 2)()
    assert L.noise_pack_heads(pieces, 2, 24, 8, fake, None) == 1          # tokens % 16
    assert L.noise_pack_heads(pieces, 17, 32, 8, fake, None) == 1         # more layers than the launch carries
    assert L.noise_pack_heads(pieces, 2, 32, 8, fake, None) == 4          # missing pieces
    prep = _lib.HeadPrep()
    assert L.noise_head_prep(fake, 8, 2, 48, fake, fake, 64, 0.003, 1e-6, ctypes.byref(prep), None) == 1  # n % 32
    assert L.noise_head_prep(fake, 8, 2, 64, fake, fake, 64, 0.003, 1e-6, ctypes.byref(prep), None) == 4  # outputs
    assert L.noise_id_head_scores(fake, 8, 2, 64, fake, fake, 96, 0.003, 1e-6, fake, fake, 1 << 30, None) == 1
    assert L.noise_id_head_scores(fake, 8, 2, 64, fake, fake, 64, 0.003, 1e-6, fake, fake, 16, None) == 3
    # the workspace value pass: a 256-byte status block, then bf16 hi + lo of the source
    assert L.noise_value_pass_workspace_bytes(2, 256) == 256 + 2 * 2 * 256 * 64 * 2
    assert L.noise_value_pass_workspace_bytes(0, 256) == 0
    src = _lib.Rows(fake, 256 * 64, 64, 1)
    vp = (fake, fake, 1, fake, ctypes.byref(src), ctypes.byref(src), 2, 256, 128)
    assert L.noise_value_pass_ws(*vp, fake, 16, None) == 3                                     # workspace too small
    assert L.noise_value_pass_ws(*vp, fake + 16, 1 << 30, None) == 2                           # not 256-byte aligned
    assert L.noise_value_pass_ws(fake, fake, 1, fake, ctypes.byref(src), ctypes.byref(src), 2, 256, -1, fake,
                                 1 << 30, None) == 1                                           # negative window
    assert L.noise_value_pass_ws(fake, fake, 7, fake, ctypes.byref(src), ctypes.byref(src), 2, 256, 128, fake,
                                 1 << 30, None) == 4                                           # dtype
    # identity-phase GEMMs
    ptrs = (ctypes.c_void_p * 8)(*([fake] * 8))
    assert L.noise_hidden_credits(ptrs, fake, fake, fake, 8, 128, 256, 128, fake, fake, 16, None) == 3  # workspace
    assert L.noise_hidden_credits(ptrs, fake, fake, fake, 8, 100, 256, 128, fake, fake, 256, None) == 1  # m % 128
    assert L.noise_hidden_credits(ptrs, fake, fake, fake, 9, 128, 256, 128, fake, fake, 256, None) == 1  # > 8 layers
    assert L.noise_at_b_layers(ptrs, ptrs, 8, 100, 128, 128, fake, fake, 256, None) == 1               # k % 64
    assert L.noise_at_b_layers(ptrs, ptrs, 8, 128, 128, 128, fake + 8, fake, 256, None) == 2           # out align
    assert L.noise_square_credit_grads(ptrs, fake, 2, 8, 64, 256, fake, fake, 256, None) == 1         # world 64 != d
    assert L.noise_square_credit_grads(ptrs, None, 2, 8, 64, 128, fake, fake, 256, None) == 4
    # readout scorers
    v = _lib.View3(fake, 1, 1, 1)
    r = ctypes.byref(v)
    assert L.noise_future_scores(r, r, fake, fake, r, r, 0, 64, 2, 2, 0, 8, fake, None) == 1   # no heads
    assert L.noise_future_scores(r, r, fake + 4, fake, r, r, 2, 64, 2, 2, 0, 8, fake, None) == 2  # dk alignment
    assert L.noise_key_response(None, fake, r, r, 2, 64, 2, 2, 0, 0, 8, fake, None) == 4
    fn = L.noise_future_scores_workspace_bytes(8, 2000)
    assert fn == 256 + 4 * 8 * 2048 * 64 * 4 and L.noise_key_response_workspace_bytes(8, 2000) == 256 + 2 * 8 * 2048 * 256
    assert L.noise_future_scores_workspace_bytes(0, 64) == 0
    fs = (r, r, fake, fake, r, r, 8, 2000, 2, 2, 0, 8, fake)
    assert L.noise_future_scores_ws(*fs, fake, fn - 1, None) == 3                               # workspace
    assert L.noise_future_scores_ws(*fs, fake + 16, fn, None) == 2                              # workspace alignment
    assert L.noise_future_scores_ws(r, r, fake + 4, fake, r, r, 8, 2000, 2, 2, 0, 8, fake, fake, fn, None) == 2  # dk
    assert L.noise_key_response_ws(r, fake, r, r, 8, 2000, 2, 2, 0, 0, -1, fake, fake, fn, None) == 1  # window < 0
    assert L.noise_key_response_ws(None, fake, r, r, 8, 2000, 2, 2, 0, 0, 8, fake, fake, fn, None) == 4
    # int32 TMA row coordinates: heads x tokens padded to 64
    assert L.noise_key_response_ws(r, fake, r, r, 1 << 16, 1 << 15, 2, 2, 0, 0, 8, fake, fake, 1 << 42, None) == 1
    assert L.noise_query_response(fake, r, r, r, r, 2, 0, 2, 64, fake, None) == 1
    qn = L.noise_query_response_workspace_bytes(256, 64, 8, 2048)
    assert qn == 256 + 4 * 8 * 2048 * 64 * 4 + 8 * 256 * 32                                   # planes + live flags
    assert L.noise_query_response_workspace_bytes(3, 5, 2, 100) == 256 + 4 * 2 * 128 * 64 * 4 + 256  # keys to 128
    assert L.noise_query_response_workspace_bytes(0, 64, 8, 2048) == 0
    assert L.noise_query_response_workspace_bytes(2, 8, 2, 40000) == 256                     # CUDA-core fall-through
    assert L.noise_query_response_ws(fake, r, r, r, r, 256, 64, 8, 2048, fake, fake, qn - 1, None) == 3  # workspace
    assert L.noise_query_response_ws(fake, r, r, r, r, 256, 64, 8, 2048, fake, fake + 16, qn, None) == 2  # alignment
    assert L.noise_query_response_ws(fake + 4, r, r, r, r, 256, 64, 8, 2048, fake, fake, qn, None) == 2  # dq alignment
    assert L.noise_query_response_ws(fake, None, r, r, r, 256, 64, 8, 2048, fake, fake, qn, None) == 4
    assert L.noise_query_response_ws(fake, r, r, r, r, 256, 64, 0, 2048, fake, fake, qn, None) == 1     # no heads
    assert L.noise_query_response_ws(fake, r, r, r, r, 1, 1, 1 << 16, 1 << 15, fake, fake, 1 << 45, None) == 1  # h Tp
    assert L.noise_expm1_f32(None, fake, 4, None) == 4
    assert L.noise_routed_response(fake, fake, fake, fake, fake, 2, 2, 2, 257, fake, None) == 1  # K > 256
    assert L.noise_routed_response_ws(fake, fake, fake, fake, fake, 2, 2, 2, 257, fake, fake, 256, None) == 1  # K
    assert L.noise_routed_response_ws(fake, fake, fake, fake, fake, 2, 2, 2, 64, fake, fake, 16, None) == 3   # ws
    assert L.noise_routed_response_ws(fake, fake, fake, fake, fake, 2, 2, 2, 64, fake + 4, fake, 256, None) == 2
    assert L.noise_routed_response_ws(None, fake, fake, fake, fake, 2, 2, 2, 64, fake, fake, 256, None) == 4
    # int32 TMA row coordinates: tokens x probes rows, tokens x heads x keys key rows
    assert L.noise_routed_response_ws(fake, fake, fake, fake, fake, 1 << 20, 1 << 11, 1, 64, fake, fake, 256,
                                      None) == 1
    assert L.noise_routed_response_ws(fake, fake, fake, fake, fake, 1 << 20, 1, 16, 256, fake, fake, 256, None) == 1
    # Dust block rerun
    jit = _lib.Jitter()
    assert L.noise_block_forward(ctypes.byref(gpt), 0, fake, None, ctypes.byref(jit), 2, 256, 128, fake, 1 << 30,
                                 None) == 4                                                   # no weights
    assert L.noise_block_forward(None, 0, fake, None, None, 2, 256, 128, fake, 1 << 30, None) == 4
    assert L.noise_block_workspace_bytes(2, 256) == L.noise_population_workspace_bytes(2, 256)
    assert L.noise_head_error_prep(fake, 3, 4096, fake, 4, fake, fake, fake, None) == 4      # dtype
    assert L.noise_head_error_chunk(fake, 0, 4096, fake, fake, fake, fake, fake, fake, 2, 8, 16, 16, 0.1, fake,
                                    None) == 1                                                  # slab out of range
    # readout cycle
    assert L.noise_cycle_weights(None, fake, fake, 4, fake, fake, fake, fake, fake, fake, None) == 4
    assert L.noise_cycle_finish(fake, fake, fake, fake, fake, fake, fake, fake, fake, 4, 0, 0.005, fake, None) == 1
    assert L.noise_coordinate_change(fake, 5, fake, 4, 0.1, fake, None) == 4                  # dtype
    assert L.noise_coordinate_change(fake, 0, fake, 4, 0.0, fake, None) == 1                  # head_sigma
    # readout scorer
    assert L.noise_readout_stats(fake, fake, fake, fake, fake, 0, 8, 4, 2, 1e-7, None) == 1    # d_rows < n
    assert L.noise_readout_stats(fake + 4, fake, fake, fake, fake, 0, 8, 8, 2, 1e-7, None) == 2
    assert L.noise_readout_staged_ws(*([fake] * 8), None, fake, None, 0, 4, 4, 2, 1040, 1, fake, 256, None) == 4
    assert L.noise_readout_direct_ws(fake, fake, fake, 1, 1, fake, 1, 1, None, None, None, fake, None, 0, 4, 2, 1, fake,
                                     256, None) == 4
    tab = _lib.ScorerTables()
    assert L.noise_readout_staged(fake, fake, fake, fake, None, None, fake, fake, ctypes.byref(tab), fake, None,
                                  0, 8, 8, 2, 1040, 1, None) == 4                              # tables missing
    tab = _lib.ScorerTables(*([fake] * 10))
    assert L.noise_readout_staged(fake, fake, fake, fake, None, None, fake, fake, ctypes.byref(tab), fake, None,
                                  0, 8, 8, 2, 1000, 1, None) == 1                              # nc < 1024
    assert L.noise_readout_direct(fake, fake, fake, 32, 1, fake, 32, 1, fake, None, ctypes.byref(tab), fake, None,
                                  0, 8, 2, 1, None) == 4                                       # gated without ve
    # int32 TMA row coordinates: (start + tokens) x 8 heads x 64 moment-table rows
    assert L.noise_readout_staged_ws(fake, fake, fake, fake, None, None, fake, fake, ctypes.byref(tab), fake, None,
                                     (1 << 22) - 1, 8, 8, 2, 1040, 1, fake, 256, None) == 1
    assert L.noise_readout_direct_ws(fake, fake, fake, 32, 1, fake, 32, 1, None, None, ctypes.byref(tab), fake, None,
                                     1 << 22, 8, 1, 1, fake, 256, None) == 1


def test_product_path_has_no_oracle_import():
    for path in (ROOT / 'noise_b200').rglob('*.py'):
        assert 'oracle' not in path.read_text(), path


def test_readout_wrappers_refuse_mismatched_operands():
    """The scorer wrappers check every operand's shape against the dimensions they pass to the kernel (a smaller one
    would be read past its end), then refuse CPU tensors: no CPU fallback."""
    import sys
    sys.path.insert(0, str(ROOT / 'tests' / 'golden'))
    from readout_inputs import future_inputs, key_inputs, query_inputs, routed_inputs
    from noise_b200 import _lib, readout
    f, k, q, r = future_inputs(), key_inputs(), query_inputs(), routed_inputs()
    bad = [
        lambda: readout.future_scores_impl(f['q'], f['target'], f['dk'], f['dv'], f['a'][:, :-1], f['contrast'], 48,
                                           64),
        lambda: readout.future_scores_impl(f['q'], f['target'][:1], f['dk'], f['dv'], f['a'], f['contrast'], 48, 64),
        lambda: readout.key_response_impl(k['q'], k['dk'], k['A'], k['C'][..., :-1], 32, 24, 64),
        lambda: readout.query_response_impl(q['dq'], q['keys'], q['values'], q['probabilities'][:, :-1], q['base']),
        lambda: readout.query_response_impl(q['dq'], q['keys'], q['values'][:, :-1], q['probabilities'], q['base']),
        lambda: readout.routed_response_impl(r['dq'], r['keys'], r['values'], r['probabilities'], r['rest'][:-1]),
        lambda: readout.routed_response_impl(r['dq'], r['keys'], r['values'][:, :, :-1], r['probabilities'],
                                             r['rest']),
    ]
    for call in bad:
        with pytest.raises(ValueError):
            call()
    with pytest.raises(_lib.NoiseError):
        readout.routed_response_impl(r['dq'], r['keys'], r['values'], r['probabilities'], r['rest'])


def test_scorer_wrappers_refuse_mismatched_operands():
    """The readout scorer's wrappers check each operand's dtype, layout and shape (the moment tables must cover the
    chunk's global tokens) before any pointer reaches a kernel, then refuse CPU tensors."""
    import sys
    import torch
    sys.path.insert(0, str(ROOT / 'tests' / 'golden'))
    from scorer_inputs import scorer_inputs, tables
    from noise_b200 import _lib, scorer
    x = scorer_inputs()
    m, n, start, nc = x['m'], x['n'], x['start'], x['nc']
    tok = slice(start, start + m)

    def staged(**bad):
        y = dict(x, **bad)
        scorer.staged_kernel(y['UP'], torch.empty(m, n, 2), y['R0'], y['VC'], y['GZ'], y['VE'], y['CS'], y['SN'],
                             *tables(y), torch.empty(m, n), None, start, n, n, True, True, False, nc)

    def direct(**bad):
        y = dict(x, **bad)
        scorer.readout_kernel(y['PJ'], y['R0'][tok], y['CS'][tok], y['SN'][tok], y['GC'], y['VE'][tok], *tables(y),
                              torch.empty(m, n), None, start, n, True, True, False)
    for call, bad in ((staged, dict(U=x['U'][:start])), (staged, dict(M1=x['M1'].float())),
                      (staged, dict(UP=x['UP'][:-1])), (staged, dict(VC=x['VC'][:, :256])),
                      (direct, dict(PJ=x['PJ'][:, :-1])), (direct, dict(GC=x['GC'][..., :4])),
                      (direct, dict(AD=x['AD'][:start + 1]))):
        with pytest.raises(ValueError):
            call(**bad)
    with pytest.raises(ValueError):  # DB rows a token must be n
        scorer.stats_kernel(x['delta'], x['X'], x['SQX'], torch.empty(m, n + 1, 512, dtype=torch.bfloat16),
                            torch.empty(m, n, 2), start, n, x['d_rows'], x['eps'])
    with pytest.raises(_lib.NoiseError):
        staged()
    with pytest.raises(_lib.NoiseError):
        direct()


def test_gemm_wrappers_refuse_short_operand_lists():
    """The identity-phase GEMMs and the readout cycle check their operand lists and shapes before any pointer array
    reaches the library (a short list would hand a kernel an undefined pointer)."""
    import sys
    import torch
    sys.path.insert(0, str(ROOT / 'tests' / 'golden'))
    from id_inputs import at_b_inputs, hidden_inputs, square_inputs
    from noise_b200 import cycle, id_kernels
    us, steps, credb, w_out_t = hidden_inputs()
    with pytest.raises(AssertionError):
        id_kernels.hidden_credits_fused(us[:7], steps, credb, w_out_t)
    with pytest.raises(AssertionError):
        id_kernels.hidden_credits_fused(us, steps, credb, w_out_t[:, :, :128])
    As, Bs = at_b_inputs()
    with pytest.raises(AssertionError):
        id_kernels.at_b_layers(As, Bs[:7], torch.empty(8, 128, 256, dtype=torch.bfloat16))
    n1s, got2 = square_inputs()
    with pytest.raises(AssertionError):
        id_kernels.square_credit_grads(n1s, got2[:, :7], torch.empty(24, 128, 128, dtype=torch.bfloat16))
    x = torch.randn(4, 512)
    with pytest.raises(ValueError):
        cycle.cycle_weights_fused(x, torch.randn(4, 2048), torch.randn(512, 512))


def test_pack_heads_refuses_mismatched_pieces():
    """pack_heads_kernel checks that every layer has all six pieces, each (n, 512), and an lse of whole sequences, before
    a pointer reaches the library."""
    import sys
    sys.path.insert(0, str(ROOT / 'tests' / 'golden'))
    from heads_inputs import pack_inputs
    from noise_b200 import heads
    p = pack_inputs()
    names = ('qs', 'ks', 'vals', 'outs', 'targets', 'lses')
    for bad in (dict(ks=p['ks'][:1]), dict(vals=[p['vals'][0], p['vals'][1][:-1]]),
                dict(lses=[p['lses'][0], p['lses'][1][:, :4]])):
        with pytest.raises(ValueError):
            heads.pack_heads_kernel(*(dict(p, **bad)[k] for k in names))


def test_dust_wrappers_refuse_mismatched_operands():
    """Dust's block rerun checks every weight's shape and the RoPE positions, and head_error the logits' vocabulary and
    the clean losses, before any pointer reaches the library."""
    import sys
    sys.path.insert(0, str(ROOT / 'tests' / 'golden'))
    from dust_inputs import dust_inputs, head_error_inputs
    from noise_b200 import dust
    x = dust_inputs()
    for w, cos, sin in ((dict(x['w'], fc=x['w']['fc'][:1024]), x['cos'], x['sin']),
                        (dict(x['w'], gate=x['w']['gate'][:4]), x['cos'], x['sin']),
                        (x['w'], x['cos'][:100], x['sin'][:100])):
        with pytest.raises(ValueError):
            dust.block_forward(x['x'], w, x['ve'], cos, sin, 128)
    h = head_error_inputs()
    with pytest.raises(ValueError):
        dust.head_error(h['raw'][..., :2048], h['y'], h['clean_loss'], h['draws'], 0.1, h['nrep'], h['noise'])
    with pytest.raises(ValueError):
        dust.head_error(h['raw'], h['y'], h['clean_loss'][:, :-1], h['draws'], 0.1, h['nrep'], h['noise'])


def test_credit_wrappers_refuse_mismatched_operands():
    """The credit ops check every operand against the rows x T x 64 the kernels address (per-row vectors [rows, T],
    RoPE tables of T positions, blocked raw / out views large enough), before any pointer reaches the library."""
    import sys
    import torch
    sys.path.insert(0, str(ROOT / 'tests' / 'golden'))
    from credit_inputs import credit_inputs
    from noise_b200 import moment_kernels as mk
    x = credit_inputs()
    q, k, v, hub = (z.bfloat16() for z in (x['qp'], x['kp'], x['values'], x['hub']))
    rows, t, _ = q.shape
    lse, sq = torch.zeros(rows, t), torch.ones(rows, t)
    bad = [
        lambda: mk.implicit_key_context_edges_impl(q, k[:, :-1], v, hub, 64),
        lambda: mk.value_pass(q, k, lse[:, :-1], x['hub'], 64),
        lambda: mk.key_scan(x['qp'], x['kp'], x['k_raw'], lse, x['values'], x['hub'], lse, x['cos'][:100],
                            x['sin'][:100], 64, 0.003),
        lambda: mk.key_scan(x['qp'], x['kp'], x['k_raw'], lse, x['values'][:1], x['hub'], lse, x['cos'], x['sin'], 64,
                            0.003),
        lambda: mk.moment_query_scores_impl(q, k, v, hub, x['q_raw'].unsqueeze(0), sq, x['kp'][..., :32], x['cos'],
                                            x['sin'], lse, lse, sq, torch.empty(1, rows, t, 64, dtype=torch.bfloat16)),
        lambda: mk.moment_query_scores_impl(q, k, v, hub, x['q_raw'].unsqueeze(0), sq, x['kp'], x['cos'], x['sin'],
                                            lse, lse, sq, torch.empty(1, rows, t // 2, 64, dtype=torch.bfloat16)),
    ]
    for call in bad:
        with pytest.raises(ValueError):
            call()


def test_population_wrappers_refuse_mismatched_operands():
    """Every parameter is packed into a slot of its GPT shape, so a mismatched one is refused before any pack; the
    head loss needs the LM head's 4096 rows."""
    import torch
    from noise_b200 import population
    from oracle import gpt
    w = gpt.init_weights(0, eggroll=True)
    bad = dict(w)
    bad['transformer.h.0.attn.c_q.weight'] = w['transformer.h.0.attn.c_q.weight'][:256]
    with pytest.raises(ValueError):
        population.PackedGPT(bad)
    missing = {k: v for k, v in w.items() if k != 'lm_head.weight'}
    with pytest.raises(ValueError):
        population.PackedGPT(missing)
    with pytest.raises(ValueError):
        population.head_loss(torch.randn(2, 128, 512), torch.randn(2048, 512), torch.zeros(2, 128, dtype=torch.long))
