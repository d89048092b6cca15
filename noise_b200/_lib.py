"""ctypes binding of the C ABI in include/noise_b200.h (the in-tree libnoise_b200.so).

There is no fallback: if the library is missing or fails to load, every op raises. Device pointers are passed as
integers (``tensor.data_ptr()``), streams as the raw ``cudaStream_t`` of the current PyTorch stream.
"""
import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / 'libnoise_b200.so'

N_LAYER, N_HEAD, HEAD_DIM, N_EMBD, VOCAB, N_PARAMS = 8, 8, 64, 512, 4096, 60
REDUCTION = {'mean': 0, 'sum': 1, 'none': 2}
STATUS_BYTES = 256
STATIC_SCRATCH_BYTES = 48 << 20  # NOISE_STATIC_SCRATCH_BYTES
ERR_TOO_LARGE = 7


class Slice(ctypes.Structure):
    """noise_slice_t."""
    _fields_ = [('a', ctypes.c_void_p), ('b', ctypes.c_void_p), ('off', ctypes.c_void_p),
                ('a_stride', ctypes.c_int64), ('b_stride', ctypes.c_int64)]


class GPT(ctypes.Structure):
    """noise_gpt_t."""
    _fields_ = [('wqkv', ctypes.c_void_p * N_LAYER), ('wproj', ctypes.c_void_p * N_LAYER),
                ('wfc', ctypes.c_void_p * N_LAYER), ('wmproj', ctypes.c_void_p * N_LAYER),
                ('wgate', ctypes.c_void_p * N_LAYER), ('whead', ctypes.c_void_p), ('wte', ctypes.c_void_p),
                ('ve', ctypes.c_void_p * N_LAYER), ('resid_lambdas', ctypes.c_void_p),
                ('x0_lambdas', ctypes.c_void_p), ('cos', ctypes.c_void_p), ('sin', ctypes.c_void_p)]


class Rows(ctypes.Structure):
    """noise_rows_t (block_rows = 0: not blocked)."""
    _fields_ = [('data', ctypes.c_void_p), ('layer_stride', ctypes.c_int64), ('token_stride', ctypes.c_int64),
                ('heads', ctypes.c_int), ('layer_map', ctypes.c_void_p), ('block_rows', ctypes.c_int),
                ('per_gpu', ctypes.c_int64), ('gpu_stride', ctypes.c_int64)]


class View3(ctypes.Structure):
    """noise_view3_t."""
    _fields_ = [('data', ctypes.c_void_p), ('stride0', ctypes.c_int64), ('stride1', ctypes.c_int64),
                ('stride2', ctypes.c_int64)]


class Jitter(ctypes.Structure):
    """noise_jitter_t."""
    _fields_ = [(n, ctypes.c_void_p) for n in ('o', 'attn', 'fc', 'mlp')]


class ScorerTables(ctypes.Structure):
    """noise_scorer_tables_t."""
    _fields_ = [(n, ctypes.c_void_p) for n in ('U', 'W', 'M1', 'M2', 'QD', 'GD', 'AD', 'CD', 'VT', 'OT')]


class HeadPieces(ctypes.Structure):
    """noise_head_pieces_t."""
    _fields_ = [(n, ctypes.c_void_p) for n in ('q', 'k', 'v', 'o', 'target')] + \
               [(n + '_stride', ctypes.c_int64) for n in ('q', 'k', 'v', 'o', 'target')] + [('lse', ctypes.c_void_p)]


class Peers(ctypes.Structure):
    """noise_peers_t."""
    _fields_ = [('base', ctypes.c_void_p * 8), ('rank', ctypes.c_int), ('world', ctypes.c_int)]


class HeadPrep(ctypes.Structure):
    """noise_head_prep_t."""
    _fields_ = [(n, ctypes.c_void_p) for n in ('q16', 'k16', 'v16', 'hub16', 'q32', 'k32', 'f2', 'f4', 'xy', 'lse',
                                               'hub_out', 'sq_q', 'sq_k', 'steps_q', 'steps_k')]


class NoiseError(RuntimeError):
    pass


_lib = None

# (name, restype, argtypes) of every exported entry point; tests check each one is present.
SIGNATURES = [
    ('noise_param_index', ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    ('noise_attention_item', ctypes.c_int, [ctypes.c_int] * 5 + [ctypes.POINTER(ctypes.c_int)] * 2),
    ('noise_population_workspace_bytes', ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    ('noise_population_loss', ctypes.c_int,
     [ctypes.POINTER(GPT), ctypes.POINTER(Slice), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
      ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_gpt_workspace_bytes', ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    ('noise_gpt_loss', ctypes.c_int,
     [ctypes.POINTER(GPT), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_head_loss_workspace_bytes', ctypes.c_size_t, [ctypes.c_int]),
    ('noise_head_loss', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
      ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_population_loss_noalloc', ctypes.c_int,
     [ctypes.POINTER(GPT), ctypes.POINTER(Slice), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
      ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_read_static_status', ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]),
    ('noise_gemm_bf16_tn', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
      ctypes.c_void_p]),
    ('noise_gemm_tf32_tn', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
      ctypes.c_void_p]),
    ('noise_pack_bf16', ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    ('noise_rank1_operands', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
      ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_rank1_operands_f32', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
      ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_rank1_small', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int,
      ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_adam_step', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_float,
      ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]),
    ('noise_implicit_key_context', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
      ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_value_pass', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(Rows), ctypes.POINTER(Rows),
      ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    ('noise_implicit_key_context_ws', ctypes.c_int,
     [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_void_p] * 3 + [ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_value_pass_workspace_bytes', ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    ('noise_value_pass_ws', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(Rows), ctypes.POINTER(Rows),
      ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_key_scan', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
      ctypes.POINTER(Rows), ctypes.POINTER(Rows), ctypes.c_void_p]),
    ('noise_moment_key_scores', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
      ctypes.c_int, ctypes.c_int, ctypes.POINTER(Rows), ctypes.POINTER(Rows), ctypes.c_void_p]),
    ('noise_moment_query_scores', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
      ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(Rows), ctypes.c_int, ctypes.c_void_p]),
    ('noise_moment_key_scores_v', ctypes.c_int,
     [ctypes.c_void_p] * 4 + [ctypes.POINTER(Rows), ctypes.c_int] + [ctypes.c_void_p] * 7 + [ctypes.c_int,
      ctypes.c_int, ctypes.POINTER(Rows), ctypes.POINTER(Rows), ctypes.c_int, ctypes.c_void_p]),
    ('noise_key_scan_workspace_bytes', ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    ('noise_key_scan_ws', ctypes.c_int,
     [ctypes.c_void_p] * 9 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.POINTER(Rows),
      ctypes.POINTER(Rows), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_moment_key_scores_workspace_bytes', ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    ('noise_moment_key_scores_ws', ctypes.c_int,
     [ctypes.c_void_p] * 4 + [ctypes.POINTER(Rows), ctypes.c_int] + [ctypes.c_void_p] * 7 + [ctypes.c_int,
      ctypes.c_int, ctypes.POINTER(Rows), ctypes.POINTER(Rows), ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
      ctypes.c_void_p]),
    ('noise_moment_query_scores_workspace_bytes', ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    ('noise_moment_query_scores_ws', ctypes.c_int,
     [ctypes.c_void_p] * 4 + [ctypes.POINTER(Rows), ctypes.c_int] + [ctypes.c_void_p] * 7 + [ctypes.c_int,
      ctypes.c_int, ctypes.c_int, ctypes.POINTER(Rows), ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
      ctypes.c_void_p]),
    ('noise_moment_query_scores_v', ctypes.c_int,
     [ctypes.c_void_p] * 4 + [ctypes.POINTER(Rows), ctypes.c_int] + [ctypes.c_void_p] * 7 + [ctypes.c_int,
      ctypes.c_int, ctypes.c_int, ctypes.POINTER(Rows), ctypes.c_int, ctypes.c_void_p]),
    ('noise_pack_heads', ctypes.c_int,
     [ctypes.POINTER(HeadPieces), ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_head_prep', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
      ctypes.c_float, ctypes.c_float, ctypes.POINTER(HeadPrep), ctypes.c_void_p]),
    ('noise_id_head_scores_workspace_bytes', ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    ('noise_id_head_scores', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
      ctypes.c_float, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_exchange_alloc', ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
    ('noise_exchange_open', ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    ('noise_exchange_close', ctypes.c_int, [ctypes.c_void_p]),
    ('noise_exchange_free', ctypes.c_int, [ctypes.c_void_p]),
    ('noise_exchange_wait', ctypes.c_int,
     [ctypes.POINTER(Peers), ctypes.c_int, ctypes.c_uint32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_alltoall_peer', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(Peers), ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32,
      ctypes.c_void_p]),
    ('noise_pack_heads_peer', ctypes.c_int,
     [ctypes.POINTER(HeadPieces), ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(Peers), ctypes.c_size_t,
      ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p]),
    ('noise_hidden_credits', ctypes.c_int,
     [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
      ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_at_b_layers', ctypes.c_int,
     [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int, ctypes.c_int,
      ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_square_credit_grads', ctypes.c_int,
     [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_future_scores', ctypes.c_int,
     [ctypes.POINTER(View3), ctypes.POINTER(View3), ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(View3),
      ctypes.POINTER(View3)] + [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_key_response', ctypes.c_int,
     [ctypes.POINTER(View3), ctypes.c_void_p, ctypes.POINTER(View3),
      ctypes.POINTER(View3)] + [ctypes.c_int] * 7 + [ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_future_scores_workspace_bytes', ctypes.c_size_t, [ctypes.c_int] * 2),
    ('noise_key_response_workspace_bytes', ctypes.c_size_t, [ctypes.c_int] * 2),
    ('noise_future_scores_ws', ctypes.c_int,
     [ctypes.POINTER(View3), ctypes.POINTER(View3), ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(View3),
      ctypes.POINTER(View3)] + [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
       ctypes.c_void_p]),
    ('noise_key_response_ws', ctypes.c_int,
     [ctypes.POINTER(View3), ctypes.c_void_p, ctypes.POINTER(View3),
      ctypes.POINTER(View3)] + [ctypes.c_int] * 7 + [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
       ctypes.c_void_p]),
    ('noise_query_response', ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(View3), ctypes.POINTER(View3), ctypes.POINTER(View3),
      ctypes.POINTER(View3)] + [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_expm1_f32', ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    ('noise_query_response_workspace_bytes', ctypes.c_size_t, [ctypes.c_int] * 4),
    ('noise_query_response_ws', ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(View3), ctypes.POINTER(View3), ctypes.POINTER(View3),
      ctypes.POINTER(View3)] + [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
       ctypes.c_void_p]),
    ('noise_routed_response', ctypes.c_int,
     [ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_routed_response_ws', ctypes.c_int,
     [ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_readout_stats', ctypes.c_int,
     [ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_void_p]),
    ('noise_readout_staged', ctypes.c_int,
     [ctypes.c_void_p] * 8 + [ctypes.POINTER(ScorerTables), ctypes.c_void_p,
      ctypes.c_void_p] + [ctypes.c_int] * 6 + [ctypes.c_void_p]),
    ('noise_readout_staged_ws', ctypes.c_int,
     [ctypes.c_void_p] * 8 + [ctypes.POINTER(ScorerTables), ctypes.c_void_p,
      ctypes.c_void_p] + [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_readout_direct_ws', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
      ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ScorerTables), ctypes.c_void_p,
      ctypes.c_void_p] + [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_readout_direct', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
      ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ScorerTables), ctypes.c_void_p,
      ctypes.c_void_p] + [ctypes.c_int] * 4 + [ctypes.c_void_p]),
    ('noise_cycle_weights', ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] + [ctypes.c_void_p] * 7),
    ('noise_cycle_finish', ctypes.c_int,
     [ctypes.c_void_p] * 9 + [ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_coordinate_change', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_block_workspace_bytes', ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
    ('noise_block_forward', ctypes.c_int,
     [ctypes.POINTER(GPT), ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(Jitter), ctypes.c_int,
      ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    ('noise_head_error_prep', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 4),
    ('noise_head_error_chunk', ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64] + [ctypes.c_void_p] * 6 + [ctypes.c_int] * 4 +
     [ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_read_status', ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]),
    ('noise_clear_status', ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    ('noise_status_string', ctypes.c_char_p, [ctypes.c_int]),
    ('noise_last_launch_count', ctypes.c_int, []),
    ('noise_profile_start', ctypes.c_int, [ctypes.c_int]),
    ('noise_profile_stop', ctypes.c_int,
     [ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int), ctypes.c_int]),
]


def lib():
    """The loaded library (raises NoiseError when it is missing: there is no CPU path)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NoiseError(f'{LIB_PATH} is missing: build it with `python -m noise_b200.build`')
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def check(status, what):
    if status != 0:
        raise NoiseError(f'{what}: {lib().noise_status_string(status).decode()} (status {status})')


def stream_handle(device=None):
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors):
    for t in tensors:
        if not t.is_cuda:
            raise NoiseError('noise_b200 ops run on CUDA tensors only (no CPU fallback)')


def read_status(workspace):
    """Device status word at the head of a workspace (synchronises the current stream)."""
    out = ctypes.c_int(0)
    check(lib().noise_read_status(workspace.data_ptr(), ctypes.byref(out), stream_handle(workspace.device)),
          'noise_read_status')
    return out.value


def read_static_status(device):
    """Device status word of the no-allocation entry point's static scratch on ``device`` (synchronises the
    device's current stream)."""
    out = ctypes.c_int(0)
    with torch.cuda.device(device):
        check(lib().noise_read_static_status(ctypes.byref(out), stream_handle(device)), 'noise_read_static_status')
    return out.value


def launches():
    return lib().noise_last_launch_count()


def _gemm(entry, dtype, a, b, out=None):
    require_cuda(a, b, *(() if out is None else (out,)))
    if a.dtype != dtype or b.dtype != dtype or a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError(f'{entry}: a [m, k] and b [n, k] of {dtype}')
    a, b = a.contiguous(), b.contiguous()
    if out is None:
        out = torch.empty((a.shape[0], b.shape[0]), dtype=torch.float32, device=a.device)
    elif out.shape != (a.shape[0], b.shape[0]) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError(f'{entry}: out must be contiguous fp32 [m, n]')
    ws = torch.empty(STATUS_BYTES, dtype=torch.uint8, device=a.device)
    check(getattr(lib(), entry)(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.shape[0], b.shape[0], a.shape[1],
                                ws.data_ptr(), stream_handle(a.device)), entry)
    out._noise_workspace = ws
    return out


def gemm_bf16_tn(a, b, out=None):
    """fp32 a @ b.T for bf16 a [m, k], b [n, k] on the tcgen05 GEMM core (n % 32 == 0, k % 8 == 0)."""
    return _gemm('noise_gemm_bf16_tn', torch.bfloat16, a, b, out)


def gemm_tf32_tn(a, b, out=None):
    """a @ b.T for fp32 a [m, k], b [n, k] at tf32 precision (torch's 'high') on the tcgen05 GEMM core (n % 32 == 0,
    k % 4 == 0)."""
    return _gemm('noise_gemm_tf32_tn', torch.float32, a, b, out)


KINDS = ['norm_mix', 'gemm_qkv', 'attention', 'gemm_cproj', 'norm_mid', 'gemm_cfc', 'gemm_mproj', 'norm_final',
         'gemm_head_ce', 'member_reduce', 'gemm_plain']


class LaunchProfile:
    """Context manager: per-kernel-kind CUDA-event times of the launches made inside it (this thread).
    After exit, ``.ms[kind]`` and ``.count[kind]`` hold the summed milliseconds and launch counts."""

    def __init__(self, capacity=100000):
        self.capacity, self.ms, self.count = capacity, {}, {}

    def __enter__(self):
        check(lib().noise_profile_start(self.capacity), 'noise_profile_start')
        return self

    def __exit__(self, *exc):
        n = len(KINDS)
        ms, cnt = (ctypes.c_float * n)(), (ctypes.c_int * n)()
        check(lib().noise_profile_stop(ms, cnt, n), 'noise_profile_stop')
        self.ms = {k: ms[i] for i, k in enumerate(KINDS) if cnt[i]}
        self.count = {k: cnt[i] for i, k in enumerate(KINDS) if cnt[i]}
        return False
