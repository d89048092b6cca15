"""Benchmark of Noise's forward-only training hot path on B200s (BASELINE.json's metric: train tokens/sec at
population 24k on 1/2/4/8 B200; population forwards/sec/GPU).

Default (--workload train): one step = one EGGROLL update at population 24,576 (12,288 antithetic
pairs, sigma 2e-3) of the fixed 37.7M GPT (random init of utils/model.py's architecture, EGGROLL's make_model) on 8
rows x 2048 synthetic Zipf(1.1) tokens: the population forward of this rank's members (rank-1 noise read in place
from EGGROLL's 2**28-value N(0, 1) buffer at the step's offsets), the fitness all-gather, the seed-rebuilt update on
this rank's pair shard with one NCCL all-reduce, and AdamW. The population is split over the ranks (strong scaling).
Unit: train tokens/s (16,384 per update, all GPUs); the line's config also carries population forwards/s/GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload train|population|credit|aux|exchange]

--workload population times the population forward alone (BASELINE config 2 per GPU: 512 members x 8 rows x 2048
tokens, weak scaling, population forwards/s); --workload credit the credit-readout kernels in isolation (config 3);
--workload aux the other entry points (un-perturbed forward, head loss, head sharding, readout scorers);
--workload exchange the identity phase's head exchange (pack + heads-in + heads-out all_to_all) as the reference does
it (pack kernel, NCCL all_to_all_single) and fused over peer memory (HeadExchange), N ranks under torchrun;
--workload epoch the first --updates updates of a one-epoch run with its projected wall time.

--impl reference times the reference on the host CPU (its own eggroll.population_loss from baseline/_ref when
installed, else the oracle restatement of it; fp32, all host threads) on a bounded sample of the same workload, rank 0
only, in the same unit.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = 'train tokens/sec at pop 24k on 1/2/4/8 B200; population forwards/sec/GPU'
UNIT = 'population forwards/s (one member x one 2048-token row, all GPUs)'  # the --workload population line
POP_METRIC = 'population forwards/sec/GPU (BASELINE config 2: 512 members x 8 x 2048 tokens per GPU)'
MEMBERS, ROWS, T, SIGMA = 512, 8, 2048, 1e-3
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per member-token row of each kernel kind, from one ncu
# capture of a 64-member x 1-row call (bench.py --members 64 --rows 1), scaled by the rows of a launch
TRAFFIC_BYTES_PER_ROW = {'norm_mix': 4437.3, 'gemm_qkv': 3750.1, 'attention': 9496.0, 'gemm_cproj': 4701.4,
                         'norm_mid': 2846.1, 'gemm_cfc': 4835.0, 'gemm_mproj': 10803.6, 'norm_final': 2846.7,
                         'gemm_head_ce': 1083.2, 'member_reduce': 16.2}
FLOP_PER_MEMBER_TOKEN = 68.3e6  # algorithmic forward FLOPs per member-token (linears + attention)
CPU_SAMPLE_MEMBERS, CPU_SAMPLE_T = 2, 2048
TRAIN_PAIRS, TRAIN_ROWS = 12288, 8  # population 24,576, eggroll.py's BATCH of 8 rows
TRAIN_UNIT = 'train tokens/s (all GPUs)'
# one update = 24,576 population forwards (members x one 2048-token row) for 8 x 2048 train tokens
TRAIN_FORWARDS, TRAIN_TOKENS = 2 * TRAIN_PAIRS, TRAIN_ROWS * T


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=5)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--workload', default='train',
                    choices=['train', 'population', 'credit', 'aux', 'exchange', 'epoch'])
    ap.add_argument('--updates', type=int, default=100, help='timed updates of the bounded epoch run (--workload epoch)')
    # smaller population cases for profiling captures only; the benchmark line uses the defaults
    ap.add_argument('--members', type=int, default=MEMBERS, help='members per GPU (population workload)')
    ap.add_argument('--rows', type=int, default=ROWS, help='2048-token rows per member (population workload)')
    return ap.parse_args()


def zipf_rows(rows, length, seed):
    p = torch.arange(1, 4097, dtype=torch.float64) ** -1.1
    g = torch.Generator().manual_seed(seed)
    return torch.multinomial((p / p.sum()).float(), rows * length, replacement=True, generator=g).view(rows, length)


# ------------------------------------------------------------------------------------------------------------------
# window attention pair counts (for the algorithmic FLOPs of the attention kernel)
# ------------------------------------------------------------------------------------------------------------------
def visible_pairs(length, window):
    return sum(min(t, window) + 1 for t in range(length))


WINDOWS = [1024, 1024, 1024, 2048, 1024, 1024, 1024, 2048]


def attention_order():
    """The attention kernel's work order this run uses (the library reads NOISE_B200_ATTN_ORDER: "1", "2" or default
    0)."""
    return {'1': 1, '2': 2}.get(os.environ.get('NOISE_B200_ATTN_ORDER'), 0)


def kernel_work(kind, members, length):
    """(algorithmic FLOPs, algorithmic HBM bytes) of ONE launch of a kernel kind on members x length rows."""
    M = members * length
    gemm = {'gemm_qkv': (512, 1536), 'gemm_cproj': (512, 512), 'gemm_cfc': (512, 2048), 'gemm_mproj': (2048, 512),
            'gemm_head_ce': (512, 4096)}
    if kind in gemm:
        k, n = gemm[kind]
        return 2.0 * M * n * k, None
    if kind == 'attention':
        pairs = sum(visible_pairs(length, w) for w in WINDOWS) / len(WINDOWS)
        return 4.0 * 64 * pairs * members * 8, None
    # HBM-bound kernels: algorithmic bytes (fp32 residual stream 2 KB / row, bf16 activations 1 KB / row)
    per_row = {'norm_mix': 2048 + 2048 + 1024 + 48,  # read x, write mixed x, write h, rank-1 dots + gates
               'norm_mid': 2048 + 1024 + 16, 'norm_final': 2048 + 1024 + 16,
               'member_reduce': 16}
    if kind in per_row:
        return None, float(per_row[kind]) * M
    return None, None


class Clocks:
    """nvidia-smi samples (200 ms) of this GPU while the timed region runs."""

    def __init__(self, device):
        self.samples, self.proc = [], None
        try:
            ident = 'GPU-' + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            ident = str(device.index)
        q = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={q}', '--format=csv,noheader,nounits',
                                          '-lms', '200', '-i', ident], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(',')]
            if len(parts) >= 9:
                self.samples.append(parts)

    def stop(self):
        if self.proc is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable']}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        sm, mx, reasons = [], [], set()
        for s in self.samples:
            try:
                sm.append(float(s[1]))
                mx.append(float(s[2]))
            except ValueError:
                continue
            for name, val in zip(names, s[5:9]):
                if val.lower().startswith('active'):
                    reasons.add(name)
        load = [c for c in sm if mx and c > 0.3 * max(mx)] or sm
        return {'sm_mhz': statistics.median(load) if load else None, 'sm_max_mhz': max(mx) if mx else None,
                'reasons': sorted(reasons), 'samples': len(self.samples)}


REFERENCE_ROOT = ROOT / 'baseline' / '_ref'
_CPU_CASE = {}


def _cpu_case(threads):
    """The CPU baseline's prepared case: ('reference', call) running the reference's own eggroll.population_loss from
    its install in baseline/_ref (eager flex attention: compiled flex attention does not lower on the CPU; the noise
    buffer shrunk from 2**28 to 2**20 values, which changes which values a member reads, not the work), else ('port',
    call) running the oracle's restatement. Either way fp32 on CPU_SAMPLE_MEMBERS members x CPU_SAMPLE_T tokens of
    EGGROLL's make_model weights."""
    if threads in _CPU_CASE:
        return _CPU_CASE[threads]
    torch.set_num_threads(threads)
    tok = zipf_rows(1, CPU_SAMPLE_T + 1, seed=0)[0]
    idx, tgt = tok[:-1], tok[1:].contiguous()
    sign = torch.tensor([SIGMA, -SIGMA])
    path = REFERENCE_ROOT / 'archive' / '10M' / 'train' / 'val' / 'eggroll.py'
    case = None
    if path.exists():
        try:
            import importlib.util
            sys.path.insert(0, str(REFERENCE_ROOT))
            import utils.model as model
            from torch.nn.attention.flex_attention import flex_attention
            model.flex = flex_attention
            spec = importlib.util.spec_from_file_location('reference_eggroll', path)
            eg = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(eg)
            eg.NOISE = 2 ** 20
            net = eg.make_model(torch.device('cpu'), 0)
            es = eg.Eggroll(net, 1)
            nz = es.noise(es.offsets(step=1), torch.tensor([0, 0]))
            case = ('reference', lambda: eg.population_loss(net, es.params, nz, sign, idx, tgt))
        except Exception as exc:  # noqa: BLE001 - the port below is the documented fallback
            print(f'cpu baseline: the reference install did not load ({exc!r}); timing the oracle port', flush=True)
    if case is None:
        from oracle import eggroll as oe, gpt as og  # the CPU baseline leg only
        w = og.init_weights(0, eggroll=True)
        buf = oe.make_buffer(2 ** 20, seed=0)
        shapes = og.param_shapes()
        nz = oe.noise(buf, oe.offsets(shapes, 1, step=1, n_noise=2 ** 20), torch.tensor([0, 0]), shapes)
        case = ('port', lambda: oe.population_loss(w, nz, sign, idx, tgt))
    _CPU_CASE[threads] = case
    return case


def cpu_reference_sample(threads):
    """(seconds of one CPU population forward of CPU_SAMPLE_MEMBERS members x CPU_SAMPLE_T tokens, its kind)."""
    kind, call = _cpu_case(threads)
    torch.set_num_threads(threads)
    t0 = time.perf_counter()
    with torch.no_grad():
        call()
    return time.perf_counter() - t0, kind


def run_reference(a):
    """The reference arm: the reference's own eggroll.population_loss (baseline/_ref; the fp32 oracle port of it when
    the install is absent) on all the host cores, rank 0 only, each step a bounded sample of the workload, reported in
    the unit of our arm's line."""
    rank = int(os.environ.get('RANK', 0))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    per = CPU_SAMPLE_MEMBERS * CPU_SAMPLE_T / 2048  # population forwards per sample
    for _ in range(max(a.warmup, 1)):
        _, kind = cpu_reference_sample(threads)
    times = [cpu_reference_sample(threads)[0] for _ in range(a.steps)]
    fwd = per * len(times) / sum(times)
    what = ("the reference's own eggroll.population_loss (baseline/_ref, eager flex attention)" if kind == 'reference'
            else 'oracle restatement of eggroll.population_loss, dense attention')
    if a.workload == 'population':
        value, unit, metric, scaling = fwd, UNIT, POP_METRIC, 'weak'
        workload = 'population forward, BASELINE config 2 shape, bounded CPU sample'
        conv = ''
    else:
        value, unit, metric, scaling = fwd * TRAIN_TOKENS / TRAIN_FORWARDS, TRAIN_UNIT, METRIC, 'strong'
        workload = 'BASELINE config 4 update (population 24,576), bounded CPU sample of its population forward'
        conv = '; x 16,384 train tokens per 24,576 population forwards of an update'
    sample = (f'{CPU_SAMPLE_MEMBERS} members x {CPU_SAMPLE_T} tokens of the fp32 population forward per step '
              f'({what}){conv}')
    print(json.dumps({
        'impl': 'reference', 'metric': metric, 'value': value, 'unit': unit, 'n_gpus': a.gpus, 'steps': a.steps,
        'warmup': a.warmup, 'ms_per_step': 1e3 * sum(times) / len(times), 'higher_is_better': True,
        'scaling': scaling, 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
        'config': {'workload': workload, 'members_per_step': CPU_SAMPLE_MEMBERS, 'seq_len': CPU_SAMPLE_T,
                   'population_forwards_per_s': fwd},
        'cpu_baseline': {'value': value, 'unit': unit, 'cores': threads, 'kind': kind, 'sample': sample},
        'e2e': {'value': value, 'unit': unit, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }), flush=True)


def kernel_roofline(prof, m_launch, clk, ms, forwards):
    """{'roofline', 'kernels', 'clocks'} of a timed region: per kernel kind its launches, CUDA-event time per launch,
    share and achieved rate; the roofline object of the dominant kind (algorithmic FLOPs or bytes of one launch on
    m_launch members x T rows over its mean launch time, against MEASURED_PEAKS.json); ``step`` = the forward's
    algorithmic FLOPs of ``forwards`` population forwards over the ``ms`` of the timed region."""
    kinds = {}
    peaks = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text()) if (ROOT / 'MEASURED_PEAKS.json').exists() else {}
    tf_peak = peaks.get('bf16_tflops_sustained', 1400.0)
    total = sum(prof.ms.values())
    for k, kms in prof.ms.items():
        n = prof.count[k]
        flops, nbytes = kernel_work(k, m_launch, T)
        per = kms / n
        kinds[k] = {'launches': n, 'ms_per_launch': round(per, 4), 'share': round(kms / total, 4)}
        if flops:
            kinds[k]['tflops'] = round(flops / (per / 1e3) / 1e12, 1)
        if nbytes:
            kinds[k]['gbs'] = round(nbytes / (per / 1e3) / 1e9, 1)
    dom = max(prof.ms, key=prof.ms.get)
    flops, nbytes = kernel_work(dom, m_launch, T)
    per_launch_s = prof.ms[dom] / prof.count[dom] / 1e3
    tr = TRAFFIC_BYTES_PER_ROW.get(dom)
    step_tf = forwards * T * FLOP_PER_MEMBER_TOKEN / (ms / 1e3) / 1e12
    src = 'MEASURED_PEAKS.json (of measured)' if peaks else 'fallback'
    if flops:
        roofline = {'kernel': dom, 'bound': 'tensor', 'achieved': round(flops / per_launch_s / 1e12, 1),
                    'peak': tf_peak, 'unit': 'TFLOP/s', 'frac': round(flops / per_launch_s / 1e12 / tf_peak, 4),
                    'peak_source': src + ' bf16_tflops_sustained', 'algorithmic_flops_per_launch': flops}
    else:
        hbm = peaks.get('hbm_gbs', 6650.0)
        roofline = {'kernel': dom, 'bound': 'hbm', 'achieved': round(nbytes / per_launch_s / 1e9, 1), 'peak': hbm,
                    'unit': 'GB/s', 'frac': round(nbytes / per_launch_s / 1e9 / hbm, 4),
                    'peak_source': src + ' hbm_gbs', 'algorithmic_bytes_per_launch': nbytes}
    roofline['traffic'] = tr * m_launch * T if tr is not None else None
    roofline['step'] = {'achieved_tflops': round(step_tf, 1), 'frac': round(step_tf / tf_peak, 4)}
    if dom == 'attention':
        # attention's other roof: one exponential per visible pair on the MUFU pipe, at its nominal 16 a SM-cycle
        # (not a measured peak) and the median SM clock sampled under load
        mhz = (clk or {}).get('sm_mhz') or peaks.get('sm_max_mhz', 1965.0)
        exp_rate = flops / 256.0 / per_launch_s
        mufu_peak = 16 * 148 * mhz * 1e6
        roofline['mufu'] = {'achieved_gexp_s': round(exp_rate / 1e9, 1),
                            'nominal_peak_gexp_s': round(mufu_peak / 1e9, 1),
                            'frac': round(exp_rate / mufu_peak, 4), 'sm_mhz': mhz,
                            'basis': 'nominal 16 ex2 per SM-cycle x 148 SMs at the median SM clock under load'}
    return {'roofline': roofline, 'kernels': kinds, 'clocks': clk}


def cpu_baseline_train():
    """The CPU baseline in train tokens/s: the population forward's fp32 oracle port timed on the host cores (a
    bounded sample), scaled by the forwards an update needs (24,576 member rows for 8 x 2048 train tokens; the
    update's rebuild and AdamW, under 2% of an update here, are left out)."""
    threads = os.cpu_count() or 1
    cpu_reference_sample(threads)  # warm-up
    runs = [cpu_reference_sample(threads) for _ in range(2)]
    kind = runs[0][1]
    fwd = CPU_SAMPLE_MEMBERS * CPU_SAMPLE_T / 2048 / statistics.median(r[0] for r in runs)
    what = "the reference's own eggroll.population_loss (eager flex)" if kind == 'reference' else \
        'the oracle restatement of eggroll.population_loss'
    return {'value': fwd * TRAIN_TOKENS / TRAIN_FORWARDS, 'unit': TRAIN_UNIT, 'cores': threads, 'kind': kind,
            'sample': f'{CPU_SAMPLE_MEMBERS} members x {CPU_SAMPLE_T} tokens of {what}, fp32, median of 2 '
                      f'({fwd:.3f} population forwards/s), x 16,384 train tokens per 24,576 population forwards'}


def run_ours(a):
    import noise_b200
    from noise_b200 import _lib
    from noise_b200.eggroll import Population, make_params

    rank, world = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    device = torch.device('cuda', local)
    torch.cuda.set_device(device)
    if world > 1:
        torch.distributed.init_process_group('nccl', device_id=device, timeout=timedelta(seconds=300))
    dist = world > 1

    params = make_params(device, seed=0)
    pairs = a.members // 2 * world
    pop = Population(params, pairs, sigma=SIGMA, seed=0, rank=rank, world=world)
    host_rows = [zipf_rows(a.rows, T + 1, seed=1000 * s + 7).pin_memory() for s in range(2)]
    dev_rows = [r.to(device) for r in host_rows]
    torch.cuda.synchronize()

    def step(i, tokens):
        _, fit = pop.evaluate(tokens, step=i + 1, rows_per_member=a.rows, reduction='sum')
        return fit

    for i in range(a.warmup):
        step(i, dev_rows[i % 2])
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()

    # device-resident timed region
    clocks = Clocks(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with _lib.LaunchProfile() as prof:
        e0.record()
        for i in range(a.steps):
            step(a.warmup + i, dev_rows[i % 2])
            launches += pop.launches
        e1.record()
        torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)

    # end-to-end: host token rows -> device, evaluate, fitness -> host, every step
    fit_host = torch.empty(a.members * world, pin_memory=True)
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for i in range(a.steps):
        tokens = host_rows[i % 2].to(device, non_blocking=True)
        fit = step(a.warmup + a.steps + i, tokens)
        fit_host.copy_(fit, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    f1.record()
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1)
    if dist:
        t = torch.tensor([ms, ms_e2e], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, ms_e2e = t.tolist()

    work = a.members * a.rows * world * a.steps  # population forwards (member x 2048-token row) in the timed region
    value = work / (ms / 1e3)
    e2e_value = work / (ms_e2e / 1e3)

    m_launch = min(pop.chunk, a.members)  # members per library call
    forwards = a.members * a.rows * a.steps  # this rank's population forwards in the timed region
    line = {
        'metric': POP_METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': a.steps, 'warmup': a.warmup,
        'ms_per_step': ms / a.steps, 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
        'dtype': 'bf16',
        'data': 'synthetic: Zipf(1.1) token rows over vocab 4096; random-init weights of the utils/model.py GPT '
                '(EGGROLL make_model); EGGROLL 2**28 N(0,1) noise buffer',
        'config': {'workload': ('BASELINE config 2 per GPU: population forward of 512 antithetic members x 8 rows x '
                                '2048 tokens (summed-CE fitness), NCCL all-gather of fitness'
                                if (a.members, a.rows) == (MEMBERS, ROWS) else
                                f'profiling case (not the benchmark config): {a.members} members x {a.rows} rows'),
                   'members_per_gpu': a.members, 'rows_per_member': a.rows, 'seq_len': T, 'sigma': SIGMA,
                   'member_tokens_per_s': value * T, 'train_tokens_per_step': a.rows * T,
                   'l2': 'inputs larger than L2 (per-call activations ~11 GB)', 'parallelism': f'members x{world}',
                   'attention_order': attention_order()},
        'e2e': {'value': e2e_value, 'unit': UNIT, 'h2d_bytes_per_step': a.rows * (T + 1) * 8,
                'd2h_bytes_per_step': a.members * world * 4},
        'gpu_launches': launches,
    }
    line.update(kernel_roofline(prof, m_launch, clk, ms, forwards))
    if rank == 0 and world == 1:
        threads = os.cpu_count() or 1
        cpu_reference_sample(threads)  # warm-up
        runs = [cpu_reference_sample(threads) for _ in range(2)]
        cv = CPU_SAMPLE_MEMBERS * CPU_SAMPLE_T / 2048 / statistics.median(r[0] for r in runs)
        line['cpu_baseline'] = {'value': cv, 'unit': UNIT, 'cores': threads, 'kind': runs[0][1],
                                'sample': f'{CPU_SAMPLE_MEMBERS} members x {CPU_SAMPLE_T} tokens, fp32 '
                                          f'eggroll.population_loss ({runs[0][1]}), median of 2'}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------------------------------------------------------
# credit kernels in isolation
# ------------------------------------------------------------------------------------------------------------------
CREDIT_FLOP_PER_PAIR = {  # algorithmic FLOPs per visible (receiver, key) pair, one multiply-add = 2
    'implicit_key_context': 256, 'value_pass': 384, 'key_scan': 704, 'moment_query_scores': 1152,
    'moment_key_scores': 832}


REFERENCE_MOMENT_KERNELS = ROOT / 'baseline' / '_ref' / 'train' / 'speedrun' / 'moment_kernels.py'


def reference_moment_kernels():
    """The reference's own Triton credit kernels (train/speedrun/moment_kernels.py, unmodified, from the reference
    install in baseline/_ref) with KEY_IMPL = VALUE_IMPL = None: the B200 reference for BASELINE config 3 (the Gluon
    versions need Hopper's wgmma). Raises FileNotFoundError when the install is absent."""
    import importlib.util
    if not REFERENCE_MOMENT_KERNELS.exists():
        raise FileNotFoundError(f'{REFERENCE_MOMENT_KERNELS} is missing (the reference install in baseline/_ref)')
    spec = importlib.util.spec_from_file_location('reference_moment_kernels', REFERENCE_MOMENT_KERNELS)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert mod.KEY_IMPL is None and mod.VALUE_IMPL is None
    return mod


def credit_config3(device, seed=0):
    """BASELINE config 3 inputs: rows = 16 x 8 heads, T = 2048, d = 64; q, k, v ~ N(0,1)/8 (bf16 copies feed the
    bf16 kernels), hub the per-token error signal e[b, t] u_h with e ~ N(0, 1), u_h ~ N(0, 1)/8; raw queries / keys
    N(0, 1); bf16-rounded RoPE tables; the query moments' step sizes 0.01 rms(raw)."""
    g = torch.Generator(device).manual_seed(seed)
    B, H, t = 16, 8, 2048
    rows = B * H
    rn = lambda *shape: torch.randn(*shape, device=device, generator=g)
    q, k, v = (rn(B, H, t, 64).div_(8).view(rows, t, 64) for _ in range(3))
    e = rn(B, 1, t, 1)
    u = rn(1, H, 1, 64) / 8
    hub = (e * u).reshape(rows, t, 64).contiguous()
    raw_q, raw_k = rn(rows, t, 64), rn(rows, t, 64)
    inv = 1.0 / 10000 ** (torch.arange(0, 64, 2, dtype=torch.float32, device=device) / 64)
    freqs = torch.outer(torch.arange(t, dtype=torch.float32, device=device), inv)
    sq = raw_q.square().sum(-1)
    return dict(rows=rows, t=t, q=q, k=k, v=v, hub=hub, raw_q=raw_q, raw_k=raw_k,
                cos=freqs.cos().bfloat16().float(), sin=freqs.sin().bfloat16().float(),
                b16=[z.bfloat16() for z in (q, k, v, hub)], sq=sq, steps=0.01 * (sq / 64).sqrt().clamp(min=1e-6))


def credit_calls(mk, x, window, lse, center):
    """name -> zero-argument call of each credit kernel through module mk's ops (ours, noise_b200.moment_kernels, or
    the reference's: the same signatures), returning its outputs. lse, center: the key context the downstream
    kernels read (the same tensors for both arms in a parity check)."""
    dev, rows, t = x['q'].device, x['rows'], x['t']
    b16 = x['b16']
    qs = torch.empty(1, rows, t, 64, dtype=torch.bfloat16, device=dev)
    ko, kv = torch.empty(1, rows, t, 64, device=dev), torch.empty(1, rows, t, 64, device=dev)

    def query():
        mk.moment_query_scores(*b16, x['raw_q'].unsqueeze(0), x['sq'], x['k'], x['cos'], x['sin'], lse, center,
                               x['steps'], qs, 4, window)
        return qs

    def keys():
        mk.moment_key_scores(*b16, x['raw_k'].unsqueeze(0), x['sq'], x['q'], x['cos'], x['sin'], lse, center,
                             x['steps'], ko, kv, 2)
        return ko, kv

    calls = {
        'implicit_key_context': lambda: mk.implicit_key_context_edges(*b16, window),
        'value_pass': lambda: mk.raw_value_credits(b16[0], b16[1], lse, x['hub'], window),
        'key_scan': lambda: mk.key_credits(x['q'], x['k'], x['raw_k'], lse, x['v'], x['hub'], center, x['cos'],
                                           x['sin'], window, 0.003),
        'moment_query_scores': query,
    }
    if window >= t:  # the identity phase's key moments are full-causal
        calls['moment_key_scores'] = keys
    return calls


def run_credit(a):
    """One line per window: every credit kernel on BASELINE config 3 (credit_config3), CUDA-event timed over K launches
    after W warm-ups; inputs (~0.5 GB) exceed L2. ``--impl reference`` times the reference's Triton kernels
    (reference_moment_kernels) on the same inputs and clocks; without the reference install it prints an
    ``unavailable`` line."""
    device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    torch.cuda.set_device(device)
    if a.impl == 'reference':
        try:
            mk = reference_moment_kernels()
        except Exception as exc:  # noqa: BLE001 - reported, not hidden
            print(json.dumps({'impl': 'reference', 'workload': 'credit', 'unavailable': repr(exc)}), flush=True)
            return
    else:
        import noise_b200.moment_kernels as mk
    x = credit_config3(device)
    rows, t = x['rows'], x['t']
    peaks = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text()) if (ROOT / 'MEASURED_PEAKS.json').exists() else {}
    tf_peak = peaks.get('bf16_tflops', 1590.0)
    for window in (2048, 1024):
        pairs = rows * visible_pairs(t, window)
        lse, center = mk.implicit_key_context_edges(*x['b16'], window)
        calls = credit_calls(mk, x, window, lse, center)
        clocks = Clocks(device)
        res = {}
        for name, fn in calls.items():
            for _ in range(a.warmup):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.steps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / a.steps
            flops = CREDIT_FLOP_PER_PAIR[name] * pairs
            res[name] = {'us': round(us, 1), 'tflops': round(flops / us / 1e6, 1),
                         'frac_of_tensor_peak': round(flops / us / 1e6 / tf_peak, 4),
                         'mufu_floor_us': round(pairs / (16 * 148 * 1.965e9) * 1e6, 1)}
        print(json.dumps({'metric': 'credit-readout kernel time (BASELINE config 3)', 'unit': 'us per launch',
                          'impl': a.impl, 'clocks': clocks.stop(),
                          'config': {'workload': 'credit kernels in isolation', 'B': 16, 'H': 8, 'T': t,
                                     'd_head': 64, 'window': window, 'pairs': pairs},
                          'peak': {'bf16_tflops': tf_peak, 'source': 'MEASURED_PEAKS.json bf16_tflops (burst)'},
                          'kernels': res}), flush=True)


# ------------------------------------------------------------------------------------------------------------------
# one EGGROLL training update at population 24,576 (BASELINE configs 4 / 5)
# ------------------------------------------------------------------------------------------------------------------


def run_train(a):
    """BASELINE config 4, the headline: train tokens/s of EGGROLL updates at population 24,576. Each update consumes
    8 rows x 2048 Zipf tokens (eggroll.py's BATCH), evaluates 24,576 antithetic members (3,072 per row, split evenly
    over the ranks: strong scaling), all-gathers their losses, rebuilds the update on each rank's pair shard
    (tcgen05 GEMM, K = pairs) with one NCCL all-reduce, and applies AdamW.

    One timed loop of K updates serves both numbers: per update, the token rows go host -> device (pinned), the update
    runs, and the mean loss comes back device -> host. ``value`` sums the device time of the updates alone (CUDA
    events after the copy-in and before the copy-out), ``e2e`` the whole loop including the copies and the host's
    wait for the loss. Both are max-reduced over the ranks."""
    from noise_b200 import _lib
    from noise_b200.eggroll import make_params
    from noise_b200.train import EggrollTrainer, phase_ms

    rank, world = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))
    device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    torch.cuda.set_device(device)
    dist = world > 1
    if dist:
        torch.distributed.init_process_group('nccl', device_id=device, timeout=timedelta(seconds=300))
    tr = EggrollTrainer(make_params(device, 0), TRAIN_PAIRS, TRAIN_ROWS, sigma=SIGMA, lr=1e-3, rank=rank,
                        world=world)
    host_rows = [zipf_rows(TRAIN_ROWS, T + 1, seed=100 + s).pin_memory() for s in range(a.warmup + a.steps)]
    loss_host = torch.empty(1, pin_memory=True)
    for i in range(a.warmup):
        loss = tr.step(host_rows[i].to(device, non_blocking=True), step=i + 1)
        loss_host.copy_(loss.view(1), non_blocking=True)
        torch.cuda.current_stream().synchronize()
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()

    clocks = Clocks(device)
    marks, timer, launches = [], [], 0
    ev = lambda: torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
    with _lib.LaunchProfile() as prof:
        for i in range(a.steps):
            e_in, e_go, e_done, e_out = ev(), ev(), ev(), ev()
            e_in.record()
            tokens = host_rows[a.warmup + i].to(device, non_blocking=True)
            e_go.record()
            loss = tr.step(tokens, step=a.warmup + i + 1, timer=timer)
            e_done.record()
            loss_host.copy_(loss.view(1), non_blocking=True)
            e_out.record()
            torch.cuda.current_stream().synchronize()
            launches += tr.launches
            marks.append((e_in, e_go, e_done, e_out))
        torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
    clk = clocks.stop()
    ms = sum(go.elapsed_time(done) for _, go, done, _ in marks)
    ms_e2e = marks[0][0].elapsed_time(marks[-1][3])
    phases = phase_ms(timer)
    if dist:
        names = list(EggrollTrainer.PHASES)
        t = torch.tensor([ms, ms_e2e] + [phases.get(n, 0.0) for n in names], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        vals = t.tolist()
        ms, ms_e2e = vals[:2]
        phases = dict(zip(names, vals[2:]))
    value = TRAIN_TOKENS * a.steps / (ms / 1e3)
    e2e_value = TRAIN_TOKENS * a.steps / (ms_e2e / 1e3)
    per_rank_forwards = TRAIN_FORWARDS // world * a.steps
    line = {
        'metric': METRIC, 'value': value, 'unit': TRAIN_UNIT, 'n_gpus': world, 'steps': a.steps,
        'warmup': a.warmup, 'ms_per_step': ms / a.steps, 'higher_is_better': True, 'scaling': 'strong',
        'vs_baseline': None, 'dtype': 'bf16',
        'data': 'synthetic: Zipf(1.1) token rows over vocab 4096; random-init weights of the utils/model.py GPT '
                '(EGGROLL make_model); EGGROLL 2**28 N(0,1) noise buffer',
        'config': {'workload': 'BASELINE config 4: one EGGROLL update per step at population 24,576 (12,288 '
                               'antithetic pairs, sigma 2e-3), 8 rows x 2048 tokens per update, members split over '
                               'the ranks; fitness all-gather, pair-sharded rebuilt update + NCCL all-reduce, AdamW',
                   'population': 2 * TRAIN_PAIRS, 'members_per_gpu': 2 * TRAIN_PAIRS // world,
                   'rows_per_update': TRAIN_ROWS, 'seq_len': T, 'train_tokens_per_step': TRAIN_TOKENS,
                   'population_forwards_per_s_per_gpu': per_rank_forwards / (ms / 1e3),
                   'member_tokens_per_s': TRAIN_FORWARDS * T * a.steps / (ms / 1e3),
                   'phase_ms_per_step': {k: round(v / a.steps, 3) for k, v in phases.items()},
                   'l2': 'inputs larger than L2 (per-call activations ~11 GB)', 'parallelism': f'members x{world}',
                   'last_mean_loss': float(loss_host[0]), 'attention_order': attention_order()},
        'e2e': {'value': e2e_value, 'unit': TRAIN_UNIT, 'h2d_bytes_per_step': TRAIN_ROWS * (T + 1) * 8,
                'd2h_bytes_per_step': 4, 'ms_per_step': ms_e2e / a.steps,
                'copy_and_host_wait_ms_per_step': (ms_e2e - ms) / a.steps},
        'gpu_launches': launches,
    }
    line.update(kernel_roofline(prof, min(tr.pop.chunk, TRAIN_FORWARDS // world), clk, ms, per_rank_forwards))
    if rank == 0 and world == 1:
        line['cpu_baseline'] = cpu_baseline_train()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


EPOCH_ROWS = 14648  # utils/prepare_data.py's TRAIN_ROWS: rows of 2,049 tokens, one update per 8 rows


def run_epoch(a):
    """BASELINE config 5, bounded: the first --updates updates (default 100) of one epoch over 14,648 synthetic
    Zipf(1.1) rows of 2,049 tokens (seed 0), 8 rows per update (1,831 updates an epoch), population 24,576 split over
    the ranks, EGGROLL with AdamW as in run_train. Prints the timed updates' train tokens/s (max over ranks of the
    CUDA-event time), the host wall time, the projected wall time of the whole epoch (1,831 x the mean update time)
    and the mean loss of the first and last timed updates. The reference's own run (eggroll.py) trains on FineWeb;
    synthetic rows stand in for it here."""
    from noise_b200.eggroll import make_params
    from noise_b200.train import EggrollTrainer

    rank, world = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))
    device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    torch.cuda.set_device(device)
    dist = world > 1
    if dist:
        torch.distributed.init_process_group('nccl', device_id=device, timeout=timedelta(seconds=300))
    rows = zipf_rows(EPOCH_ROWS, T + 1, seed=0)
    n_updates = EPOCH_ROWS // TRAIN_ROWS
    updates = min(a.updates, n_updates - a.warmup)
    tr = EggrollTrainer(make_params(device, 0), TRAIN_PAIRS, TRAIN_ROWS, sigma=SIGMA, lr=1e-3, rank=rank,
                        world=world)
    batch = lambda u: rows[u * TRAIN_ROWS:(u + 1) * TRAIN_ROWS].pin_memory().to(device, non_blocking=True)
    for u in range(a.warmup):
        tr.step(batch(u), step=u + 1)
    torch.cuda.synchronize()
    if dist:
        torch.distributed.barrier()
    losses = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for u in range(a.warmup, a.warmup + updates):
        losses.append(tr.step(batch(u), step=u + 1))
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms, wall * 1e3], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, wall = t[0].item(), t[1].item() / 1e3
    per_update = ms / 1e3 / updates
    if rank == 0:
        loss = torch.stack(losses).float().cpu()
        print(json.dumps({
            'metric': 'one-epoch-equivalent training (BASELINE config 5), bounded to the first updates',
            'value': TRAIN_TOKENS * updates / (ms / 1e3), 'unit': TRAIN_UNIT, 'n_gpus': world,
            'updates_timed': updates, 'warmup': a.warmup, 'ms_per_update': per_update * 1e3,
            'host_wall_s': wall, 'epoch_updates': n_updates, 'epoch_train_tokens': n_updates * TRAIN_TOKENS,
            'projected_epoch_wall_s': per_update * n_updates,
            'mean_loss_first': float(loss[:5].mean()), 'mean_loss_last': float(loss[-5:].mean()),
            'scaling': 'strong', 'dtype': 'bf16',
            'data': 'synthetic: 14,648 Zipf(1.1) rows of 2,049 tokens (seed 0), 8 rows per update',
            'config': {'workload': 'BASELINE config 5 (EGGROLL updates at population 24,576, one row feeds one '
                                   'update)', 'population': 2 * TRAIN_PAIRS, 'parallelism': f'members x{world}'}}),
              flush=True)
    if dist:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def _timed(fn, steps, warmup):
    """Microseconds per call of fn, CUDA events on the current stream after warm-up calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / steps


def run_aux(a):
    """The path's other entry points at representative shapes, one JSON line: per op the time per call and its
    algorithmic rate (TFLOP/s for contractions, GB/s of compulsory bytes for data movement)."""
    from noise_b200 import gpt_loss, head_loss, heads, readout, scorer
    from noise_b200.eggroll import make_params
    device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    torch.cuda.set_device(device)
    g = torch.Generator(device).manual_seed(0)
    rn = lambda *s, scale=1.0: torch.randn(*s, device=device, generator=g) * scale
    ru = lambda *s, scale=1.0: torch.rand(*s, device=device, generator=g) * scale
    res = {}

    def rate(name, us, flops=None, nbytes=None, **extra):
        r = {'us': round(us, 1)}
        if flops:
            r['tflops'] = round(flops / us / 1e6, 2)
        if nbytes:
            r['gbs'] = round(nbytes / us / 1e3, 1)
        r.update(extra)
        res[name] = r

    # GPT.forward (config 1 shape: 4 rows x 2048 tokens, un-perturbed) and the fused LM-head loss (16,384 rows)
    params = make_params(device, 0)
    tok = zipf_rows(4, T + 1, seed=5).to(device)
    us = _timed(lambda: gpt_loss(None, params, tok[:, :-1], tok[:, 1:], 'sum'), a.steps, a.warmup)
    rate('gpt_loss', us, flops=4 * T * FLOP_PER_MEMBER_TOKEN, tokens_per_s=round(4 * T / us * 1e6))
    x = rn(16384, 512)
    tg = torch.randint(0, 4096, (16384,), device=device, generator=g)
    us = _timed(lambda: head_loss(x, params['lm_head.weight'], tg, 4096), a.steps, a.warmup)
    rate('head_loss', us, flops=2 * 16384 * 4096 * 512)
    # identity-phase head sharding: 8 layers, 8,192 local tokens (8 rows of 1,024); 8 source ranks x 1,024 tokens
    n, t = 8192, 1024
    pieces = [[rn(n, 512).bfloat16() for _ in range(8)] for _ in range(5)]
    lses = [rn(n // t, 8, t) for _ in range(8)]
    us = _timed(lambda: heads.pack_heads_kernel(*pieces, lses), a.steps, a.warmup)
    rate('pack_heads', us, nbytes=8 * 8 * n * (5 * 128 + 4 + 644))
    got = rn(8, 8, 1024, 322).bfloat16()
    got.view(torch.int16)[..., 320:] = rn(8, 8, 1024).add_(3).unsqueeze(-1).view(torch.int16).view(8, 8, 1024, 2)
    ang = torch.outer(torch.arange(t, device=device, dtype=torch.float32),
                      1.0 / 10000 ** (torch.arange(0, 64, 2, device=device, dtype=torch.float32) / 64))
    cs, sn = ang.cos(), ang.sin()
    us = _timed(lambda: heads.head_prep_fused(got, cs, sn, 8, t), a.steps, a.warmup)
    rate('head_prep', us, nbytes=65536 * (644 + 4 * 128 + 256 + 128 + 256 + 64 + 24))
    back = torch.empty(8, 8, 3, 1024, 64, dtype=torch.bfloat16, device=device)
    us = _timed(lambda: heads.id_head_scores(got, (cs, sn), back, 8, t), a.steps, a.warmup)
    rate('id_head_scores', us, rows=64, tokens=t)
    # identity-phase GEMMs on the same 8,192 local tokens, 8 layers, D 512, hidden 2048
    from noise_b200 import id_kernels
    m = n
    fc = [rn(m, 2048).bfloat16() for _ in range(8)]
    credb = rn(8, m, 512, scale=0.1).bfloat16()
    w_out_t = rn(8, 512, 2048, scale=0.05).bfloat16()
    fc_steps = ru(8, m, scale=0.5).add_(0.01)
    us = _timed(lambda: id_kernels.hidden_credits_fused(fc, fc_steps, credb, w_out_t), a.steps, a.warmup)
    rate('hidden_credits', us, flops=2 * 8 * m * 512 * 2048)
    n2s = [rn(m, 512).bfloat16() for _ in range(8)]
    hid = [rn(m, 2048, scale=0.1).bfloat16() for _ in range(8)]
    gwide = torch.empty(16, 512, 2048, dtype=torch.bfloat16, device=device)
    us = _timed(lambda: id_kernels.at_b_layers(n2s, hid, gwide[:8]), a.steps, a.warmup)
    rate('at_b_layers_wide', us, flops=2 * 8 * m * 512 * 2048)
    gsq = torch.empty(32, 512, 512, dtype=torch.bfloat16, device=device)
    us = _timed(lambda: id_kernels.at_b_layers(n2s, list(credb), gsq[24:]), a.steps, a.warmup)
    rate('at_b_layers_square', us, flops=2 * 8 * m * 512 * 512)
    got2 = rn(8, 8, 3, m, 64, scale=0.2).bfloat16()
    us = _timed(lambda: id_kernels.square_credit_grads(n2s, got2, gsq[:24]), a.steps, a.warmup)
    rate('square_credit_grads', us, flops=2 * 24 * m * 512 * 512)
    # track-1 readout scorers
    H, Tq, P, M, start, window = 8, 2048, 16, 256, 512, 1024
    q, tgt = rn(H, Tq, 64), rn(H, Tq, 64, scale=0.125)
    dk, dv = rn(H, P, M, 64, scale=0.05), rn(H, P, M, 64, scale=0.05)
    A, C = ru(H, Tq, M, scale=0.1), rn(H, Tq, M)
    pairs = H * P * M * window
    us = _timed(lambda: readout.future_scores(q, tgt, dk, dv, A, C, start, window), a.steps, a.warmup)
    rate('future_scores', us, flops=pairs * 4 * 64)
    us = _timed(lambda: readout.key_response(q, dk, A, C, start, start, window), a.steps, a.warmup)
    rate('key_response', us, flops=pairs * 2 * 64)
    mq, pq = 256, 64
    dq, keys, vals = rn(mq, pq, H, 64, scale=0.3), rn(H, Tq, 64), rn(H, Tq, 64)
    pos = torch.arange(mq, device=device) * (Tq // mq) + Tq // mq - 1
    lag = pos[:, None] - torch.arange(Tq, device=device)[None]
    prob = (ru(H, mq, Tq) * ((lag >= 0) & (lag <= window))).contiguous()
    base = rn(H, mq, 64)
    visible = int(((lag >= 0) & (lag <= window)).sum())
    us = _timed(lambda: readout.query_response(dq, keys, vals, prob, base), a.steps, a.warmup)
    rate('query_response', us, flops=H * pq * visible * 4 * 64)
    mr, pr, kr = 2048, 64, 128
    rdq, rk, rv = (rn(mr, pr, H, 64, scale=0.3).bfloat16(), rn(mr, H, kr, 64).bfloat16(), rn(mr, H, kr, 64).bfloat16())
    rp, rest = ru(mr, H, kr, scale=1.0 / kr), rn(mr, H, 64, scale=0.1)
    us = _timed(lambda: readout.routed_response(rdq, rk, rv, rp, rest), a.steps, a.warmup)
    rate('routed_response', us, flops=mr * H * pr * kr * 4 * 64)
    # the true-path readout's scorer: a chunk of 128 tokens x 256 moved rows, tables of a 2,048-token sequence
    Ts, ms, ns = 2048, 128, 256
    up, st = rn(ms * ns, 1040, scale=0.05).bfloat16(), torch.stack([ru(ms, ns) + 0.5, rn(ms, ns, scale=0.01)], -1)
    r0, vc, gz, ve = rn(Ts, 8, 64), rn(Ts, 512), rn(Ts, 8), rn(Ts, 8, 64, scale=0.1)
    tabs = [rn(Ts, 8, 64, scale=0.1), rn(Ts, 8, 64, scale=0.1), rn(Ts, 8, 64, 64, scale=0.05).bfloat16(),
            rn(Ts, 8, 64, 64, scale=0.05).bfloat16(), rn(Ts, 8, 64), rn(Ts, 8, 64, scale=0.1), ru(Ts, 8, scale=0.2),
            rn(Ts, 8), rn(Ts, 8, 64), rn(Ts, 8, 64)]
    rcs, rsn = torch.ones(Ts, 32, device=device), torch.zeros(Ts, 32, device=device)
    out = torch.empty(ms, ns, device=device)
    se = torch.empty(ms, ns, 512, dtype=torch.bfloat16, device=device)
    us = _timed(lambda: scorer.staged_kernel(up, st, r0, vc, gz, ve, rcs, rsn, *tabs, out, se, 0, ns, ns, True, True,
                                             True, 1040), a.steps, a.warmup)
    rate('readout_staged', us, flops=ms * ns * 8 * 2 * 2 * 64 * 64)
    # the identity phase's readout cycle: 4,096 tokens (its 7 GEMMs of 4,096 x 4,096 x 512, fp32 ones at the caller's
    # matmul precision)
    import types
    from noise_b200 import cycle
    nc_ = 4096
    hmat = torch.ones(1, 1, device=device)
    while hmat.shape[0] < 512:
        hmat = torch.cat([torch.cat([hmat, hmat], 1), torch.cat([hmat, -hmat], 1)], 0)
    model = types.SimpleNamespace(H=hmat, step_t=torch.tensor(3, device=device), lm_head=rn(512, 4096, scale=0.05))
    xc, yc = rn(nc_, 512), torch.randint(0, 4096, (nc_,), device=device, generator=g)
    us = _timed(lambda: cycle.top_credit(model, xc, yc), a.steps, a.warmup)
    rate('top_credit', us, flops=nc_ * (7 * 2 * 4096 * 512 + 2 * 512 * 512), tokens=nc_,
         fp32_contractions='tf32 tcgen05 GEMM (the reference\'s high precision)')
    raw = rn(nc_, 4096, scale=3)
    us = _timed(lambda: cycle.coordinate_change(raw, yc), a.steps, a.warmup)
    rate('coordinate_change', us, nbytes=nc_ * 4096 * 8)
    print(json.dumps({'metric': 'auxiliary entry points of the path: time per call', 'unit': 'us per call',
                      'steps': a.steps, 'warmup': a.warmup,
                      'config': {'workload': 'representative shapes (bench.py run_aux)'}, 'kernels': res}), flush=True)


def run_exchange(a):
    """The identity phase's two exchanges at 8 layers x 8,192 local tokens per rank (rows of 1,024): the reference's
    way (pack_heads_kernel, then NCCL all_to_all_single for heads in and for heads out) against HeadExchange (the pack
    writing straight into the owners' buffers, the heads-out stores, the epoch-flag waits). One step = both
    exchanges; CUDA events over K steps after W warm-ups, max over ranks. One JSON line (rank 0)."""
    from noise_b200 import heads
    device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    torch.cuda.set_device(device)
    world = int(os.environ.get('WORLD_SIZE', 1))
    dist = torch.distributed
    if world > 1:
        dist.init_process_group('nccl', device_id=device, timeout=timedelta(seconds=120))
    rank = dist.get_rank() if world > 1 else 0
    layers, n, t = 8, 8192, 1024
    g = torch.Generator(device).manual_seed(rank)
    pieces = [[torch.randn(n, 512, device=device, generator=g).bfloat16() for _ in range(layers)] for _ in range(5)]
    lses = [torch.randn(n // t, 8, t, device=device, generator=g) for _ in range(layers)]
    back = torch.randn(world, layers, 3, n, 64, device=device, generator=g).bfloat16()
    ex = heads.HeadExchange(layers, n, t)

    def reference_step():
        send = heads.pack_heads_kernel(*pieces, lses)
        got, got2 = torch.empty_like(send), torch.empty_like(back)
        if world > 1:
            dist.all_to_all_single(got, send)
            dist.all_to_all_single(got2, back)
        else:
            got.copy_(send)
            got2.copy_(back)

    def fused_step():
        ex.send_heads(*pieces, lses)
        ex.wait_heads()
        ex.send_back(back)
        ex.wait_back()

    def timed(fn):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        us = torch.tensor([e0.elapsed_time(e1) * 1e3 / a.steps], device=device)
        if world > 1:
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
        return us.item()

    ref_us = timed(reference_step)
    ours_us = timed(fused_step)
    status = ex.read_status()
    ex.close()
    moved = 8 * layers * n * heads.PACK * 2 + back.numel() * 2  # bytes a rank sends per step (own share included)
    remote = moved * (world - 1) / world
    if rank == 0:
        print(json.dumps({'metric': 'identity-phase head exchange time per step (pack + heads in + heads out)',
                          'unit': 'us per step', 'n_gpus': world, 'steps': a.steps, 'warmup': a.warmup,
                          'config': {'workload': 'head exchange', 'layers': layers, 'tokens_per_rank': n,
                                     'seq_len': t, 'bytes_sent_per_rank': moved},
                          'fused_us': round(ours_us, 1), 'reference_us': round(ref_us, 1),
                          'speedup': round(ref_us / ours_us, 3),
                          'nvlink_gbs_per_rank_fused': round(remote / ours_us / 1e3, 1) if world > 1 else None,
                          'status': status}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    a = args_()
    if a.workload == 'credit':
        run_credit(a)
    elif a.impl == 'reference':
        run_reference(a)
    elif a.workload == 'train':
        run_train(a)
    elif a.workload == 'aux':
        run_aux(a)
    elif a.workload == 'exchange':
        run_exchange(a)
    elif a.workload == 'epoch':
        run_epoch(a)
    else:
        run_ours(a)


if __name__ == '__main__':
    main()
