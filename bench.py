#!/usr/bin/env python
"""Batch-1 greedy decode throughput of the Qwen3-1.7B-shape int8 model on B200 (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

A step is one decode token: one replay of the CUDA graph that holds the native decode step (one cooperative kernel
per token, the dataflow step). Workload = BASELINE config 2: random-init weights (seed 0), int8 per-row weights
with bf16 scales, a 32-token uniform prompt, then 256 greedy tokens (contexts 33..288). Before the timed region the
whole 256-token window runs once (every KV row of the window written); the K timed steps are then spread evenly
over the window's positions (K >= 256: whole windows in order; K < 256: position 32 + floor(256 i / K) for step i,
set on the device before the replay when it does not follow from the previous step), so any K measures the
config's context mix. The 1.72 GB of weights streamed per token are far larger than L2 (126 MB), so no flush is
needed between steps.

Printed JSON line (rank 0):
  value        decode tok/s over all ranks, device-timed (CUDA events around the K replays, max over ranks)
  e2e          the same metric through GraphGreedyDecoder.generate with a pinned host prompt: H2D prompt copy,
               per-token D2H token reads, (n - 1) / (total - ttft) as research/realmodel/bench_int8.py
  roofline     the step kernel (dataflow_step_kernel unless --step says otherwise), one launch per token: achieved = algorithmic bytes per token (weights, scales,
               norms, embedding row, KV at each timed step's context) / (device time / K) against the measured
               HBM copy bandwidth; traffic = its ncu dram bytes per launch (profiles/step_kernel_traffic.json)
  cpu_baseline the reference's CPU path (oracle/torch_ref.py) on this host's cores, bounded sample
With N > 1 (torchrun, one rank per GPU) the same workload runs as N independent replicas (scaling "weak": the value
is the tokens of all ranks per second), so every N measures the same thing; the line adds `tensor_parallel`, BASELINE
config 5 (Qwen3-8B shape, 4096-token prompt, 256 tokens) sharded over the N GPUs (efficientgpt_b200.tp: one
persistent kernel per GPU and token, o_proj / down_proj partial sums exchanged over NVLink inside it).

--impl reference times the reference's CPU decode path (oracle/torch_ref.py: the seeded model built, quantised
and prefilled on the CPU, no GPU and no library of this package) for the same K steps on rank 0.

Other workloads: --workload qwen3_8b (config 5 at any N), nanogpt (config 1), gemm_prefill (the prefill GEMMs on
tcgen05 against the reference's dequantise + cuBLAS arithmetic), ragged (B = 1, 4, 16 sequences decoded together), gemv_sweep / attn_sweep (configs 3
and 4, one JSON line per case), profile_step (a small engine for ncu captures: --layers, --steps).
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
METRIC = 'batch-1 decode tok/s and % of HBM roofline, Qwen3-1.7B-shape int8, 1 B200'
PROMPT_LEN, NEW_TOKENS = 32, 256
FALLBACK_PEAKS = {'hbm_gbs': 6650.0}
STEP_KERNELS = {'dataflow': 'dataflow_step_kernel', 'persistent': 'decode_step_kernel',
                'sequence': 'gemv_tc_kernel (step)'}
TRAFFIC_FILE = ROOT / 'profiles' / 'step_kernel_traffic.json'
L2_BYTES = 126 * 2 ** 20
REF_MAX_STEPS = 512  # the reference arm's CPU steps are ~0.3 s each: bound the run to a few minutes


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=256)
    ap.add_argument('--warmup', type=int, default=8)
    ap.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-tp', action='store_true', help='N > 1: skip the config-5 tensor-parallel measurement')
    ap.add_argument('--step', choices=('dataflow', 'persistent', 'sequence'), default=None,
                    help='decode step of configs 2 and profile_step (default: the engine\'s choice, dataflow)')
    ap.add_argument('--cpu-sample', type=int, default=16, help='timed CPU decode tokens of cpu_baseline')
    ap.add_argument('--workload', default='qwen3_1.7b',
                    choices=['qwen3_1.7b', 'qwen3_8b', 'nanogpt', 'gemv_sweep', 'attn_sweep', 'gemm_prefill',
                             'ragged', 'profile_step'])
    ap.add_argument('--layers', type=int, default=4, help='profile_step: decoder layers')
    ap.add_argument('--reps', type=int, default=50, help='gemv_sweep / attn_sweep: launches per graph')
    ap.add_argument('--only', default='', help='gemv_sweep / attn_sweep: cases whose name contains this text')
    a = ap.parse_args(argv)
    if a.warmup < 3:
        ap.error('--warmup must be >= 3')
    if a.steps < 1:
        ap.error('--steps must be >= 1')
    return a


def dist_setup():
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=torch.device('cuda', local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device='cuda')
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measured_peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return d, 'measured'
    return FALLBACK_PEAKS, 'fallback'


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms while the timed region runs."""
    Q = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
         'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
         'clocks_event_reasons.sw_power_cap')

    def __init__(self):
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.Q}', '--format=csv,noheader,nounits',
                                          '-lms', '100'], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self, gpu_index):
        if self.proc is None:
            return None
        time.sleep(0.05)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in out.splitlines():
            f = [x.strip() for x in line.split(',')]
            if len(f) < 9 or f[0] != str(gpu_index):
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == 'active':
                    reasons.add(n)
        if not sm:
            return None
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': smax, 'reasons': sorted(reasons), 'samples': len(sm)}


def traffic_per_launch(kernel):
    """ncu dram bytes (read + write) per launch of `kernel` at config 2, from the machine-readable capture record
    (profiles/step_kernel_traffic.json: {kernel: {"traffic_bytes_per_launch": ..., ...}}); None when absent."""
    if not TRAFFIC_FILE.exists():
        return None
    rec = json.loads(TRAFFIC_FILE.read_text()).get(kernel) or {}
    return rec.get('traffic_bytes_per_launch')


def window_positions(k, start=PROMPT_LEN, window=NEW_TOKENS):
    """Decode positions of the K timed steps: whole windows in order when K >= window, else spread evenly."""
    if k >= window:
        return [start + (i % window) for i in range(k)]
    return [start + (i * window) // k for i in range(k)]


def time_replays(graph, k, positions=None, set_pos=None):
    """Device time (ms) of k replays; `positions` (length k) puts the step at that position first whenever it does
    not follow from the previous replay (set_pos runs on the same stream, inside the timed region)."""
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for i in range(k):
        if positions is not None and (i == 0 or positions[i] != positions[i - 1] + 1):
            set_pos(positions[i])
        graph.replay()
    e1.record(st)
    e1.synchronize()
    return e0.elapsed_time(e1)


# --------------------------------------------------------------------------------------------- reference arm
def run_reference(a, rank):
    """The reference's CPU decode path (oracle/torch_ref.py) on this host's cores, rank 0 only: the seeded model
    built and quantised on the CPU, the prompt prefilled on the CPU (the op's > 16-row branch), W untimed and K timed
    decode tokens (at most REF_MAX_STEPS). Neither the product package nor its library is loaded."""
    if rank != 0:
        return
    from oracle.torch_ref import TorchCpuQwen3, cpu_model_weights, qwen3_config
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    big = a.workload == 'qwen3_8b'
    prompt_len = 4096 if big else PROMPT_LEN
    steps = min(a.steps, REF_MAX_STEPS)
    t_build = time.perf_counter()
    w = cpu_model_weights(qwen3_config('qwen3_8b' if big else 'qwen3_1.7b'), seed=0,
                          cap=prompt_len + NEW_TOKENS + a.warmup + steps)
    cpu = TorchCpuQwen3(w, prompt_len + NEW_TOKENS + a.warmup + steps)
    prompt = torch.randint(0, 151936, (prompt_len,), generator=torch.Generator().manual_seed(0)).tolist()
    tok = cpu.prefill(prompt)
    build_s = time.perf_counter() - t_build
    pos = prompt_len
    for _ in range(a.warmup):
        tok = cpu.step(tok, pos)
        pos += 1
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = cpu.step(tok, pos)
        pos += 1
    dt = time.perf_counter() - t0
    v = steps / dt
    sample = (f'{steps} decode tokens after {a.warmup} untimed ones, contexts {prompt_len + a.warmup + 2}..'
              f'{prompt_len + a.warmup + steps + 1}; seeded model built, quantised and prefilled on the CPU '
              f'({build_s:.0f} s, untimed); torch CPU ops, bf16((x.float() @ q.float().T) * s) per linear')
    cb = {'value': v, 'unit': 'tok/s', 'cores': threads, 'kind': 'port', 'sample': sample}
    metric = METRIC if not big else METRIC.replace('Qwen3-1.7B', 'Qwen3-8B').replace('1 B200', f'{a.gpus} B200')
    line = {'impl': 'reference', 'metric': metric, 'value': v, 'unit': 'tok/s', 'n_gpus': a.gpus, 'steps': steps,
            'warmup': a.warmup, 'ms_per_step': 1e3 / v, 'higher_is_better': True,
            'scaling': 'strong' if big else 'weak', 'vs_baseline': None, 'dtype': 'int8-weight/bf16',
            'data': 'synthetic',
            'config': {'workload': ('qwen3_8b int8 decode, BASELINE config 5' if big else
                                    'qwen3_1.7b int8 decode, BASELINE config 2') + ' (CPU port of the reference path)',
                       'prompt': prompt_len, 'new_tokens': NEW_TOKENS, 'scale_dtype': 'bf16',
                       'init': 'HF random init N(0,0.02) on the CPU, seed 0'},
            'cpu_baseline': cb, 'e2e': {'value': v, 'unit': 'tok/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------- config 2
def build(device, pdl=True, step=None):
    from efficientgpt_b200.configs import qwen3_1p7b_config, random_model
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    from efficientgpt_b200.int8_linear import quantize_model
    model = random_model(qwen3_1p7b_config(), device, seed=0)
    quantize_model(model, scale_dtype=torch.bfloat16)
    torch.cuda.empty_cache()
    dec = GraphGreedyDecoder(model, max_cache_len=PROMPT_LEN + NEW_TOKENS, pdl=pdl, step=step)
    prompt = torch.randint(0, model.config.vocab_size, (1, PROMPT_LEN), generator=torch.Generator().manual_seed(0))
    return model, dec, prompt


def cpu_baseline(dec, n_tokens):
    """The reference's CPU decode path (oracle/torch_ref.py) on this host with the timed engine's weights: the
    prompt prefilled on the CPU, 1 warm-up + n_tokens timed decode steps right after it."""
    from oracle.torch_ref import TorchCpuQwen3
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cpu = TorchCpuQwen3.from_engine(dec.engine, PROMPT_LEN + n_tokens + 2)
    prompt = torch.randint(0, dec.engine.vocab, (PROMPT_LEN,), generator=torch.Generator().manual_seed(0)).tolist()
    tok = cpu.prefill(prompt)
    tok = cpu.step(tok, PROMPT_LEN)
    t0 = time.perf_counter()
    for i in range(n_tokens):
        tok = cpu.step(tok, PROMPT_LEN + 1 + i)
    dt = time.perf_counter() - t0
    return {'value': n_tokens / dt, 'unit': 'tok/s', 'cores': threads, 'kind': 'port',
            'sample': f'{n_tokens} decode tokens (after 1 warm-up token) of the same Qwen3-1.7B-shape int8 model at '
                      f'context {PROMPT_LEN + 2}..{PROMPT_LEN + 1 + n_tokens}, torch CPU ops, '
                      f'bf16((x.float() @ q.float().T) * s) per linear'}


def run_config2(a, world, rank, local):
    """Config 2 on every rank (N independent replicas at N > 1); returns rank 0's line (None elsewhere)."""
    model, dec, prompt = build('cuda', step=a.step)
    eng = dec.engine
    dec._capture()
    eng.prefill(prompt.cuda())

    def set_pos(p):
        eng.position.fill_(p)

    # warm-up, then one whole window (every KV row of contexts 33..288 written), then the timed region
    time_replays(dec.graph, a.warmup, window_positions(a.warmup), set_pos)
    set_pos(PROMPT_LEN)
    time_replays(dec.graph, NEW_TOKENS)
    positions = window_positions(a.steps)
    barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    ms = time_replays(dec.graph, a.steps, positions, set_pos)
    clocks = sampler.stop(local) if rank == 0 else None
    ms = max_over_ranks(ms, world)
    barrier(world)
    from efficientgpt_b200._lib import device_error
    err = device_error()
    tok_s = a.steps / (ms / 1e3) * world

    # algorithmic bytes per token over the timed steps (context = position + 1 keys)
    kv_mean = statistics.fmean(eng.kv_bytes_per_token(p + 1) for p in positions)
    bytes_tok = eng.weight_bytes() + kv_mean
    peaks, peak_src = measured_peaks()
    hbm = float(peaks['hbm_gbs'])
    gbs = bytes_tok / (ms / 1e3 / a.steps) / 1e9
    launches_per_step = 1 if eng.persistent else 5 * eng.n_layers + 1
    kernel = STEP_KERNELS[eng.step_kind]
    roofline = {'bound': 'hbm', 'kernel': kernel,
                'achieved': round(gbs, 1), 'peak': hbm, 'unit': 'GB/s', 'frac': round(gbs / hbm, 4),
                'traffic': traffic_per_launch(kernel) if eng.persistent else None, 'launches_per_step': launches_per_step,
                'bytes_per_launch': round(bytes_tok / launches_per_step),
                'avg_launch_us': round(ms * 1e3 / a.steps / launches_per_step, 3), 'peak_source': peak_src,
                'mean_context': round(statistics.fmean(p + 1 for p in positions), 1)}

    e2e = None
    if not a.no_e2e:
        host_prompt = prompt.pin_memory()
        vals = []
        for _ in range(3):
            out, st = dec.generate(host_prompt, NEW_TOKENS)
            vals.append((st['tokens'] - 1) / (st['total_s'] - st['ttft_s']))
        e2e_v = max_over_ranks(-statistics.median(vals), world)  # the slowest rank's rate, times the ranks
        e2e = {'value': -e2e_v * world, 'unit': 'tok/s', 'h2d_bytes_per_step': PROMPT_LEN * 8 / NEW_TOKENS,
               'd2h_bytes_per_step': 8, 'ttft_ms': round(st['ttft_s'] * 1e3, 3),
               'api': 'efficientgpt_b200.GraphGreedyDecoder.generate (pinned host prompt, 256 new tokens)'}

    cb = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cb = cpu_baseline(dec, a.cpu_sample)
    line = None
    if rank == 0:
        line = {
            'metric': METRIC if world == 1 else METRIC.replace('1 B200', f'{world} B200 (independent replicas)'),
            'value': round(tok_s, 2), 'unit': 'tok/s', 'n_gpus': world, 'steps': a.steps,
            'warmup': a.warmup, 'ms_per_step': round(ms / a.steps, 5), 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'int8-weight/bf16', 'data': 'synthetic',
            'config': {'workload': 'qwen3_1.7b int8 decode, BASELINE config 2', 'prompt': PROMPT_LEN,
                       'new_tokens': NEW_TOKENS, 'scale_dtype': 'bf16', 'init': 'HF random init N(0,0.02), seed 0',
                       'parallelism': f'replicas{world}' if world > 1 else 'single',
                       'timed_positions': 'whole windows' if a.steps >= NEW_TOKENS else
                       f'{a.steps} positions spread over {PROMPT_LEN}..{PROMPT_LEN + NEW_TOKENS - 1}',
                       'l2': 'no flush: 1.72 GB of weights streamed per step, larger than L2',
                       'step': eng.step_kind},
            'tok_s_per_gpu': round(tok_s / world, 2),
            'roofline': roofline,
            'device_error': err,
            'e2e': e2e,
            'cpu_baseline': cb,
            'gpu_launches': a.steps * launches_per_step,
            'clocks': clocks,
        }
    del dec, model
    torch.cuda.empty_cache()
    return line


# --------------------------------------------------------------------------------------------- config 5 / TP
def run_tp(a, world, rank, local, workload='qwen3_8b'):
    """Tensor-parallel decode over the `world` GPUs (world 1: the same engine on one GPU): K timed replays of a
    graph holding one step, device time max over ranks; every rank builds the same seeded model and keeps its
    shard. Returns rank 0's line (None elsewhere)."""
    from efficientgpt_b200 import tp
    from efficientgpt_b200.configs import qwen3_1p7b_config, qwen3_8b_config, random_model
    from efficientgpt_b200.int8_linear import quantize_model
    big = workload == 'qwen3_8b'
    prompt_len = 4096 if big else PROMPT_LEN
    cfg = qwen3_8b_config() if big else qwen3_1p7b_config()
    dev = torch.device('cuda', local)
    model = random_model(cfg, dev, seed=0)
    quantize_model(model, scale_dtype=torch.bfloat16)
    shape = tp.Qwen3Shape.from_config(model.config)
    full = tp.full_weights(model)
    weights = tp.shard(full, shape, rank, world) if world > 1 else full
    if world > 1:
        del full, model
    torch.cuda.empty_cache()
    eng = tp.TPQwen3Engine(shape, weights, rank, world, prompt_len + NEW_TOKENS)
    prompt = torch.randint(0, shape.vocab, (1, prompt_len), generator=torch.Generator().manual_seed(0))
    eng.feed(prompt.to(dev))
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        eng.step()
        eng.step()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        eng.step()

    def set_pos(p):
        eng.position.fill_(p)

    set_pos(prompt_len)
    barrier(world)
    time_replays(graph, a.warmup, window_positions(a.warmup, prompt_len), set_pos)
    set_pos(prompt_len)
    barrier(world)
    time_replays(graph, NEW_TOKENS)
    positions = window_positions(a.steps, prompt_len)
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    torch.cuda.synchronize(dev)
    barrier(world)  # after the sampler's start-up: the ranks' kernels wait on one another with a bounded wait
    ms = time_replays(graph, a.steps, positions, set_pos)
    clocks = sampler.stop(local) if rank == 0 else None
    ms = max_over_ranks(ms, world)
    barrier(world)
    from efficientgpt_b200._lib import device_error
    err = device_error()
    tok_s = a.steps / (ms / 1e3)  # one token per step for the whole job (all ranks decode the same token)

    bytes_rank = eng.weight_bytes() + statistics.fmean(eng.kv_bytes_per_token(p + 1) for p in positions)
    peaks, peak_src = measured_peaks()
    hbm = float(peaks['hbm_gbs'])
    gbs = bytes_rank / (ms / 1e3 / a.steps) / 1e9
    nvlink = 2 * shape.n_layers * shape.hidden * 16 * (world - 1) + 16 * (world - 1) if world > 1 else 0

    # end to end through the engine's public API: pinned host prompt in, every token read back to the host
    e2e = None
    if not a.no_e2e:
        host_prompt = prompt.pin_memory()
        torch.cuda.synchronize(dev)
        barrier(world)
        t0 = time.perf_counter()
        eng.feed(host_prompt.to(dev, non_blocking=True))
        host_tok = torch.empty(NEW_TOKENS, dtype=torch.int64).pin_memory()
        host_tok[0:1].copy_(eng.token, non_blocking=True)
        torch.cuda.synchronize(dev)
        t1 = time.perf_counter()
        for i in range(1, NEW_TOKENS):
            graph.replay()
            host_tok[i:i + 1].copy_(eng.token, non_blocking=True)
        torch.cuda.synchronize(dev)
        t2 = time.perf_counter()
        dt = max_over_ranks(t2 - t1, world)
        e2e = {'value': (NEW_TOKENS - 1) / dt, 'unit': 'tok/s', 'h2d_bytes_per_step': prompt_len * 8 / NEW_TOKENS,
               'd2h_bytes_per_step': 8, 'ttft_ms': round((t1 - t0) * 1e3, 3),
               'api': 'efficientgpt_b200.tp.TPQwen3Engine.feed (pinned host prompt), then one graph replay and one '
                      'token read per step'}
    line = None
    if rank == 0:
        wl = ('qwen3_8b int8 decode, BASELINE config 5' if big else 'qwen3_1.7b int8 decode, BASELINE config 2')
        line = {
            'metric': METRIC if not big else METRIC.replace('Qwen3-1.7B', 'Qwen3-8B').replace('1 B200', f'{world} B200'),
            'value': round(tok_s, 2), 'unit': 'tok/s', 'n_gpus': world, 'steps': a.steps, 'warmup': a.warmup,
            'ms_per_step': round(ms / a.steps, 5), 'higher_is_better': True, 'scaling': 'strong',
            'vs_baseline': None, 'dtype': 'int8-weight/bf16', 'data': 'synthetic',
            'config': {'workload': wl, 'prompt': prompt_len, 'new_tokens': NEW_TOKENS, 'scale_dtype': 'bf16',
                       'init': 'HF random init N(0,0.02) on the GPU, seed 0',
                       'parallelism': f'tp{world}' if world > 1 else 'single',
                       'l2': f'no flush: {bytes_rank / 1e9:.2f} GB streamed per step per GPU, larger than L2',
                       'step': eng.step_kind},
            'roofline': {'bound': 'hbm', 'kernel': STEP_KERNELS[eng.step_kind],
                         'achieved': round(gbs, 1), 'peak': hbm, 'unit': 'GB/s', 'frac': round(gbs / hbm, 4),
                         'traffic': None, 'launches_per_step': 1 if eng.persistent else 5 * shape.n_layers + 1,
                         'bytes_per_launch': round(bytes_rank), 'avg_launch_us': round(ms * 1e3 / a.steps, 3),
                         'peak_source': peak_src, 'per': 'GPU (each rank streams its shard)'},
            'nvlink_bytes_per_token_per_gpu': nvlink,
            'device_error': err,
            'e2e': e2e,
            'cpu_baseline': None,
            'gpu_launches': a.steps * (1 if eng.persistent else 5 * shape.n_layers + 1),
            'clocks': clocks,
        }
    del graph
    eng.close()
    torch.cuda.empty_cache()
    return line


# --------------------------------------------------------------------------------------------- config 1
def run_nanogpt(a, rank):
    """the nanoGPT decode step (one CUDA graph per token) over the contexts 65..128 window, and
    the oracle's numpy restatement of the reference CPU path for a bounded sample. Rank 0 only."""
    if rank != 0:
        return
    from efficientgpt_b200.int8_linear import quantize_model
    from efficientgpt_b200.nanogpt import GPT, GPTConfig, GraphDecoder
    cfg = GPTConfig(block_size=256, vocab_size=50304, n_layer=6, n_head=6, n_embd=384, bias=True)
    model = GPT(cfg, seed=0).cuda().eval()
    params = {n: p.detach().cpu().numpy().copy() for n, p in model.named_parameters()}
    quantize_model(model)
    prompt = torch.randint(0, cfg.vocab_size, (1, 64), generator=torch.Generator().manual_seed(0))
    dec = GraphDecoder(model, prompt.cuda())
    eng = dec.engine.engine
    dec.engine.reset(prompt.cuda())

    def set_pos(p):
        eng.position.fill_(p)

    time_replays(dec.graph, a.warmup, window_positions(a.warmup, 64, 64), set_pos)
    set_pos(64)
    positions = window_positions(a.steps, 64, 64)
    ms = time_replays(dec.graph, a.steps, positions, set_pos)
    bytes_tok = sum(b.numel() * b.element_size() for b in model.buffers() if b.dtype in (torch.int8, torch.float32))
    peaks, peak_src = measured_peaks()
    hbm = float(peaks['hbm_gbs'])
    gbs = bytes_tok / (ms / 1e3 / a.steps) / 1e9
    e2e = None
    if not a.no_e2e:
        host = prompt.pin_memory()
        vals = []
        for _ in range(3):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            dev_prompt = host.to('cuda', non_blocking=True)
            dec.engine.reset(dev_prompt)
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            for _ in range(63):
                dec.graph.replay()
            out = dec.engine.finish(64).cpu()
            t2 = time.perf_counter()
            vals.append(63 / (t2 - t1))
        e2e = {'value': statistics.median(vals), 'unit': 'tok/s', 'h2d_bytes_per_step': 64 * 8 / 64,
               'd2h_bytes_per_step': out.numel() * 8 / 64, 'ttft_ms': round((t1 - t0) * 1e3, 3),
               'api': 'efficientgpt_b200.nanogpt.GraphDecoder (pinned host prompt, 64 tokens, history read back)'}
    cb = None
    if not a.no_cpu_baseline:
        from oracle.nanogpt_ref import NanoGPTRef
        params['lm_head.weight'] = params['transformer.wte.weight']
        ref = NanoGPTRef(params, {'block_size': 256, 'n_layer': 6, 'n_head': 6, 'n_embd': 384}, semantics='cuda')
        lg = ref.forward(prompt[0].tolist(), 0)
        n = max(1, a.cpu_sample)
        t0 = time.perf_counter()
        pos = 64
        for _ in range(n):
            lg = ref.forward([int(lg.argmax())], pos)
            pos += 1
        cb = {'value': n / (time.perf_counter() - t0), 'unit': 'tok/s', 'cores': os.cpu_count(), 'kind': 'port',
              'sample': f'{n} decode tokens at context 65..{64 + n}, numpy restatement of the reference CPU path '
                        '(oracle/nanogpt_ref.py: x @ (q * s).T + b per linear, fp32)'}
    line = {'metric': 'batch-1 decode tok/s, nanoGPT 6x384 int8 (BASELINE config 1), 1 B200', 'value': round(a.steps / (ms / 1e3), 2),
            'unit': 'tok/s', 'n_gpus': 1, 'steps': a.steps, 'warmup': a.warmup, 'ms_per_step': round(ms / a.steps, 5),
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'int8-weight/fp32',
            'data': 'synthetic',
            'config': {'workload': 'nanogpt 6x384 int8 decode, BASELINE config 1', 'prompt': 64, 'new_tokens': 64,
                       'scale_dtype': 'fp32', 'init': 'N(0,0.02), seed 0', 'parallelism': 'single',
                       'l2': 'no flush: the 30 MB of weights are L2-resident by design (latency-bound step)'},
            'roofline': {'bound': 'hbm', 'kernel': 'nanoGPT step (graph of per-op kernels)', 'achieved': round(gbs, 1),
                         'peak': hbm, 'unit': 'GB/s', 'frac': round(gbs / hbm, 4), 'traffic': None,
                         'note': 'weights fit in L2: launch/latency-bound, the fraction is not a bandwidth limit',
                         'peak_source': peak_src},
            'e2e': e2e, 'cpu_baseline': cb, 'gpu_launches': a.steps * (1 + 8 * 6 + 2)}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------- configs 3 and 4
def _time_graph(fn, reps):
    """us per launch of `fn(i)` captured `reps` times in one graph, replayed 5 times (CUDA events)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        g.replay()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / (5 * reps) * 1e3


def run_gemv_sweep(a):
    """each (N, K) as a graph of `reps` launches over enough weight copies that one pass exceeds
    L2 (every launch reads HBM); CUDA-core kernel and the exact tensor-core kernel, alone and PDL-chained.
    Algorithmic bytes N*K + 2N (bf16 scales) + 2K (x) + 2N (out)."""
    from efficientgpt_b200 import ops
    peaks, src = measured_peaks()
    peak = float(peaks['hbm_gbs'])
    for n, k, what in ((4096, 2048, 'qkv'), (2048, 2048, 'o'), (12288, 2048, 'gate_up'), (2048, 6144, 'down'),
                       (151936, 2048, 'lm_head')):
        if a.only not in f'config 3 {what}':
            continue
        g = torch.Generator(device='cuda').manual_seed(0)
        copies = max(1, math.ceil(2 * L2_BYTES / (n * k)))
        ws = [torch.randint(-127, 128, (n, k), dtype=torch.int8, device='cuda', generator=g) for _ in range(copies)]
        s = (torch.rand(n, device='cuda', generator=g) * 0.019 + 0.001).to(torch.bfloat16)
        x = torch.randn(1, k, device='cuda', generator=g).to(torch.bfloat16)
        out = torch.empty(1, n, dtype=torch.bfloat16, device='cuda')
        nbytes = n * k + 2 * n + 2 * k + 2 * n
        f = lambda t: round(nbytes / (t * 1e-6) / 1e9 / peak, 4)
        res = {}
        for name, kw in (('alu', {}), ('alu_pdl', {'pdl': True}), ('exact', {'exact': True}),
                         ('exact_pdl', {'exact': True, 'pdl': True})):
            res[name] = _time_graph(lambda i: ops.gemv_i8(x, ws[i % copies], s, out=out, **kw), a.reps)
        print(json.dumps({'kernel': 'gemv_i8_kernel / gemv_tc_kernel', 'case': f'config 3 {what} N={n} K={k}',
                          'bytes': nbytes, 'peak_gbs': peak, 'peak_source': src, 'l2': f'{copies} weight copies rotated',
                          **{f'us_{m}': round(t, 3) for m, t in res.items()},
                          **{f'frac_{m}': f(t) for m, t in res.items()}}), flush=True)
        del ws


def run_gemm_prefill(a):
    """Prefill GEMMs of BASELINE config 5 (Qwen3-8B shape, 4096-token prompt) and config 2's gate|up at the same
    prompt length: egpt_gemm_i8_tc (bf16 x, int8 weights widened in shared memory, tcgen05) against the reference's
    own arithmetic on PyTorch (dequantise to bf16, cuBLAS GEMM, scale in fp32), both timed as graphs of `reps`
    launches. Compute-bound: 2 M N K flops against the measured dense bf16 peak."""
    from efficientgpt_b200 import ops
    peaks, src = measured_peaks()
    peak = float(peaks.get('bf16_tflops', 0)) or None
    m = 4096
    for what, n, k in (('8B qkv', 6144, 4096), ('8B o', 4096, 4096), ('8B gate_up', 24576, 4096),
                       ('8B down', 4096, 12288), ('1.7B gate_up', 12288, 2048)):
        if a.only not in f'prefill {what}':
            continue
        g = torch.Generator(device='cuda').manual_seed(n + k)
        x = torch.randn(m, k, device='cuda', generator=g).to(torch.bfloat16)
        q = torch.randint(-127, 128, (n, k), dtype=torch.int8, device='cuda', generator=g)
        sc = (torch.rand(n, device='cuda', generator=g) * 0.019 + 0.001).to(torch.bfloat16)
        out = torch.empty(m, n, dtype=torch.bfloat16, device='cuda')
        t_tc = _time_graph(lambda i: ops.gemm_i8_tc(x, q, sc, out=out), a.reps)
        t_ref = _time_graph(lambda i: ((x @ q.to(torch.bfloat16).t()).float() * sc.float()).to(torch.bfloat16), a.reps)
        tf = lambda t: 2.0 * m * n * k / (t * 1e-6) / 1e12
        print(json.dumps({'kernel': 'gemm_i8_tc_kernel', 'case': f'prefill {what} M={m} N={n} K={k}',
                          'us_tcgen05': round(t_tc, 2), 'tflops_tcgen05': round(tf(t_tc), 1),
                          'us_reference_torch': round(t_ref, 2), 'tflops_reference_torch': round(tf(t_ref), 1),
                          'peak_tflops': peak, 'frac_tcgen05': round(tf(t_tc) / peak, 4) if peak else None,
                          'peak_source': src}), flush=True)
        del x, q, out
    # causal attention over the prompt: egpt_attn_prefill (tcgen05) against PyTorch's SDPA (the reference's call);
    # useful flops 2 nq d p (p + 1) (QK^T and P.V over the causal triangle)
    for what, p, nq, nkv in (('8B', 4096, 32, 8), ('1.7B', 4096, 16, 8), ('8B', 1024, 32, 8)):
        if a.only not in f'prefill attention {what} p={p}':
            continue
        d = 128
        g = torch.Generator(device='cuda').manual_seed(p + nq)
        q = torch.randn(p, nq * d, device='cuda', generator=g).to(torch.bfloat16)
        kc = torch.randn(nkv, p, d, device='cuda', generator=g).to(torch.bfloat16)
        vc = torch.randn(nkv, p, d, device='cuda', generator=g).to(torch.bfloat16)
        out = torch.empty(p, nq * d, dtype=torch.bfloat16, device='cuda')
        t_tc = _time_graph(lambda i: ops.attn_prefill(q, kc, vc, 0, nq, nkv, d, scale=d ** -0.5, out=out), a.reps)
        qh = q.view(p, nq, d).transpose(0, 1).unsqueeze(0)
        t_ref = _time_graph(lambda i: torch.nn.functional.scaled_dot_product_attention(
            qh, kc.unsqueeze(0), vc.unsqueeze(0), is_causal=True, scale=d ** -0.5, enable_gqa=True), a.reps)
        tf = lambda t: 2.0 * nq * d * p * (p + 1) / (t * 1e-6) / 1e12
        print(json.dumps({'kernel': 'attn_prefill_kernel', 'case': f'prefill attention {what} p={p} nq={nq} nkv={nkv}',
                          'us_tcgen05': round(t_tc, 2), 'tflops_tcgen05': round(tf(t_tc), 1),
                          'us_reference_sdpa': round(t_ref, 2), 'tflops_reference_sdpa': round(tf(t_ref), 1),
                          'peak_tflops': peak, 'frac_tcgen05': round(tf(t_tc) / peak, 4) if peak else None,
                          'peak_source': src}), flush=True)
        del q, kc, vc, out


def run_ragged(a):
    """Ragged small-batch greedy decode (efficientgpt_b200.ragged) on the BASELINE config 2 model: B in {1, 4, 16}
    sequences with prompt lengths spread over 8..32, `--steps` graph replays timed with CUDA events after the
    prompts; aggregate tok/s = B x steps / time. The weights stream once per step for the whole batch."""
    from efficientgpt_b200.configs import qwen3_1p7b_config, random_model
    from efficientgpt_b200.int8_linear import quantize_model
    from efficientgpt_b200.ragged import RaggedGraphDecoder
    cfg = qwen3_1p7b_config()
    model = random_model(cfg, 'cuda', 0)
    quantize_model(model, scale_dtype=torch.bfloat16)
    for b in (1, 4, 16):
        g = torch.Generator().manual_seed(b)
        lengths = torch.randint(8, 33, (b,), generator=g)
        prompts = torch.randint(0, cfg.vocab_size, (b, int(lengths.max())), generator=g)
        dec = RaggedGraphDecoder(model, b, int(lengths.max()) + a.steps + a.warmup + 1)
        dec.generate(prompts.cuda(), lengths.cuda(), a.warmup + 1)  # capture, prefill, warm-up replays
        for r in range(b):
            dec.engine.prefill_row(r, prompts[r, :int(lengths[r])].cuda())
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            dec.graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / a.steps
        print(json.dumps({'workload': 'ragged', 'model': 'qwen3_1.7b int8 (config 2 shape)', 'batch': b,
                          'prompt_lengths': lengths.tolist(), 'steps': a.steps, 'ms_per_step': round(ms, 4),
                          'tok_s': round(b * 1e3 / ms, 1)}), flush=True)
        del dec


def run_attn_sweep(a):
    """16 q / 8 kv heads of 128, one query, L in {512, 2048, 8192, 32768}; graphs of `reps`
    launches over enough cache copies to exceed L2. Algorithmic bytes 4096 L + 8192."""
    from efficientgpt_b200 import ops
    peaks, src = measured_peaks()
    peak = float(peaks['hbm_gbs'])
    nq, nkv, d = 16, 8, 128
    for length in (512, 2048, 8192, 32768):
        if a.only not in f'config 4 L={length}':
            continue
        g = torch.Generator(device='cuda').manual_seed(length)
        per = 2 * nkv * length * d * 2
        copies = max(1, math.ceil(2 * L2_BYTES / per))
        ks = [torch.randn(nkv, length, d, device='cuda', generator=g).to(torch.bfloat16) for _ in range(copies)]
        vs = [torch.randn(nkv, length, d, device='cuda', generator=g).to(torch.bfloat16) for _ in range(copies)]
        q = torch.randn(1, nq * d, device='cuda', generator=g).to(torch.bfloat16)
        pos = torch.tensor([length - 1], device='cuda')
        max_split = 64
        ws = ops.attn_ws(1, nq, nkv, d, max_split, 'cuda')
        out = torch.empty(1, nq * d, dtype=torch.bfloat16, device='cuda')
        for ref in (False, True):
            us = _time_graph(lambda i: ops.attn_decode(q, ks[i % copies], vs[i % copies], pos, nq, nkv, d,
                                                       scale=d ** -0.5, max_split=max_split, ws=ws, out=out,
                                                       ref_softmax=ref), a.reps)
            nbytes = 4096 * length + 8192
            gbs = nbytes / (us * 1e-6) / 1e9
            print(json.dumps({'kernel': 'attn_block_max_kernel + attn_stream_kernel' if ref else 'attn_stream_kernel',
                              'case': f'config 4 L={length}' + (' ref_softmax' if ref else ''),
                              'us': round(us, 3), 'bytes': nbytes, 'achieved_gbs': round(gbs, 1), 'peak_gbs': peak,
                              'frac': round(gbs / peak, 4), 'peak_source': src,
                              'l2': f'{copies} cache copies rotated'}), flush=True)
        del ks, vs


def run_profile_step(a):
    """A small decode workload for ncu captures: the Qwen3-1.7B shape with --layers decoder layers, a 32-token
    prefill and --steps decode steps of the --step kernel."""
    from efficientgpt_b200 import _lib
    from efficientgpt_b200.configs import qwen3_1p7b_config, random_model
    from efficientgpt_b200.engine import Qwen3Engine
    from efficientgpt_b200.int8_linear import quantize_model
    cfg = qwen3_1p7b_config()
    cfg.num_hidden_layers = a.layers
    model = random_model(cfg, 'cuda', 0)
    quantize_model(model, scale_dtype=torch.bfloat16)
    eng = Qwen3Engine(model, PROMPT_LEN + NEW_TOKENS, step=a.step)
    eng.prefill(torch.randint(0, cfg.vocab_size, (1, PROMPT_LEN), generator=torch.Generator().manual_seed(0)).cuda())
    for _ in range(a.steps):
        eng.step()
    torch.cuda.synchronize()
    err = _lib.device_error()
    if err != 0:
        raise RuntimeError(f'device error {err}')
    print(json.dumps({'workload': 'profile_step', 'layers': a.layers, 'steps': a.steps, 'token': int(eng.token),
                      'position': int(eng.position), 'bytes_per_step': eng.weight_bytes(),
                      'step': eng.step_kind}), flush=True)


def main():
    a = parse()
    if a.impl == 'reference':
        # the CPU path: no process group, no GPU; ranks other than 0 exit without work
        run_reference(a, int(os.environ.get('RANK', '0')))
        return
    world, rank, local = dist_setup()
    single = {'nanogpt': lambda: run_nanogpt(a, rank), 'gemv_sweep': lambda: run_gemv_sweep(a),
              'gemm_prefill': lambda: run_gemm_prefill(a), 'ragged': lambda: run_ragged(a),
              'attn_sweep': lambda: run_attn_sweep(a), 'profile_step': lambda: run_profile_step(a)}
    if a.workload in single:
        if rank == 0:
            single[a.workload]()
        line = None
    elif a.workload == 'qwen3_8b':
        line = run_tp(a, world, rank, local, 'qwen3_8b')
    else:
        line = run_config2(a, world, rank, local)
        if world > 1 and not a.no_tp:
            tp_line = run_tp(a, world, rank, local, 'qwen3_8b')
            if line is not None:
                line['tensor_parallel'] = {k: tp_line[k] for k in ('metric', 'value', 'unit', 'ms_per_step', 'config',
                                                                   'roofline', 'nvlink_bytes_per_token_per_gpu',
                                                                   'device_error', 'e2e', 'gpu_launches', 'clocks')}
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()


if __name__ == '__main__':
    sys.path.insert(0, str(ROOT))
    main()
