#!/usr/bin/env python
"""Batch-1 greedy decode throughput of the Qwen3-1.7B-shape int8 model on B200 (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token: one replay of the CUDA graph that holds the native decode step (one persistent
cooperative kernel per token; 141 kernels per token on the launch-sequence path). Workload = BASELINE config 2: random-init weights (seed 0), int8 per-row weights with bf16 scales,
a 32-token uniform prompt, then 256 greedy tokens; the timed loop replays that 256-token window (position reset
to 32 every 256 steps), so contexts run 33..288 as in the config. The 1.72 GB of weights streamed per token are
far larger than L2 (126 MB), so no flush is needed between steps.

Printed JSON line (rank 0):
  value        decode tok/s over all ranks, device-timed (CUDA events around the K replays, max over ranks)
  e2e          the same metric through GraphGreedyDecoder.generate with a pinned host prompt: H2D prompt copy,
               per-token D2H token reads, (n - 1) / (total - ttft) as research/realmodel/bench_int8.py
  step_roofline  algorithmic bytes per token (weights + scales + norms + embedding row + KV at each step's
               context) / step time, against the measured HBM copy bandwidth
  roofline     the dominant kernel. Persistent step (default on this shape): decode_step_kernel, one launch
               per token, so achieved = algorithmic bytes per token / (device time / K); traffic = its ncu
               dram bytes per launch from the committed summary. Launch sequence: the step's GEMV launches
               replayed alone as one PDL-chained graph (gemv_i8_kernel).
  gemv_chain   the GEMV launches of the launch-sequence path replayed alone (for comparison)
  cpu_baseline the reference's CPU path (oracle/torch_ref.py) on this host's cores, bounded sample
With N > 1 (torchrun, one rank per GPU) the default workload is BASELINE config 5, the model the reference's north
star shards: Qwen3-8B shape, 4096-token prompt fed through the step, 256 greedy tokens, tensor-parallel over the N
GPUs (efficientgpt_b200.tp: one persistent kernel per GPU and token, o_proj / down_proj partial sums exchanged over
NVLink inside it; scaling "strong"). --workload selects either model at any N (qwen3_8b on one GPU runs the
launch sequence: its 12288-wide MLP does not fit the persistent kernel's shared memory); --replicas runs N
independent one-GPU replicas of config 2 instead (scaling "weak").
"""
import argparse
import json
import os
import re
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
PROFILE_SUMMARY = ROOT / 'profiles' / 'decode_step_kernel_qwen3_1p7b.md'


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=2048)
    ap.add_argument('--warmup', type=int, default=16)
    ap.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-pdl', action='store_true')
    ap.add_argument('--launch-sequence', action='store_true', help='per-stage kernels instead of the persistent step')
    ap.add_argument('--no-gemv-chain', action='store_true', help='skip the GEMV-launches-alone comparison graph')
    ap.add_argument('--cpu-sample', type=int, default=3, help='timed CPU decode tokens (after one warm-up token)')
    ap.add_argument('--workload', choices=['qwen3_1.7b', 'qwen3_8b', 'nanogpt'], default=None,
                    help='default: qwen3_1.7b (config 2) on one GPU, qwen3_8b (config 5, tensor-parallel) on N > 1')
    ap.add_argument('--replicas', action='store_true', help='N > 1: independent replicas instead of tensor parallelism')
    a = ap.parse_args()
    if a.warmup < 3:
        ap.error('--warmup must be >= 3')
    if a.workload is None:
        a.workload = 'qwen3_8b' if a.gpus > 1 and not a.replicas else 'qwen3_1.7b'
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
        self.out = None

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


def profile_traffic():
    """dram bytes read+write per launch of the dominant kernel, from the committed ncu summary (or None)."""
    if not PROFILE_SUMMARY.exists():
        return None
    m = re.search(r'traffic_bytes_per_launch\s*[:=]\s*([0-9.eE+]+)', PROFILE_SUMMARY.read_text())
    return float(m.group(1)) if m else None


def build(device, pdl, persistent=None):
    from efficientgpt_b200.configs import qwen3_1p7b_config, random_model
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    from efficientgpt_b200.int8_linear import quantize_model
    model = random_model(qwen3_1p7b_config(), device, seed=0)
    quantize_model(model, scale_dtype=torch.bfloat16)
    torch.cuda.empty_cache()
    dec = GraphGreedyDecoder(model, max_cache_len=PROMPT_LEN + NEW_TOKENS, pdl=pdl, persistent=persistent)
    prompt = torch.randint(0, model.config.vocab_size, (1, PROMPT_LEN), generator=torch.Generator().manual_seed(0))
    return model, dec, prompt


def gemv_chain_graph(eng):
    """A graph with only the step's GEMV launches (same shapes, weights and buffers, PDL-chained)."""
    from efficientgpt_b200 import _lib as L, ops
    H, I = eng.hidden, eng.inter
    x_h = eng.h.view(1, H)
    qkv = eng.qkv.view(1, -1)
    attn = eng.attn.view(1, -1)
    act = eng.act.view(1, I)

    def chain():
        for lay in eng.layers:
            ops.gemv_i8(x_h, lay['w_qkv'], lay['s_qkv'], out=qkv, norm_w=lay['ln_in'], eps=eng.eps, pdl=True)
            ops.gemv_i8(attn, lay['w_o'], lay['s_o'], epilogue=L.EPI_RESIDUAL, residual=x_h, pdl=True)
            ops.gemv_i8(x_h, lay['w_gu'], lay['s_gu'], out=act, epilogue=L.EPI_SILU_MUL, norm_w=lay['ln_post'],
                        eps=eng.eps, pdl=True)
            ops.gemv_i8(act, lay['w_down'], lay['s_down'], epilogue=L.EPI_RESIDUAL, residual=x_h, pdl=True)
        ops.lm_head_argmax(eng.h, eng.w_lm, eng.s_lm, eng.lm_ws, norm_w=eng.final_norm, eps=eng.eps, token=eng.token,
                           pdl=True)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            chain()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain()
    nbytes = 0
    for lay in eng.layers:
        for w, s_ in (('w_qkv', 's_qkv'), ('w_o', 's_o'), ('w_gu', 's_gu'), ('w_down', 's_down')):
            n, k = lay[w].shape
            nbytes += n * k + n * lay[s_].element_size() + 2 * k + 2 * n
        nbytes += 2 * lay['ln_in'].numel() + 2 * lay['ln_post'].numel() + 2 * H + 2 * H  # norm weights, residual rw
    nbytes += eng.w_lm.numel() + eng.s_lm.numel() * eng.s_lm.element_size() + 2 * H * 2
    return g, nbytes, 4 * len(eng.layers) + 1


def time_replays(graph, k, reset=None, window=NEW_TOKENS):
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for i in range(k):
        if reset is not None and i and i % window == 0:
            reset()
        graph.replay()
    e1.record(st)
    e1.synchronize()
    return e0.elapsed_time(e1)


def cpu_baseline(dec, n_tokens):
    """The reference's CPU decode path (oracle/torch_ref.py) on this host: 1 warm-up + n_tokens timed steps at
    the contexts right after the 32-token prompt (KV of the prompt copied from the GPU prefill)."""
    from oracle.torch_ref import TorchCpuQwen3
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    eng = dec.engine
    cpu = TorchCpuQwen3(eng, PROMPT_LEN + n_tokens + 2)
    cpu.k[:, 0, :, :PROMPT_LEN] = eng.kv[:, 0, :, :PROMPT_LEN].cpu()
    cpu.v[:, 0, :, :PROMPT_LEN] = eng.kv[:, 1, :, :PROMPT_LEN].cpu()
    tok = int(eng.token)
    tok = cpu.step(tok, PROMPT_LEN)
    t0 = time.perf_counter()
    for i in range(n_tokens):
        tok = cpu.step(tok, PROMPT_LEN + 1 + i)
    dt = time.perf_counter() - t0
    return {'value': n_tokens / dt, 'unit': 'tok/s', 'cores': threads, 'kind': 'port',
            'sample': f'{n_tokens} decode tokens (after 1 warm-up token) of the same Qwen3-1.7B-shape int8 model at '
                      f'context {PROMPT_LEN + 2}..{PROMPT_LEN + 1 + n_tokens}, torch CPU ops, '
                      f'bf16((x.float() @ q.float().T) * s) per linear'}


class _CpuWeights:
    """The attributes oracle/torch_ref.TorchCpuQwen3 reads, from tp.full_weights of a quantised model."""

    def __init__(self, model):
        from efficientgpt_b200 import tp
        c = model.config
        shape = tp.Qwen3Shape.from_config(c)
        full = tp.full_weights(model)
        self.nq, self.nkv, self.d, self.eps = shape.nq, shape.nkv, shape.d, shape.eps
        self.hidden, self.inter = shape.hidden, shape.inter
        self.layers = full['layers']
        self.embed, self.final_norm, self.w_lm, self.s_lm = full['embed'], full['final_norm'], full['w_lm'], full['s_lm']
        self.rope_cos, self.rope_sin = tp.rope_tables(shape, 4096 + NEW_TOKENS, model.device, full['rotary'])


def run_reference_8b(a, world, rank):
    """The reference's CPU decode path on the config-5 model: a bounded sample of decode steps at context
    4097.. with the 4096 prompt positions of the KV cache filled from a seeded draw (a CPU prefill of 4096 tokens
    through an 8B model would take far longer than the run allows)."""
    if rank != 0:
        return
    from oracle.torch_ref import TorchCpuQwen3
    from efficientgpt_b200.configs import qwen3_8b_config, random_model
    from efficientgpt_b200.int8_linear import quantize_model
    model = random_model(qwen3_8b_config(), 'cuda', seed=0)
    quantize_model(model, scale_dtype=torch.bfloat16)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n = max(1, min(a.steps, a.cpu_sample))
    cpu = TorchCpuQwen3(_CpuWeights(model), 4096 + n + 2)
    del model
    g = torch.Generator().manual_seed(0)
    cpu.k[:, :, :, :4096].copy_(torch.randn(cpu.k[:, :, :, :4096].shape, generator=g).to(torch.bfloat16))
    cpu.v[:, :, :, :4096].copy_(torch.randn(cpu.v[:, :, :, :4096].shape, generator=g).to(torch.bfloat16))
    tok = cpu.step(11, 4096)
    t0 = time.perf_counter()
    for i in range(n):
        tok = cpu.step(tok, 4097 + i)
    v = n / (time.perf_counter() - t0)
    cb = {'value': v, 'unit': 'tok/s', 'cores': threads, 'kind': 'port',
          'sample': f'{n} decode tokens (after 1 warm-up token) of the Qwen3-8B-shape int8 model at context '
                    f'4098..{4097 + n}, KV of the 4096 prompt positions from a seeded draw, torch CPU ops, '
                    f'bf16((x.float() @ q.float().T) * s) per linear'}
    line = {'impl': 'reference', 'metric': METRIC.replace('Qwen3-1.7B', 'Qwen3-8B').replace('1 B200', f'{world} B200'),
            'value': v, 'unit': 'tok/s', 'n_gpus': world, 'steps': n, 'warmup': 1, 'ms_per_step': 1e3 / v,
            'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'int8-weight/bf16',
            'data': 'synthetic',
            'config': {'workload': 'qwen3_8b int8 decode, BASELINE config 5 (CPU port of the reference path)',
                       'prompt': 4096, 'new_tokens': NEW_TOKENS, 'scale_dtype': 'bf16'},
            'cpu_baseline': cb, 'e2e': {'value': v, 'unit': 'tok/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def run_reference(a, world, rank):
    if a.workload == 'qwen3_8b':
        run_reference_8b(a, world, rank)
        return
    if rank != 0:
        return
    _, dec, _ = build('cuda', pdl=True)
    dec.engine.prefill(torch.randint(0, dec.engine.vocab, (1, PROMPT_LEN),
                                     generator=torch.Generator().manual_seed(0)).cuda())
    n = max(1, min(a.steps, a.cpu_sample))
    cb = cpu_baseline(dec, n)
    line = {'impl': 'reference', 'metric': METRIC, 'value': cb['value'], 'unit': 'tok/s', 'n_gpus': a.gpus,
            'steps': n, 'warmup': 1, 'ms_per_step': 1e3 / cb['value'], 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'int8-weight/bf16', 'data': 'synthetic',
            'config': {'workload': 'qwen3_1.7b int8 decode, BASELINE config 2 (CPU port of the reference path)',
                       'prompt': PROMPT_LEN, 'new_tokens': NEW_TOKENS, 'scale_dtype': 'bf16'},
            'cpu_baseline': cb, 'e2e': {'value': cb['value'], 'unit': 'tok/s', 'h2d_bytes_per_step': 0,
                                        'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def run_tp(a, world, rank, local):
    """Tensor-parallel decode over the `world` GPUs (world 1: the same engine on one GPU): K timed replays of a
    graph holding one step, device time max over ranks; every rank builds the same seeded model and keeps its
    shard."""
    from efficientgpt_b200 import tp
    from efficientgpt_b200.configs import qwen3_1p7b_config, qwen3_8b_config, random_model
    from efficientgpt_b200.int8_linear import quantize_model
    big = a.workload == 'qwen3_8b'
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

    def reset():
        eng.position.fill_(prompt_len)

    reset()
    time_replays(graph, a.warmup)
    reset()
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    torch.cuda.synchronize(dev)
    barrier(world)  # after the sampler's start-up: the ranks' kernels wait on one another with a bounded wait
    ms = time_replays(graph, a.steps, reset)
    clocks = sampler.stop(local) if rank == 0 else None
    ms = max_over_ranks(ms, world)
    barrier(world)
    from efficientgpt_b200._lib import device_error
    err = device_error()
    tok_s = a.steps / (ms / 1e3)  # one token per step for the whole job (all ranks decode the same token)

    ctxs = [prompt_len + 1 + (i % NEW_TOKENS) for i in range(a.steps)]
    bytes_rank = eng.weight_bytes() + statistics.fmean(eng.kv_bytes_per_token(c) for c in ctxs)
    peaks, peak_src = measured_peaks()
    hbm = float(peaks['hbm_gbs'])
    gbs = bytes_rank / (ms / 1e3 / a.steps) / 1e9
    nvlink = 2 * shape.n_layers * shape.hidden * 8 * (world - 1) + 8 * (world - 1) if world > 1 else 0

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
               'api': 'efficientgpt_b200.tp.TPQwen3Engine.feed (pinned host prompt: GEMM prefill beyond 64 tokens, '
                      'token by token below), then one graph replay and one token read per step'}
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
                       'step': 'persistent' if eng.persistent else 'launch sequence'},
            'roofline': {'bound': 'hbm', 'kernel': 'decode_step_kernel' if eng.persistent else 'gemv_i8_kernel',
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
        print(json.dumps(line), flush=True)
    del graph
    eng.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_nanogpt(a, world, rank):
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

    def reset():
        eng.position.fill_(64)

    time_replays(dec.graph, a.warmup)
    reset()
    ms = time_replays(dec.graph, a.steps, reset, window=64)
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


def main():
    a = parse()
    world, rank, local = dist_setup()
    if a.workload == 'nanogpt':
        run_nanogpt(a, world, rank)
        return
    if a.impl == 'reference':
        run_reference(a, world, rank)
        return
    if a.workload == 'qwen3_8b' or (world > 1 and not a.replicas):
        run_tp(a, world, rank, local)
        return
    model, dec, prompt = build('cuda', pdl=not a.no_pdl, persistent=False if a.launch_sequence else None)
    eng = dec.engine
    dec._capture()
    eng.prefill(prompt.cuda())

    def reset():
        eng.position.fill_(PROMPT_LEN)

    # warm-up, then the timed region: K replays of the graph (one token each)
    time_replays(dec.graph, a.warmup)
    reset()
    barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    ms = time_replays(dec.graph, a.steps, reset)
    clocks = sampler.stop(local) if rank == 0 else None
    ms = max_over_ranks(ms, world)
    barrier(world)
    tok_s = a.steps / (ms / 1e3) * world

    # algorithmic bytes per token over the timed window
    ctxs = [PROMPT_LEN + 1 + (i % NEW_TOKENS) for i in range(a.steps)]
    kv_mean = statistics.fmean(eng.kv_bytes_per_token(c) for c in ctxs)
    bytes_tok = eng.weight_bytes() + kv_mean
    peaks, peak_src = measured_peaks()
    hbm = float(peaks['hbm_gbs'])
    step_gbs = bytes_tok / (ms / 1e3 / a.steps) / 1e9

    # the GEMV launches of the launch-sequence path alone
    gemv, g = None, None
    if not a.no_gemv_chain or not eng.persistent:
        g, gemv_bytes, gemv_launches = gemv_chain_graph(eng)
        reps = 64
        time_replays(g, 4)
        gms = time_replays(g, reps) / reps
        gemv_gbs = gemv_bytes / (gms / 1e3) / 1e9
        gemv = {'kernel': 'gemv_i8_kernel', 'achieved': round(gemv_gbs, 1), 'peak': hbm, 'unit': 'GB/s',
                'frac': round(gemv_gbs / hbm, 4), 'launches_per_step': gemv_launches, 'bytes_per_step': gemv_bytes,
                'avg_launch_us': round(gms * 1e3 / gemv_launches, 3)}
    if eng.persistent:  # one launch per token: the kernel's duration is the step's device time
        roofline = {'bound': 'hbm', 'kernel': 'decode_step_kernel', 'achieved': round(step_gbs, 1), 'peak': hbm,
                    'unit': 'GB/s', 'frac': round(step_gbs / hbm, 4), 'traffic': profile_traffic(),
                    'launches_per_step': 1, 'bytes_per_launch': round(bytes_tok),
                    'avg_launch_us': round(ms * 1e3 / a.steps, 3), 'peak_source': peak_src}
        launches = a.steps
    else:
        roofline = dict(gemv, bound='hbm', traffic=None, peak_source=peak_src)
        launches = a.steps * (5 * eng.n_layers + 1)

    e2e = None
    if not a.no_e2e:
        reset()
        host_prompt = prompt.pin_memory()
        vals = []
        for _ in range(3):
            out, st = dec.generate(host_prompt, NEW_TOKENS)
            vals.append((st['tokens'] - 1) / (st['total_s'] - st['ttft_s']))
        e2e = {'value': statistics.median(vals) * world, 'unit': 'tok/s', 'h2d_bytes_per_step': PROMPT_LEN * 8 / NEW_TOKENS,
               'd2h_bytes_per_step': 8, 'ttft_ms': round(st['ttft_s'] * 1e3, 3),
               'api': 'efficientgpt_b200.GraphGreedyDecoder.generate (pinned host prompt, 256 new tokens)'}

    cb = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cb = cpu_baseline(dec, a.cpu_sample)

    if rank == 0:
        line = {
            'metric': METRIC, 'value': round(tok_s, 2), 'unit': 'tok/s', 'n_gpus': world, 'steps': a.steps,
            'warmup': a.warmup, 'ms_per_step': round(ms / a.steps, 5), 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'int8-weight/bf16', 'data': 'synthetic',
            'config': {'workload': 'qwen3_1.7b int8 decode, BASELINE config 2', 'prompt': PROMPT_LEN,
                       'new_tokens': NEW_TOKENS, 'scale_dtype': 'bf16', 'init': 'HF random init N(0,0.02), seed 0',
                       'parallelism': f'replicas{world}' if world > 1 else 'single',
                       'l2': 'no flush: 1.72 GB of weights streamed per step, larger than L2',
                       'pdl': not a.no_pdl, 'step': 'persistent' if eng.persistent else 'launch sequence'},
            'tok_s_per_gpu': round(tok_s / world, 2),
            'step_roofline': {'bound': 'hbm', 'bytes_per_token': round(bytes_tok), 'achieved': round(step_gbs, 1),
                              'peak': hbm, 'unit': 'GB/s', 'frac': round(step_gbs / hbm, 4), 'peak_source': peak_src},
            'roofline': roofline,
            'gemv_chain': gemv,
            'e2e': e2e,
            'cpu_baseline': cb,
            'gpu_launches': launches,
            'clocks': clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        del g
        dist.destroy_process_group()


if __name__ == '__main__':
    sys.path.insert(0, str(ROOT))
    main()
