"""Per-kernel sweeps of BASELINE configs 3 (int8 GEMV) and 4 (GQA decode attention) against the HBM roofline, and
the config-1 nanoGPT decode rate.

    python -m efficientgpt_b200.kernel_bench [--reps 50] [--skip-nanogpt] [--only lm_head]

Each case replays a CUDA graph of `reps` launches (device time from CUDA events around the replays, so host launch
cost is not counted) over enough weight / cache copies that one pass of the graph exceeds L2 (126 MB): every
launch reads from HBM. Algorithmic bytes: GEMV N*K + 2N (bf16 scales) + 2K (x) + 2N (out); attention
4096*L + 8192 (K and V of 8 kv heads x d 128 in bf16, q and out). Peak: MEASURED_PEAKS.json hbm_gbs when present.
nanoGPT (config 1: 6 layers, 384 dims, vocab 50304, block 256, int8 weights with fp32 scales, fp32 activations,
N(0, 0.02) init, 64-token prompt, 64 greedy tokens): graph replays of the native decode step timed with CUDA events
(its 30 MB of weights fit in L2, so the step is launch- and latency-bound, not HBM-bound); the CPU baseline of
config 1 is timed by `bench.py --workload nanogpt`. Prints one JSON line per case.
"""
import argparse
import json
import math
from pathlib import Path

import torch

L2_BYTES = 126 * 2 ** 20


def peak_gbs():
    p = Path(__file__).resolve().parent.parent / 'MEASURED_PEAKS.json'
    if p.exists():
        return float(json.loads(p.read_text())['hbm_gbs']), 'measured'
    return 6650.0, 'fallback'


def time_graph(fn, reps):
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
    return e0.elapsed_time(e1) / (5 * reps) * 1e3  # us per launch


def gemv_cases(reps, peak, src, only=''):
    from . import ops
    for n, k, what in ((4096, 2048, 'qkv'), (2048, 2048, 'o'), (12288, 2048, 'gate_up'), (2048, 6144, 'down'),
                       (151936, 2048, 'lm_head')):
        if only not in f'config 3 {what}':
            continue
        g = torch.Generator(device='cuda').manual_seed(0)
        copies = max(1, math.ceil(2 * L2_BYTES / (n * k)))
        ws = [torch.randint(-127, 128, (n, k), dtype=torch.int8, device='cuda', generator=g) for _ in range(copies)]
        s = (torch.rand(n, device='cuda', generator=g) * 0.019 + 0.001).to(torch.bfloat16)
        x = torch.randn(1, k, device='cuda', generator=g).to(torch.bfloat16)
        out = torch.empty(1, n, dtype=torch.bfloat16, device='cuda')
        us = time_graph(lambda i: ops.gemv_i8(x, ws[i % copies], s, out=out), reps)
        # chained with programmatic dependent launch, as the launch-sequence decode path runs it: a launch streams
        # its first weights while the previous one drains
        us_pdl = time_graph(lambda i: ops.gemv_i8(x, ws[i % copies], s, out=out, pdl=True), reps)
        # the exact int8 tensor-core kernel (EGPT_FLAG_EXACT), alone and PDL-chained
        us_tc = time_graph(lambda i: ops.gemv_i8(x, ws[i % copies], s, out=out, exact=True), reps)
        us_tc_pdl = time_graph(lambda i: ops.gemv_i8(x, ws[i % copies], s, out=out, exact=True, pdl=True), reps)
        nbytes = n * k + 2 * n + 2 * k + 2 * n
        f = lambda t: round(nbytes / (t * 1e-6) / 1e9 / peak, 4)
        gbs = nbytes / (us * 1e-6) / 1e9
        yield {'kernel': 'gemv_i8_kernel', 'case': f'config 3 {what} N={n} K={k}', 'us': round(us, 3),
               'bytes': nbytes, 'achieved_gbs': round(gbs, 1), 'peak_gbs': peak, 'frac': round(gbs / peak, 4),
               'us_pdl_chain': round(us_pdl, 3), 'frac_pdl_chain': f(us_pdl),
               'exact_tc': {'kernel': 'gemv_tc_kernel', 'us': round(us_tc, 3), 'frac': f(us_tc),
                            'us_pdl_chain': round(us_tc_pdl, 3), 'frac_pdl_chain': f(us_tc_pdl)},
               'peak_source': src, 'l2': f'{copies} weight copies rotated'}
        del ws


def attention_cases(reps, peak, src, only=''):
    from . import ops
    nq, nkv, d = 16, 8, 128
    for length in (512, 2048, 8192, 32768):
        if only not in f'config 4 L={length}':
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
            us = time_graph(lambda i: ops.attn_decode(q, ks[i % copies], vs[i % copies], pos, nq, nkv, d, scale=d ** -0.5,
                                                      max_split=max_split, ws=ws, out=out, ref_softmax=ref), reps)
            nbytes = 4096 * length + 8192
            gbs = nbytes / (us * 1e-6) / 1e9
            yield {'kernel': 'attn_split_kernel', 'case': f'config 4 L={length}' + (' ref_softmax' if ref else ''),
                   'us': round(us, 3), 'bytes': nbytes, 'achieved_gbs': round(gbs, 1), 'peak_gbs': peak,
                   'frac': round(gbs / peak, 4), 'peak_source': src, 'l2': f'{copies} cache copies rotated'}
        del ks, vs


def nanogpt_case(n_tokens=63):
    """Config-1 decode rate: graph replays of the native nanoGPT decode step (64-token prompt, contexts 65..127).
    Returns (line, model parameters as numpy arrays, prompt) so a caller can time a CPU baseline on the same model."""
    from .int8_linear import quantize_model
    from .nanogpt import GPT, GPTConfig, GraphDecoder
    cfg = GPTConfig(block_size=256, vocab_size=50304, n_layer=6, n_head=6, n_embd=384, bias=True)
    model = GPT(cfg, seed=0).cuda().eval()
    params = {n: p.detach().cpu().numpy().copy() for n, p in model.named_parameters()}
    quantize_model(model)
    prompt = torch.randint(0, cfg.vocab_size, (1, 64), generator=torch.Generator().manual_seed(0)).cuda()
    dec = GraphDecoder(model, prompt)
    eng = dec.engine
    eng.reset(prompt)
    for _ in range(3):
        dec.graph.replay()
    eng.reset(prompt)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n_tokens):
        dec.graph.replay()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / n_tokens
    line = {'kernel': 'nanoGPT decode step (one CUDA graph: 48 library kernels + history write)',
            'case': 'config 1 (6x384, vocab 50304), context 65..127', 'tok_s': round(1e3 / ms, 1),
            'ms_per_token': round(ms, 4), 'bound': 'latency (weights 30 MB, L2-resident)'}
    return line, params, prompt


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reps', type=int, default=50)
    ap.add_argument('--skip-nanogpt', action='store_true')
    ap.add_argument('--only', default='', help='run only the cases whose name contains this text (e.g. lm_head)')
    a = ap.parse_args()
    peak, src = peak_gbs()
    for line in gemv_cases(a.reps, peak, src, a.only):
        print(json.dumps(line), flush=True)
    for line in attention_cases(a.reps, peak, src, a.only):
        print(json.dumps(line), flush=True)
    if not a.skip_nanogpt:
        print(json.dumps(nanogpt_case()[0]), flush=True)


if __name__ == '__main__':
    main()
