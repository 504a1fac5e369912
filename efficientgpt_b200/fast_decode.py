"""Sync-free greedy decoding with one CUDA graph per token, on the native B200 decode step.

Drop-in for BagelsFun/efficientgpt research/realmodel/fast_decode.py:25-111 GraphGreedyDecoder: same
constructor (model, max_cache_len, lookahead=8), same `generate(input_ids, max_new_tokens, eos_ids=(),
on_token=None) -> (tokens, {'ttft_s', 'total_s', 'tokens', 'capture_s'})`, same guards (batch 1,
max_new_tokens >= 1, prompt + new tokens <= max_cache_len) and the same host loop: per token one graph replay
plus a non-blocking copy of the token into pinned memory and an event; tokens are emitted as their events
complete, run-ahead is bounded by `lookahead`, EOS stops emission and run-ahead tokens are never emitted.

What changed is the step inside the graph: instead of the Inductor-compiled HF forward, the graph holds the
native step of Qwen3Engine (5 hand-written kernels per layer + lm_head/argmax, chained with programmatic
dependent launch), and the prompt runs through the engine's native prefill. The model must be a transformers
Qwen3 model quantised with efficientgpt_b200.quantize_model.
"""
import time

import torch

from .engine import Qwen3Engine


class GraphGreedyDecoder:
    """One CUDA graph per decode step; token and position live on the device."""

    def __init__(self, model, max_cache_len, lookahead=8, pdl=True, persistent=None):
        self.model, self.max_cache_len, self.lookahead = model, max_cache_len, lookahead
        self.engine = Qwen3Engine(model, max_cache_len, pdl=pdl, persistent=persistent)
        self.device = self.engine.device
        self.token = self.engine.token
        self.position = self.engine.position
        self.host = torch.empty(max_cache_len, dtype=torch.long, pin_memory=True)
        self.graph = None

    @torch.inference_mode()
    def _capture(self):
        eng = self.engine
        eng.reset()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):  # warm-up outside capture (loads the module, sets kernel attributes)
            for _ in range(3):
                eng.position.zero_()
                eng.step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            eng.step()
        eng.reset()

    @torch.inference_mode()
    def generate(self, input_ids, max_new_tokens, eos_ids=(), on_token=None):
        p = input_ids.shape[1]
        if input_ids.shape[0] != 1:
            raise ValueError('GraphGreedyDecoder supports batch size 1')
        if max_new_tokens < 1:
            raise ValueError('max_new_tokens must be >= 1')
        if p + max_new_tokens > self.max_cache_len:
            raise ValueError('prompt + max_new_tokens exceeds max_cache_len')
        capture_s = 0.0
        if self.graph is None:
            t = time.perf_counter()
            self._capture()
            capture_s = time.perf_counter() - t
        self.engine.reset()
        eos = set(eos_ids)
        t0 = time.perf_counter()
        self.engine.prefill(input_ids.to(self.device, non_blocking=True))
        events, out, emitted, first, launched, done = [], [], 0, None, 0, False
        while not done:
            self.host[launched:launched + 1].copy_(self.token.view(-1), non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            events.append(ev)
            launched += 1
            if launched < max_new_tokens:
                self.graph.replay()  # computes the next token into self.token
            while emitted < launched and (events[emitted].query() or launched - emitted > self.lookahead
                                          or launched >= max_new_tokens):
                events[emitted].synchronize()
                tok = int(self.host[emitted])
                if first is None:
                    first = time.perf_counter()
                out.append(tok)
                if on_token:
                    on_token(tok)
                emitted += 1
                if tok in eos:
                    done = True
                    break
            if launched >= max_new_tokens and emitted >= launched:
                done = True
        torch.cuda.synchronize()
        return out, {'ttft_s': first - t0, 'total_s': time.perf_counter() - t0, 'tokens': len(out),
                     'capture_s': capture_s}
