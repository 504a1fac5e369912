"""Sync-free greedy decoding with one CUDA graph per token, on the native B200 decode step.

Drop-in for BagelsFun/efficientgpt research/realmodel/fast_decode.py:25-111 GraphGreedyDecoder: same constructor
(model, max_cache_len, lookahead=8), same `generate(input_ids, max_new_tokens, eos_ids=(), on_token=None) ->
(tokens, {'ttft_s', 'total_s', 'tokens', 'capture_s'})`, the same errors (batch 1, max_new_tokens >= 1, prompt + new
tokens <= max_cache_len) and the same streaming contract: the device runs at most `lookahead` tokens ahead of the
host, tokens reach `on_token` in order as soon as their step has finished, EOS stops the stream and tokens computed
past it are never emitted.

The step inside the graph is Qwen3Engine's native step: by default ONE cooperative kernel per token
(egpt_decode_step_dataflow: every layer, the lm_head and the argmax, reading token and position from device
memory and writing the next ones); shapes that kernel does not cover take egpt_decode_step_persistent or the
per-stage launch sequence (egpt_decode_step). The prompt runs through the engine's native prefill. The model must be a transformers
Qwen3 model quantised with efficientgpt_b200.quantize_model.

Host side: a fixed ring of lookahead + 1 pinned int64 slots, each with one reusable CUDA event. Step i's token is
copied into slot i mod R and the slot's event recorded; the next replay is launched before the host looks at any
slot, so the GPU never waits for Python. A slot is rewritten only after the token it held was emitted (at most
`lookahead` steps are pending when a new one is issued).
"""
import collections
import time

import torch

from .engine import Qwen3Engine


class GraphGreedyDecoder:
    """One CUDA graph per decode step; token and position live on the device."""

    def __init__(self, model, max_cache_len, lookahead=8, pdl=True, persistent=None, step=None, keep_logits=False):
        if lookahead < 0:
            raise ValueError('lookahead must be >= 0')
        self.model, self.max_cache_len, self.lookahead = model, max_cache_len, lookahead
        self.engine = Qwen3Engine(model, max_cache_len, pdl=pdl, persistent=persistent, step=step,
                                  keep_logits=keep_logits)
        self.device = self.engine.device
        self.token = self.engine.token
        self.position = self.engine.position
        self.ring_size = lookahead + 1
        self.ring = torch.zeros(self.ring_size, dtype=torch.long, pin_memory=True)
        self.ring_events = [torch.cuda.Event() for _ in range(self.ring_size)]
        self.graph = None

    @torch.inference_mode()
    def _capture(self):
        eng = self.engine
        eng.reset()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up outside capture (loads the library, sets kernel attributes)
            for _ in range(3):
                eng.position.zero_()
                self._step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        eng.reset()

    def _step(self):
        """The work of one graph replay: the next token from the current one."""
        self.engine.step()

    def _first(self):
        """After the prefill: step 0's token is on the device (greedy: the prefill's argmax)."""

    def _check(self, input_ids, max_new_tokens):
        if input_ids.dim() != 2 or input_ids.shape[0] != 1:
            raise ValueError('GraphGreedyDecoder supports batch size 1')
        if max_new_tokens < 1:
            raise ValueError('max_new_tokens must be >= 1')
        if input_ids.shape[1] + max_new_tokens > self.max_cache_len:
            raise ValueError('prompt + max_new_tokens exceeds max_cache_len')

    def _publish(self, step):
        """Queue step's token (on the device now) into its ring slot and mark the slot with its event."""
        slot = step % self.ring_size
        self.ring[slot:slot + 1].copy_(self.token.view(-1), non_blocking=True)
        self.ring_events[slot].record()

    def _read(self, step):
        slot = step % self.ring_size
        self.ring_events[slot].synchronize()
        return int(self.ring[slot])

    @torch.inference_mode()
    def generate(self, input_ids, max_new_tokens, eos_ids=(), on_token=None):
        self._check(input_ids, max_new_tokens)
        capture_s = 0.0
        if self.graph is None:
            t = time.perf_counter()
            self._capture()
            capture_s = time.perf_counter() - t  # reported on its own, outside the time to first token
        self.engine.reset()
        stop = frozenset(eos_ids)
        tokens, first_at = [], None
        pending = collections.deque()  # steps whose token is queued but not yet emitted, oldest first
        t0 = time.perf_counter()
        self.engine.prefill(input_ids.to(self.device, non_blocking=True))  # leaves step 0's token on the device
        self._first()

        def emit(step):
            nonlocal first_at
            tok = self._read(step)
            if first_at is None:
                first_at = time.perf_counter()
            tokens.append(tok)
            if on_token:
                on_token(tok)
            return tok in stop

        finished = False
        for step in range(max_new_tokens):
            self._publish(step)
            pending.append(step)
            if step + 1 < max_new_tokens:
                self.graph.replay()  # step + 1's token, computed while the host emits
            # emit every finished step; block on the oldest once the device is `lookahead` steps ahead
            while pending and (len(pending) > self.lookahead or self.ring_events[pending[0] % self.ring_size].query()):
                if emit(pending.popleft()):
                    finished = True
                    break
            if finished:
                break
        while not finished and pending:
            finished = emit(pending.popleft())
        torch.cuda.synchronize()
        return tokens, {'ttft_s': first_at - t0, 'total_s': time.perf_counter() - t0, 'tokens': len(tokens),
                        'capture_s': capture_s}


class SampledGraphDecoder(GraphGreedyDecoder):
    """Stochastic decoding in the same graph loop: each replay runs the native step with its logits kept, then draws
    the next token on the device (efficientgpt_b200.sampling: temperature -> top-k -> top-p -> inverse CDF) from the
    caller's pre-drawn uniforms, one per generated token, the contract of research/phase5/sampling.py:133-152
    (SampledGraphDecoder) and SampledEngine.reset/step (103-124): token 0 from the prompt's last logits with u[0],
    token i with u[i]. generate(input_ids, max_new_tokens, uniforms, eos_ids=(), on_token=None), uniforms float32
    [1, >= max_new_tokens] (e.g. sampling.draw_uniforms); otherwise as GraphGreedyDecoder."""

    def __init__(self, model, max_cache_len, cfg, lookahead=8, pdl=True, step=None):
        from .sampling import sample_ws
        super().__init__(model, max_cache_len, lookahead=lookahead, pdl=pdl, step=step, keep_logits=True)
        self.cfg = cfg
        self.uniforms = torch.zeros(1, max_cache_len, dtype=torch.float32, device=self.device)
        self.u_index = torch.zeros((), dtype=torch.int64, device=self.device)
        self.ws = sample_ws(1, self.device)

    def _draw(self):
        from .sampling import sample
        eng = self.engine
        sample(eng.logits.view(1, -1), self.cfg, self.uniforms, out=eng.token.view(1, 1), ws=self.ws,
               u_index=self.u_index)

    def _step(self):
        self.engine.step()
        self._draw()

    def _first(self):
        self.u_index.zero_()
        self._draw()

    def generate(self, input_ids, max_new_tokens, uniforms, eos_ids=(), on_token=None):
        self._check(input_ids, max_new_tokens)
        if uniforms.dim() != 2 or uniforms.shape[0] != 1 or uniforms.shape[1] < max_new_tokens or \
                uniforms.dtype != torch.float32:
            raise ValueError('uniforms must be float32 [batch, >= count]')
        self.uniforms[:, :max_new_tokens].copy_(uniforms[:, :max_new_tokens], non_blocking=True)
        return super().generate(input_ids, max_new_tokens, eos_ids=eos_ids, on_token=on_token)
