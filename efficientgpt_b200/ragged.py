"""Ragged small-batch greedy decoding: up to 16 sequences of different prompt lengths decoded together.

Drop-in for the contract of BagelsFun/efficientgpt research/phase5/ragged.py (RaggedEngine / RaggedGraphDecoder,
there for nanoGPT) on the Qwen3 int8 path: right-padded prompts [B, Pmax] (pad values ignored) plus lengths [B] in
[1, Pmax]; the output is the generated tokens [B, count] only; row b writes generated token t at cache slot
lengths[b] + t and attends to slots <= its own position, so pad and stale K/V are never read. Capacity =
Pmax + count. Every row matches batch-1 greedy decoding under the near-tie rule (a GEMV over B rows is not
bit-identical to the batch-1 step, which uses the exact one-row kernel).

Per step, on the device (one CUDA graph per step in RaggedGraphDecoder): the B token embeddings, per layer RMSNorm
over the B rows, the q|k|v, o, gate|up (SiLU·up) and down (residual) projections over all B rows at once, so the
weights stream once per step for the whole batch (the point of small-batch decode, int8_linear.py:18
MAX_DECODE_ROWS): for 4..16 rows on the tcgen05 GEMM (egpt_gemm_i8_tc with one rounding, bf16(acc * s), K split
over several CTAs per weight tile, then the epilogue at the reference's rounding points), for fewer on the GEMV
kernel; one attention launch for the B
sequences (egpt_attn_decode with
EGPT_FLAG_RAGGED | EGPT_FLAG_APPEND: row b's q/k RMSNorm, RoPE at position[b] and K/V append into its own cache
heads, then its own causal range); the final norm, the lm_head projection over the B rows and a row-wise argmax.
Prompts are prefilled row by row on the same kernels in 16-row blocks.
"""
import torch

from . import _lib as L
from . import ops
from .engine import Qwen3Engine

MAX_ROWS = 16


def check_ragged(prompts, lengths, count, capacity):
    """The reference's request checks (research/phase5/ragged.py:24-30), plus the row limit of the GEMV."""
    if prompts.dim() != 2 or prompts.shape[0] < 1:
        raise ValueError('prompts must be [batch, Pmax]')
    if prompts.shape[0] > MAX_ROWS:
        raise ValueError(f'at most {MAX_ROWS} rows')
    if count < 1:
        raise ValueError('count must be >= 1')
    if lengths.shape != (prompts.size(0),) or lengths.dtype != torch.long:
        raise ValueError('lengths must be int64 [batch]')
    if int(lengths.min()) < 1 or int(lengths.max()) > prompts.size(1):
        raise ValueError('lengths must be in [1, prompts.size(1)]')
    if prompts.size(1) + count > capacity:
        raise ValueError('Pmax + count exceeds the capacity')


class RaggedEngine:
    """B sequences with per-row positions on the Qwen3 int8 kernels (weights fused once by Qwen3Engine)."""

    def __init__(self, model, batch, capacity, attn_max_split=8):
        if not 1 <= batch <= MAX_ROWS:
            raise ValueError(f'batch must be in [1, {MAX_ROWS}]')
        self.base = Qwen3Engine(model, capacity, step='sequence')
        b = self.base
        self.batch, self.cap, self.device = batch, capacity, b.device
        self.kv = torch.zeros(b.n_layers, 2, batch * b.nkv, capacity, b.d, dtype=torch.bfloat16, device=b.device)
        self.tokens = torch.zeros(batch, dtype=torch.long, device=b.device)
        self.positions = torch.zeros(batch, dtype=torch.long, device=b.device)
        self.max_split = attn_max_split
        self.attn_ws = ops.attn_ws(batch, b.nq, b.nkv, b.d, attn_max_split, b.device)
        self.logits = torch.empty(batch, b.vocab, dtype=torch.bfloat16, device=b.device)
        # 4..16 rows: the projections on the tcgen05 GEMM (one 128-row tile holds the batch, K split over several
        # CTAs per weight tile); fewer rows: the GEMV kernel. Measured on the config-2 model: B = 16 2.93 ms per
        # step on the GEMM against 10.43 on the GEMV; B = 4 3.22 ms on the GEMV; B = 1 1.83 ms on the GEMV
        dims = (b.hidden, b.inter, b.nq * b.d)
        self.use_gemm = batch >= 4 and all(k % 64 == 0 for k in dims)
        self.gemm_ws = {}  # fp32 split-K workspaces per (N, K), reused by every step (and by the captured graph)

    def _proj(self, x, w, s, epilogue=L.EPI_NONE, residual=None):
        """bf16(acc * s) over the batch rows, then the epilogue at the reference's rounding points."""
        if not self.use_gemm:
            return ops.gemv_i8(x, w, s, epilogue=epilogue, residual=residual)
        y = ops.gemm_i8_tc(x, w, s, double_round=False, ws=self._ws(w))
        if epilogue == L.EPI_RESIDUAL:
            return residual + y
        if epilogue == L.EPI_SILU_MUL:
            half = y.shape[1] // 2
            return torch.nn.functional.silu(y[:, :half]) * y[:, half:]
        return y

    def _ws(self, w):
        n, k = w.shape
        if (n, k) not in self.gemm_ws:
            need = int(L.load().egpt_gemm_i8_tc_ws_bytes(self.batch, n, k))
            self.gemm_ws[(n, k)] = torch.empty(max(need, 16), dtype=torch.uint8, device=self.device)
        return self.gemm_ws[(n, k)]

    def _row_kv(self, row):
        b = self.base
        return self.kv[:, :, row * b.nkv:(row + 1) * b.nkv]

    @torch.no_grad()
    def prefill_row(self, row, ids):
        """Prompt ids (int64 [p] on the device) of one row from position 0, on the 16-row-block kernels; leaves the
        row's first generated token and position p."""
        b = self.base
        kv = self._row_kv(row)
        p = ids.numel()
        pos0 = torch.zeros(1, dtype=torch.long, device=self.device)
        h = ops.embed(ids, b.embed)
        ws = ops.attn_ws(p, b.nq, b.nkv, b.d, self.max_split, self.device)
        for i, lay in enumerate(b.layers):
            x = ops.rmsnorm(h, lay['ln_in'], b.eps)
            qkv = b._linear(x, lay['w_qkv'], lay['s_qkv'])
            q = ops.qk_norm_rope_kv_append(qkv, kv[i, 0], kv[i, 1], pos0, b.nq, b.nkv, b.d, q_norm_w=lay['q_norm'],
                                           k_norm_w=lay['k_norm'], eps=b.eps, rope_cos=b.rope_cos,
                                           rope_sin=b.rope_sin)
            a = ops.attn_decode(q, kv[i, 0], kv[i, 1], pos0, b.nq, b.nkv, b.d, scale=b.scale,
                                max_split=self.max_split, ws=ws, ref_softmax=True)
            h = b._linear(a, lay['w_o'], lay['s_o'], epilogue=L.EPI_RESIDUAL, residual=h)
            x = ops.rmsnorm(h, lay['ln_post'], b.eps)
            act = b._linear(x, lay['w_gu'], lay['s_gu'], epilogue=L.EPI_SILU_MUL)
            h = b._linear(act, lay['w_down'], lay['s_down'], epilogue=L.EPI_RESIDUAL, residual=h)
        x = ops.rmsnorm(h[p - 1:p], b.final_norm, b.eps)
        logits = ops.gemv_i8(x, b.w_lm, b.s_lm)
        self.tokens[row:row + 1].copy_(ops.argmax_rows(logits))
        self.positions[row] = p

    @torch.no_grad()
    def step(self):
        """One token for every row: tokens <- argmax(model(tokens, positions)); positions += 1 (no host sync)."""
        b = self.base
        h = ops.embed(self.tokens, b.embed)
        for i, lay in enumerate(b.layers):
            x = ops.rmsnorm(h, lay['ln_in'], b.eps)
            qkv = self._proj(x, lay['w_qkv'], lay['s_qkv'])
            a = ops.attn_decode(qkv, self.kv[i, 0], self.kv[i, 1], self.positions, b.nq, b.nkv, b.d, scale=b.scale,
                                max_split=self.max_split, ws=self.attn_ws, append=True, ragged=True,
                                q_norm_w=lay['q_norm'], k_norm_w=lay['k_norm'], eps=b.eps, rope_cos=b.rope_cos,
                                rope_sin=b.rope_sin, ref_softmax=True)
            h = self._proj(a, lay['w_o'], lay['s_o'], epilogue=L.EPI_RESIDUAL, residual=h)
            x = ops.rmsnorm(h, lay['ln_post'], b.eps)
            act = self._proj(x, lay['w_gu'], lay['s_gu'], epilogue=L.EPI_SILU_MUL)
            h = self._proj(act, lay['w_down'], lay['s_down'], epilogue=L.EPI_RESIDUAL, residual=h)
        x = ops.rmsnorm(h, b.final_norm, b.eps)
        if self.use_gemm:
            ops.gemm_i8_tc(x, b.w_lm, b.s_lm, double_round=False, out=self.logits, ws=self._ws(b.w_lm))
        else:
            ops.gemv_i8(x, b.w_lm, b.s_lm, out=self.logits)
        self.tokens.copy_(ops.argmax_rows(self.logits))
        self.positions.add_(1)

    @torch.no_grad()
    def generate_eager(self, prompts, lengths, count):
        check_ragged(prompts, lengths, count, self.cap)
        if prompts.shape[0] != self.batch:
            raise ValueError('prompts must have the engine batch size')
        out = torch.empty(self.batch, count, dtype=torch.long, device=self.device)
        for r in range(self.batch):
            self.prefill_row(r, prompts[r, :int(lengths[r])].to(self.device))
        out[:, 0] = self.tokens
        for t in range(1, count):
            self.step()
            out[:, t] = self.tokens
        return out


class RaggedGraphDecoder:
    """RaggedEngine with the step captured once as a CUDA graph (the reference's RaggedGraphDecoder contract):
    generate(prompts, lengths, count) -> tokens [B, count] (int64, on the device)."""

    def __init__(self, model, batch, capacity):
        self.engine = RaggedEngine(model, batch, capacity)
        self.graph = None
        self.out = torch.zeros(batch, capacity, dtype=torch.long, device=self.engine.device)
        self.col = torch.zeros(1, dtype=torch.long, device=self.engine.device)

    def _capture(self):
        eng = self.engine
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up outside capture
            for _ in range(2):
                eng.positions.zero_()
                self._replay_body()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._replay_body()

    def _replay_body(self):
        self.engine.step()
        self.col.add_(1)
        self.out.index_copy_(1, self.col, self.engine.tokens.view(-1, 1))

    @torch.no_grad()
    def generate(self, prompts, lengths, count):
        eng = self.engine
        check_ragged(prompts, lengths, count, eng.cap)
        if prompts.shape[0] != eng.batch:
            raise ValueError('prompts must have the decoder batch size')
        if self.graph is None:
            self._capture()
        for r in range(eng.batch):
            eng.prefill_row(r, prompts[r, :int(lengths[r])].to(eng.device))
        self.col.zero_()
        self.out[:, 0] = eng.tokens
        for _ in range(count - 1):
            self.graph.replay()
        return self.out[:, :count].clone()
