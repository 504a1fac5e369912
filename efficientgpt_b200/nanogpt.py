"""nanoGPT-architecture int8 decode on the native kernels.

Mirrors the reference's static-KV decoder for its nanoGPT model (research/phase4/decoder.py: StaticKVDecoder
reset/step/finish/generate_eager at 75-163, GraphDecoder at 166-210) for models quantised with
`efficientgpt_b200.quantize_model` (int8 per-row weights, fp32 scales, fp32 activations). The reference's int8 op
refuses fp32 activations (research/realmodel/int8_linear.py:92-93), so its config-1 path is the torch dequant matmul
x @ (q.float() * s[:, None]).T + b; here every linear is egpt_gemv_i8 on fp32 x (bias and residual / erf-GELU fused
into the epilogue), LayerNorm is egpt_layernorm_f32, attention is the fp32 path of egpt_attn_decode, and the lm_head
with its greedy argmax (position += 1) is egpt_lm_head_argmax. Batch 1 only.

`GPT` / `GPTConfig` here are a minimal module with the reference model's attribute names (model.py:18-150:
transformer.wte / wpe / h[i].ln_1, attn.c_attn, attn.c_proj, ln_2, mlp.c_fc, mlp.c_proj / ln_f, lm_head tied to
wte), so the decoder accepts either the reference's GPT or this one.
"""
import math
from dataclasses import dataclass

import torch
from torch import nn

from . import _lib as L
from . import ops
from .int8_linear import Int8Linear


@dataclass
class GPTConfig:
    block_size: int = 1024
    vocab_size: int = 50304
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    dropout: float = 0.0
    bias: bool = True


class _LayerNorm(nn.Module):
    def __init__(self, n, bias):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n))
        self.bias = nn.Parameter(torch.zeros(n)) if bias else None


class _Attention(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.c_attn = nn.Linear(c.n_embd, 3 * c.n_embd, bias=c.bias)
        self.c_proj = nn.Linear(c.n_embd, c.n_embd, bias=c.bias)
        self.n_head = c.n_head


class _MLP(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.c_fc = nn.Linear(c.n_embd, 4 * c.n_embd, bias=c.bias)
        self.c_proj = nn.Linear(4 * c.n_embd, c.n_embd, bias=c.bias)


class _Block(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.ln_1 = _LayerNorm(c.n_embd, c.bias)
        self.attn = _Attention(c)
        self.ln_2 = _LayerNorm(c.n_embd, c.bias)
        self.mlp = _MLP(c)


class GPT(nn.Module):
    """Parameters of a nanoGPT model (no training code). Random init: N(0, 0.02) weights, zero biases, residual
    projections N(0, 0.02 / sqrt(2 n_layer)) (the GPT-2 scheme of the reference's model.py), drawn from `seed`."""

    def __init__(self, config, seed=0):
        super().__init__()
        self.config = config
        c = config
        self.transformer = nn.ModuleDict(dict(
            wte=nn.Embedding(c.vocab_size, c.n_embd), wpe=nn.Embedding(c.block_size, c.n_embd),
            h=nn.ModuleList([_Block(c) for _ in range(c.n_layer)]), ln_f=_LayerNorm(c.n_embd, c.bias)))
        self.lm_head = nn.Linear(c.n_embd, c.vocab_size, bias=False)
        self.transformer.wte.weight = self.lm_head.weight
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if name.endswith('.bias'):
                    p.zero_()
                elif '.ln_' in name or name.startswith('transformer.ln_f'):
                    p.fill_(1.0)
                else:
                    std = 0.02 / math.sqrt(2 * c.n_layer) if name.endswith('c_proj.weight') else 0.02
                    p.copy_(torch.randn(p.shape, generator=g) * std)

    @torch.no_grad()
    def load_params(self, params):
        """Copy a {name: array} state (e.g. a fixture of the reference model) into the parameters."""
        for name, p in self.named_parameters():
            p.copy_(torch.as_tensor(params[name]).to(p.dtype))
        return self


def _check_request(model, prompt, count):
    """research/phase4/decoder.py:62-71."""
    if count < 1 or prompt.ndim != 2 or prompt.size(1) < 1:
        raise ValueError('Need nonempty rank-2 prompt and >=1 output token')
    if prompt.size(1) + count > model.config.block_size:
        raise ValueError('Prompt + output exceeds context window; sliding window is not supported')
    if prompt.dtype != torch.long or prompt.device != next(model.parameters()).device:
        raise ValueError('Prompt must use int64 indices on model device')
    if model.training:
        raise ValueError('Model must be in eval() mode')


class NanoGPTEngine:
    """Static-KV int8 decode state of one nanoGPT model on the device (batch 1)."""

    def __init__(self, model, keep_logits=False):
        if not torch.cuda.is_available():
            raise RuntimeError('NanoGPTEngine needs a CUDA device (there is no CPU path)')
        c = model.config
        tr = model.transformer
        self.model = model
        self.device = tr.wte.weight.device
        if self.device.type != 'cuda':
            raise ValueError('the model must be on a CUDA device')
        if tr.wte.weight.dtype != torch.float32:
            raise ValueError('nanoGPT decode runs fp32 activations: keep the model in fp32')
        self.C, self.H, self.cap, self.V, self.n_layer = c.n_embd, c.n_head, c.block_size, c.vocab_size, c.n_layer
        self.d = self.C // self.H
        self.layers = []
        for blk in tr.h:
            lins = (blk.attn.c_attn, blk.attn.c_proj, blk.mlp.c_fc, blk.mlp.c_proj)
            if not all(isinstance(x, Int8Linear) for x in lins):
                raise ValueError('NanoGPTEngine needs a model quantised with efficientgpt_b200.quantize_model')
            if any(x.scale.dtype != torch.float32 for x in lins):
                raise ValueError('nanoGPT uses fp32 scales')
            self.layers.append({
                'ln1': (blk.ln_1.weight, blk.ln_1.bias), 'ln2': (blk.ln_2.weight, blk.ln_2.bias),
                'attn': lins[0], 'proj': lins[1], 'fc': lins[2], 'mproj': lins[3]})
        if not isinstance(model.lm_head, Int8Linear):
            raise ValueError('lm_head must be quantised (quantize_model(include_lm_head=True))')
        self.wte, self.wpe = tr.wte.weight, tr.wpe.weight
        self.ln_f = (tr.ln_f.weight, tr.ln_f.bias)
        self.lm = model.lm_head
        dev, f32 = self.device, torch.float32
        self.kv = torch.zeros((self.n_layer, 2, self.H, self.cap, self.d), dtype=f32, device=dev)
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.position = torch.zeros(1, dtype=torch.int64, device=dev)
        self.x = torch.zeros((1, self.C), dtype=f32, device=dev)
        self.hn = torch.zeros((1, self.C), dtype=f32, device=dev)
        self.qkv = torch.zeros((1, 3 * self.C), dtype=f32, device=dev)
        self.q = torch.zeros((1, self.C), dtype=f32, device=dev)
        self.y = torch.zeros((1, self.C), dtype=f32, device=dev)
        self.m = torch.zeros((1, 4 * self.C), dtype=f32, device=dev)
        self.logits = torch.zeros(self.V, dtype=f32, device=dev) if keep_logits else None
        self.lm_ws = ops.lm_head_ws(self.V, dev)
        self.attn_ws = ops.attn_ws(1, self.H, self.H, self.d, 1, dev)

    def _linear(self, x, lin, **kw):
        return ops.gemv_i8_rows(x, lin.qweight, lin.scale, bias=lin.bias, double_round=False, **kw)

    def _block(self, lay, x, hn, q_rows):
        """One transformer block over rows x (in place); q_rows: rows of the query buffer to use."""
        rows = x.shape[0]
        ops.layernorm_f32(x, *lay['ln1'], 1e-5, out=hn)
        qkv = self._linear(hn, lay['attn'], out=self.qkv if rows == 1 else None)
        q = ops.qk_norm_rope_kv_append(qkv, self.kv[lay['i'], 0], self.kv[lay['i'], 1], self.position, self.H,
                                       self.H, self.d, q_out=q_rows)
        y = ops.attn_decode(q, self.kv[lay['i'], 0], self.kv[lay['i'], 1], self.position, self.H, self.H, self.d,
                            scale=self.d ** -0.5, max_split=1, ws=self.attn_ws if rows == 1 else None,
                            out=self.y if rows == 1 else None)
        self._linear(y, lay['proj'], epilogue=L.EPI_RESIDUAL, residual=x)
        ops.layernorm_f32(x, *lay['ln2'], 1e-5, out=hn)
        m = self._linear(hn, lay['fc'], epilogue=L.EPI_GELU, out=self.m if rows == 1 else None)
        self._linear(m, lay['mproj'], epilogue=L.EPI_RESIDUAL, residual=x)

    @torch.no_grad()
    def step(self):
        """One token at *position from *token (device state): writes the next token and position + 1."""
        ops.embed(self.token, self.wte, pos_table=self.wpe, out=self.x, position=self.position)
        for i, lay in enumerate(self.layers):
            lay['i'] = i
            self._block(lay, self.x, self.hn, self.q)
        ops.layernorm_f32(self.x, *self.ln_f, 1e-5, out=self.hn)
        ops.lm_head_argmax(self.hn[0], self.lm.qweight, self.lm.scale, self.lm_ws, logits=self.logits,
                           token=self.token, position=self.position, advance=True)

    @torch.no_grad()
    def prefill(self, ids):
        """Rows of the prompt from position 0 (research/phase4/decoder.py:11-42 reference_step on the prompt):
        fills the caches, leaves token = first generated id and position = p."""
        ids = ids.reshape(-1).to(device=self.device, dtype=torch.int64).contiguous()
        p = ids.numel()
        if p < 1 or p > self.cap:
            raise ValueError('prompt length must be in [1, block_size]')
        self.position.zero_()
        x = ops.embed(ids, self.wte, pos_table=self.wpe)
        hn = torch.empty_like(x)
        for i, lay in enumerate(self.layers):
            lay['i'] = i
            self._block(lay, x, hn, None)
        ops.layernorm_f32(x[p - 1:p], *self.ln_f, 1e-5, out=self.hn)
        ops.lm_head_argmax(self.hn[0], self.lm.qweight, self.lm.scale, self.lm_ws, logits=self.logits,
                           token=self.token)
        self.position.fill_(p)
        return self.token


class StaticKVDecoder:
    """research/phase4/decoder.py:75-163 for batch 1 on the native kernels: reset(prompt) -> first logits (when kept)
    and token; step() advances one token on the device; finish(count) -> [1, p + count] history."""

    def __init__(self, model, batch=1, keep_logits=False):
        if model.training:
            raise ValueError('Call model.eval() before constructing decoder')
        if batch != 1:
            raise ValueError('the native nanoGPT decoder is batch 1')
        self.model = model
        self.batch = batch
        self.engine = NanoGPTEngine(model, keep_logits=keep_logits)
        self.limit = model.config.block_size
        self.history = torch.zeros((1, self.limit), dtype=torch.long, device=self.engine.device)
        self.prompt_len = None

    @torch.no_grad()
    def reset(self, prompt):
        if prompt.shape[0] != self.batch:
            raise ValueError('Decoder batch size is fixed')
        if prompt.size(1) >= self.limit:
            raise ValueError('Need room for at least one output token')
        _check_request(self.model, prompt, 1)
        self.engine.prefill(prompt)
        p = prompt.size(1)
        self.history[:, :p].copy_(prompt)
        self.prompt_len = p
        return self.engine.logits

    @torch.no_grad()
    def step(self):
        e = self.engine
        self.history.index_copy_(1, e.position, e.token.view(1, 1))  # history[pos] = token, on the device
        e.step()

    @torch.no_grad()
    def finish(self, count):
        if self.prompt_len is None:
            raise ValueError('Call reset first')
        p = self.prompt_len
        if p + count > self.limit:
            raise ValueError('Exceeded context window')
        self.history[:, p + count - 1:p + count].copy_(self.engine.token.view(1, 1))
        return self.history[:, :p + count].clone()

    @torch.no_grad()
    def generate_eager(self, prompt, count):
        _check_request(self.model, prompt, count)
        self.reset(prompt)
        for _ in range(count - 1):
            self.step()
        return self.finish(count)


class GraphDecoder:
    """research/phase4/decoder.py:166-210: one captured recurrent step (CUDA graph), replayed count - 1 times."""

    def __init__(self, model, prompt):
        if prompt.device.type != 'cuda':
            raise ValueError('CUDA Graphs require a CUDA device')
        self.engine = StaticKVDecoder(model, prompt.size(0))
        self.graph = None
        self._capture(prompt)

    @torch.no_grad()
    def _capture(self, prompt):
        eng = self.engine
        s = torch.cuda.Stream(device=prompt.device)
        s.wait_stream(torch.cuda.current_stream(prompt.device))
        with torch.cuda.stream(s):
            for _ in range(3):
                eng.reset(prompt)
                eng.step()
        torch.cuda.current_stream(prompt.device).wait_stream(s)
        eng.reset(prompt)
        torch.cuda.synchronize(prompt.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            eng.step()
        torch.cuda.synchronize(prompt.device)
        eng.reset(prompt)

    @torch.no_grad()
    def generate(self, prompt, count):
        _check_request(self.engine.model, prompt, count)
        self.engine.reset(prompt)
        for _ in range(count - 1):
            self.graph.replay()
        return self.engine.finish(count)
