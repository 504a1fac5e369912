"""The reference's CPU decode path, restated with torch CPU ops (test infrastructure / timed CPU baseline; see
oracle/__init__.py).

BagelsFun/efficientgpt's int8 path on a host without its Triton kernel is HF transformers' Qwen3 forward
(modeling_qwen3.py) in eager bf16 with every linear computed as the int8 op's arithmetic: <= 16 rows
bf16((x.float() @ q.float().T) * s), more rows bf16(bf16(x @ bf16(q).T) * s) (research/realmodel/int8_linear.py:
67-98; the "torch dequant-matmul decode" of the north star), a static KV cache, and argmax on the last row
(research/realmodel/fast_decode.py:45-49, 81-83). This module runs exactly that with torch's CPU kernels (eager
bf16 rounding, CPU SDPA), so that bench.py can time it on the box's host cores.

Two ways in:
  * cpu_model_weights(cfg, seed) builds the seeded transformers model ON THE CPU and quantises every linear with
    the reference's quantiser (int8_linear.py:106-117) in torch CPU ops: the reference arm of bench.py uses this
    and never imports the product package or loads its library;
  * TorchCpuQwen3.from_engine(engine) copies an already-quantised product engine's tensors to the host (the
    cpu_baseline of the product's own bench line, same weights as the timed GPU step).
"""
import torch
import torch.nn.functional as F

MAX_DECODE_ROWS = 16  # int8_linear.py:18


def qwen3_config(name):
    """BASELINE config 2 ('qwen3_1.7b') or config 5 ('qwen3_8b') as a transformers Qwen3Config."""
    from transformers import Qwen3Config
    common = dict(vocab_size=151936, head_dim=128, num_key_value_heads=8, max_position_embeddings=40960,
                  rope_theta=1e6, rms_norm_eps=1e-6, initializer_range=0.02)
    if name == 'qwen3_1.7b':
        return Qwen3Config(hidden_size=2048, intermediate_size=6144, num_hidden_layers=28, num_attention_heads=16,
                           tie_word_embeddings=True, **common)
    if name == 'qwen3_8b':
        return Qwen3Config(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36, num_attention_heads=32,
                           tie_word_embeddings=False, **common)
    raise ValueError(name)


def quantize_weight(w, semantics='cuda'):
    """int8_linear.py:106-117 in torch CPU ops: s = max(max|w| / 127, 1e-12) fp32 per row, q = clamp(rint(w / s)).
    semantics='cuda' evaluates max|w| / 127 as max|w| * fl32(1/127) (what PyTorch does on the GPU, where the
    reference quantises), 'cpu' as a true division. Rows in chunks of 8192 (elementwise per row: same bits)."""
    qs, ss = [], []
    inv = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(127.0, dtype=torch.float32)
    for r0 in range(0, w.shape[0], 8192):
        wf = w[r0:r0 + 8192].float()
        amax = wf.abs().amax(dim=1)
        s = (amax * inv if semantics == 'cuda' else amax / 127.0).clamp_min(1e-12)
        qs.append(torch.round(wf / s[:, None]).clamp_(-127, 127).to(torch.int8))
        ss.append(s)
    return torch.cat(qs), torch.cat(ss)


def cpu_model_weights(cfg, seed=0, scale_dtype=torch.bfloat16, cap=4096 + 512):
    """The seeded random-init transformers Qwen3 model built on the CPU (torch.manual_seed(seed), the model's own
    N(0, 0.02) init), cast to bf16, every linear (lm_head included, untied as quantize_model does) quantised;
    returns the weight dict TorchCpuQwen3 takes. RoPE tables from the model's own rotary embedding (bf16)."""
    from transformers import Qwen3ForCausalLM
    torch.manual_seed(seed)
    with torch.device('cpu'):
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    m = model.model
    d = cfg.head_dim

    def q8(lin):
        q, s = quantize_weight(lin.weight.detach())
        return q, s.to(scale_dtype)

    layers = []
    for lay in m.layers:
        a, mlp = lay.self_attn, lay.mlp
        layers.append({'q': q8(a.q_proj), 'k': q8(a.k_proj), 'v': q8(a.v_proj), 'o': q8(a.o_proj),
                       'gate': q8(mlp.gate_proj), 'up': q8(mlp.up_proj), 'down': q8(mlp.down_proj),
                       'ln_in': lay.input_layernorm.weight.detach().clone(),
                       'ln_post': lay.post_attention_layernorm.weight.detach().clone(),
                       'q_norm': a.q_norm.weight.detach().clone(), 'k_norm': a.k_norm.weight.detach().clone()})
    pos = torch.arange(cap).view(1, -1)
    cos, sin = m.rotary_emb(torch.zeros(1, dtype=torch.bfloat16), pos)
    w = {'nq': cfg.num_attention_heads, 'nkv': cfg.num_key_value_heads, 'd': d, 'eps': cfg.rms_norm_eps,
         'hidden': cfg.hidden_size, 'inter': cfg.intermediate_size, 'layers': layers,
         'embed': m.embed_tokens.weight.detach().clone(), 'final_norm': m.norm.weight.detach().clone(),
         'lm': q8(model.lm_head), 'cos': cos[0].to(torch.bfloat16), 'sin': sin[0].to(torch.bfloat16)}
    del model
    return w


def _linear(x, q, s):
    """The op (int8_linear.py:88-98) on the CPU: <= 16 rows the decode kernel's arithmetic, more rows the prefill's."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.shape[0] <= MAX_DECODE_ROWS:
        y = ((x2.float() @ q.float().t()) * s.float()).to(torch.bfloat16)
    else:
        y = ((x2 @ q.to(torch.bfloat16).t()).float() * s.float()).to(torch.bfloat16)
    return y.reshape(*x.shape[:-1], q.shape[0])


def _rmsnorm(x, w, eps):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * y.to(torch.bfloat16)


def _rope(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rot * sin


class TorchCpuQwen3:
    """Prefill and decode steps of a quantised Qwen3 on the CPU with a static KV cache of `cap` positions."""

    def __init__(self, weights, cap):
        self.w = weights
        self.nq, self.nkv, self.d, self.eps = weights['nq'], weights['nkv'], weights['d'], weights['eps']
        self.cap = cap
        self.cos, self.sin = weights['cos'][:cap], weights['sin'][:cap]
        if self.cos.shape[0] < cap:
            raise ValueError('RoPE tables shorter than the cache')
        nl = len(weights['layers'])
        self.k = torch.zeros(nl, 1, self.nkv, cap, self.d, dtype=torch.bfloat16)
        self.v = torch.zeros_like(self.k)

    @classmethod
    def from_engine(cls, engine, cap):
        """Weights of a product Qwen3Engine (already quantised on the GPU), copied to host memory."""
        cpu = torch.device('cpu')
        nq_rows, nkv_rows = engine.nq * engine.d, engine.nkv * engine.d
        layers = []
        for lay in engine.layers:
            w_qkv, s_qkv = lay['w_qkv'].to(cpu), lay['s_qkv'].to(cpu)
            w_gu, s_gu = lay['w_gu'].to(cpu), lay['s_gu'].to(cpu)
            layers.append({
                'q': (w_qkv[:nq_rows], s_qkv[:nq_rows]),
                'k': (w_qkv[nq_rows:nq_rows + nkv_rows], s_qkv[nq_rows:nq_rows + nkv_rows]),
                'v': (w_qkv[nq_rows + nkv_rows:], s_qkv[nq_rows + nkv_rows:]),
                'o': (lay['w_o'].to(cpu), lay['s_o'].to(cpu)),
                'gate': (w_gu[:engine.inter], s_gu[:engine.inter]), 'up': (w_gu[engine.inter:], s_gu[engine.inter:]),
                'down': (lay['w_down'].to(cpu), lay['s_down'].to(cpu)),
                'ln_in': lay['ln_in'].to(cpu), 'ln_post': lay['ln_post'].to(cpu),
                'q_norm': lay['q_norm'].to(cpu), 'k_norm': lay['k_norm'].to(cpu)})
        cos, sin = engine.rope_cos.to(cpu), engine.rope_sin.to(cpu)
        w = {'nq': engine.nq, 'nkv': engine.nkv, 'd': engine.d, 'eps': engine.eps, 'hidden': engine.hidden,
             'inter': engine.inter, 'layers': layers, 'embed': engine.embed.to(cpu),
             'final_norm': engine.final_norm.to(cpu), 'lm': (engine.w_lm.to(cpu), engine.s_lm.to(cpu)),
             'cos': torch.cat([cos, cos], -1), 'sin': torch.cat([sin, sin], -1)}
        return cls(w, cap)

    @torch.inference_mode()
    def forward(self, tokens, pos0):
        """Rows `tokens` (list of ids) at positions pos0.. through the model, KV written at those positions;
        attention over positions 0..p for row p (causal). Returns the next greedy token of the last row."""
        n = len(tokens)
        w = self.w
        h = w['embed'][torch.tensor(tokens)].view(1, n, -1)
        cos = self.cos[pos0:pos0 + n].view(1, 1, n, -1)
        sin = self.sin[pos0:pos0 + n].view(1, 1, n, -1)
        grp = self.nq // self.nkv
        end = pos0 + n
        for i, L in enumerate(w['layers']):
            x = _rmsnorm(h, L['ln_in'], self.eps)
            q = _rmsnorm(_linear(x, *L['q']).view(1, n, self.nq, self.d), L['q_norm'], self.eps).transpose(1, 2)
            k = _rmsnorm(_linear(x, *L['k']).view(1, n, self.nkv, self.d), L['k_norm'], self.eps).transpose(1, 2)
            v = _linear(x, *L['v']).view(1, n, self.nkv, self.d).transpose(1, 2)
            q, k = _rope(q, cos, sin), _rope(k, cos, sin)
            self.k[i, :, :, pos0:end] = k
            self.v[i, :, :, pos0:end] = v
            kk = self.k[i, :, :, :end].repeat_interleave(grp, 1)
            vv = self.v[i, :, :, :end].repeat_interleave(grp, 1)
            mask = None
            if n > 1:  # row r sees positions <= pos0 + r
                mask = torch.arange(end).view(1, -1) <= (pos0 + torch.arange(n)).view(-1, 1)
            a = F.scaled_dot_product_attention(q, kk, vv, attn_mask=mask, scale=self.d ** -0.5)
            h = h + _linear(a.transpose(1, 2).reshape(1, n, -1), *L['o'])
            x = _rmsnorm(h, L['ln_post'], self.eps)
            h = h + _linear(F.silu(_linear(x, *L['gate'])) * _linear(x, *L['up']), *L['down'])
        logits = _linear(_rmsnorm(h[:, -1:], w['final_norm'], self.eps), *w['lm'])
        return int(logits.reshape(-1).argmax())

    def prefill(self, tokens):
        """The prompt at positions 0..len-1 (one pass: the op's > 16-row branch for prompts longer than 16)."""
        return self.forward(list(tokens), 0)

    def step(self, token, pos):
        """One decode token at position `pos`; returns the next greedy token id."""
        return self.forward([int(token)], pos)
