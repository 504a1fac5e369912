"""Qwen3 int8 decode in numpy, at the reference's eager bf16 rounding points (test infrastructure; see
oracle/__init__.py).

Restates the forward that BagelsFun/efficientgpt's GraphGreedyDecoder runs (research/realmodel/fast_decode.py:
45-49, 83-85) on transformers' Qwen3ForCausalLM (modeling_qwen3.py) with every nn.Linear replaced by the int8
op (research/realmodel/int8_linear.py:88-157):
  RMSNorm      modeling_qwen3.py:59-64   w * bf16(x * rsqrt(mean(x^2) + eps))
  RoPE         modeling_qwen3.py:137-148 cos/sin of inv_freq * pos in fp32, cast to bf16; :159-180 rotate-half
  attention    modeling_qwen3.py:258-291 q/k norm after the projections, RoPE, cache write, GQA SDPA, o_proj
               (SDPA with fp32 scores/softmax and bf16 probabilities into P.V, rounded per 128-key block of
               the reference GPU kernel's cache walk, see attn_ref.REF_KEY_BLOCK)
  MLP          modeling_qwen3.py:81-82   down(bf16(silu(gate)) * up)
  layer        modeling_qwen3.py:305-335 bf16 residual adds
  lm_head      modeling_qwen3.py:503-505 int8 op on the last row only, bf16 logits; argmax, first index on ties
"""
import numpy as np

from .attn_ref import REF_KEY_BLOCK, decode_attention_fp32
from .bf16 import from_torch, round_bf16
from .int8_ref import int8_linear, int8_matmul, quantize_weight


def rmsnorm(x, w, eps):
    x = np.asarray(x, np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    inv = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    return round_bf16(w * round_bf16(x * inv))


def default_inv_freq(d, theta):
    """modeling_qwen3.py:113-130 compute_default_rope_parameters: 1 / theta^(2i/d) in fp32."""
    exps = np.arange(0, d, 2, dtype=np.int64).astype(np.float32) / np.float32(d)
    return (np.float32(1.0) / np.power(np.float32(theta), exps).astype(np.float32)).astype(np.float32)


def rope_table(cap, inv_freq):
    """cos, sin [cap, d] as bf16 values (modeling_qwen3.py:137-148): freqs = inv_freq * pos in fp32, emb =
    cat(freqs, freqs), cos/sin in fp32, cast to bf16. inv_freq is the model's buffer as it is at run time:
    `model.to(torch.bfloat16)` also casts that buffer, so a bf16 model uses bf16-rounded frequencies."""
    inv_freq = np.asarray(inv_freq, np.float32)
    freqs = inv_freq[None, :] * np.arange(cap, dtype=np.float32)[:, None]
    emb = np.concatenate([freqs, freqs], axis=-1)
    return round_bf16(np.cos(emb)), round_bf16(np.sin(emb))


def apply_rope(x, cos, sin):
    """x [..., heads, d] with cos/sin [..., 1, d]: bf16(bf16(x*cos) + bf16(rotate_half(x)*sin))."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return round_bf16(round_bf16(x * cos) + round_bf16(rot * sin))


def silu(g):
    return g / (np.float32(1.0) + np.exp(-g))


class Qwen3Ref:
    """int8 Qwen3 decoder with a static KV cache of `cap` slots. Weights are quantised here by the oracle's own
    quantize_weight from the bf16 model; scale_dtype 'bf16' stores bf16(s) (BASELINE configs 2 and 5)."""

    def __init__(self, cfg, layers, embed, final_norm, lm_q, lm_s, cap):
        self.cfg = cfg
        self.layers = layers
        self.embed = embed
        self.final_norm = final_norm
        self.lm_q, self.lm_s = lm_q, lm_s
        self.cap = cap
        self.cos, self.sin = rope_table(cap, cfg['inv_freq'])
        nkv, d = cfg['n_kv_heads'], cfg['head_dim']
        self.k = np.zeros((len(layers), nkv, cap, d), np.float32)
        self.v = np.zeros((len(layers), nkv, cap, d), np.float32)

    @classmethod
    def from_hf(cls, model, cap, scale_dtype='fp32', semantics='cuda'):
        """Build from an (unquantised, bf16) transformers Qwen3ForCausalLM. `semantics` selects the quantiser's
        scalar-division behaviour ('cuda': the reference quantising on the GPU; 'cpu': on the host)."""
        c = model.config
        cfg = {'hidden': c.hidden_size, 'n_q_heads': c.num_attention_heads, 'n_kv_heads': c.num_key_value_heads,
               'head_dim': getattr(c, 'head_dim', c.hidden_size // c.num_attention_heads),
               'intermediate': c.intermediate_size, 'vocab': c.vocab_size, 'eps': c.rms_norm_eps,
               'inv_freq': from_torch(model.model.rotary_emb.inv_freq)}

        def quant(lin):
            q, s = quantize_weight(from_torch(lin.weight), semantics)
            return q, (round_bf16(s) if scale_dtype == 'bf16' else s)

        layers = []
        for blk in model.model.layers:
            a, m = blk.self_attn, blk.mlp
            layers.append({'q': quant(a.q_proj), 'k': quant(a.k_proj), 'v': quant(a.v_proj), 'o': quant(a.o_proj),
                           'gate': quant(m.gate_proj), 'up': quant(m.up_proj), 'down': quant(m.down_proj),
                           'ln_in': from_torch(blk.input_layernorm.weight),
                           'ln_post': from_torch(blk.post_attention_layernorm.weight),
                           'q_norm': from_torch(a.q_norm.weight), 'k_norm': from_torch(a.k_norm.weight)})
        lm_q, lm_s = quant(model.lm_head)
        return cls(cfg, layers, from_torch(model.model.embed_tokens.weight), from_torch(model.model.norm.weight),
                   lm_q, lm_s, cap)

    def forward(self, ids, pos0):
        """Rows `ids` at positions pos0.. (prefill when len(ids) > 1); returns the bf16 logits of the last row."""
        cfg = self.cfg
        nq, nkv, d, eps = cfg['n_q_heads'], cfg['n_kv_heads'], cfg['head_dim'], cfg['eps']
        ids = np.asarray(ids, np.int64)
        m = len(ids)
        if pos0 + m > self.cap:
            raise ValueError('prompt + new tokens exceed the cache')
        h = self.embed[ids]
        cos = self.cos[pos0:pos0 + m][:, None, :]
        sin = self.sin[pos0:pos0 + m][:, None, :]
        scale = d ** -0.5
        for li, L in enumerate(self.layers):
            x = rmsnorm(h, L['ln_in'], eps)
            q = int8_linear(x, *L['q']).reshape(m, nq, d)
            k = int8_linear(x, *L['k']).reshape(m, nkv, d)
            v = int8_linear(x, *L['v']).reshape(m, nkv, d)
            q = apply_rope(rmsnorm(q, L['q_norm'], eps), cos, sin)
            k = apply_rope(rmsnorm(k, L['k_norm'], eps), cos, sin)
            self.k[li, :, pos0:pos0 + m] = k.transpose(1, 0, 2)
            self.v[li, :, pos0:pos0 + m] = v.transpose(1, 0, 2)
            o = np.stack([decode_attention_fp32(q[i], self.k[li], self.v[li], pos0 + i + 1, scale, p_bf16=True,
                                                block=REF_KEY_BLOCK)
                          for i in range(m)])
            o = round_bf16(o).reshape(m, nq * d)
            h = round_bf16(h + int8_linear(o, *L['o']))
            x = rmsnorm(h, L['ln_post'], eps)
            g = int8_linear(x, *L['gate'])
            u = int8_linear(x, *L['up'])
            a = round_bf16(round_bf16(silu(g)) * u)
            h = round_bf16(h + int8_linear(a, *L['down']))
        hn = rmsnorm(h[-1:], self.final_norm, eps)
        return int8_matmul(hn, self.lm_q, self.lm_s)[0]

    def generate(self, prompt, n_new):
        """Greedy tokens and the bf16 logits of every step (reference GraphGreedyDecoder.generate semantics)."""
        prompt = [int(t) for t in prompt]
        logits = self.forward(prompt, 0)
        toks, all_logits = [], []
        pos = len(prompt)
        for i in range(n_new):
            tok = int(np.argmax(logits))
            toks.append(tok)
            all_logits.append(logits)
            if i == n_new - 1:
                break
            logits = self.forward([tok], pos)
            pos += 1
        return toks, all_logits
