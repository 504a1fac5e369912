"""nanoGPT int8 decode in numpy (test infrastructure; see oracle/__init__.py).

Restates research/phase4/decoder.py reference_step (11-42) on the reference's GPT (model.py:18-108) with every
Linear quantised by research/realmodel/int8_linear.py quantize_weight (106-117) and evaluated, as BASELINE config 1
specifies for fp32 activations, as the torch dequant matmul x @ (q.float() * s[:, None]).T + b:
  LayerNorm   model.py:18-27   F.layer_norm(x, w, b, eps 1e-5): (x - mean) / sqrt(biased var + eps) * w + b
  attention   model.py:29-76   q, k, v = c_attn(x).split; SDPA (scale d^-0.5, causal); c_proj
  MLP         model.py:78-92   c_proj(GELU(c_fc(x))), GELU = 0.5 x (1 + erf(x / sqrt 2)) (nn.GELU())
  block       model.py:94-107  x + attn(ln_1(x)); x + mlp(ln_2(x))
  embedding   model.py:176-180 wte[ids] + wpe[pos]; lm_head on ln_f of the last row (decoder.py:41)
All arithmetic is fp32.
"""
import numpy as np
from scipy.special import erf

from .int8_ref import quantize_weight

LINEARS = ('attn.c_attn', 'attn.c_proj', 'mlp.c_fc', 'mlp.c_proj')


def layernorm(x, w, b, eps=1e-5):
    x = np.asarray(x, np.float32)
    mu = x.mean(-1, keepdims=True, dtype=np.float32)
    var = ((x - mu) ** 2).mean(-1, keepdims=True, dtype=np.float32)
    y = (x - mu) / np.sqrt(var + np.float32(eps)) * w
    return (y + b if b is not None else y).astype(np.float32)


def gelu(x):
    return (np.float32(0.5) * x * (np.float32(1.0) + erf(x / np.float32(np.sqrt(2.0))).astype(np.float32))).astype(np.float32)


def linear(x, q, s, b):
    y = np.asarray(x, np.float32) @ (q.astype(np.float32) * s[:, None]).T
    return (y + b if b is not None else y).astype(np.float32)


class NanoGPTRef:
    """int8 nanoGPT with a static K/V cache of block_size slots, batch 1."""

    def __init__(self, params, cfg, semantics='cpu'):
        self.cfg = cfg
        C, H = cfg['n_embd'], cfg['n_head']
        self.H, self.d = H, C // H

        def get(name):
            return np.asarray(params[name], np.float32) if name in params else None

        def quant(name):
            q, s = quantize_weight(get(name + '.weight'), semantics)
            return q, s, get(name + '.bias')
        self.wte, self.wpe = get('transformer.wte.weight'), get('transformer.wpe.weight')
        self.layers = []
        for i in range(cfg['n_layer']):
            pre = f'transformer.h.{i}.'
            self.layers.append({'ln_1': (get(pre + 'ln_1.weight'), get(pre + 'ln_1.bias')),
                                'ln_2': (get(pre + 'ln_2.weight'), get(pre + 'ln_2.bias')),
                                **{n: quant(pre + n) for n in LINEARS}})
        self.ln_f = (get('transformer.ln_f.weight'), get('transformer.ln_f.bias'))
        lm = get('lm_head.weight') if 'lm_head.weight' in params else self.wte
        self.lm_q, self.lm_s = quantize_weight(lm, semantics)
        T = cfg['block_size']
        self.k = np.zeros((cfg['n_layer'], H, T, self.d), np.float32)
        self.v = np.zeros_like(self.k)

    def forward(self, ids, pos0):
        """Rows `ids` at positions pos0..; returns the fp32 logits of the last row."""
        ids = np.asarray(ids, np.int64)
        m = len(ids)
        if pos0 + m > self.cfg['block_size']:
            raise ValueError('Prompt + output exceeds model context window')
        x = (self.wte[ids] + self.wpe[pos0:pos0 + m]).astype(np.float32)
        C, H, d = self.cfg['n_embd'], self.H, self.d
        for li, Lr in enumerate(self.layers):
            hn = layernorm(x, *Lr['ln_1'])
            qkv = linear(hn, *Lr['attn.c_attn'])
            q, k, v = (qkv[:, i * C:(i + 1) * C].reshape(m, H, d) for i in range(3))
            self.k[li, :, pos0:pos0 + m] = k.transpose(1, 0, 2)
            self.v[li, :, pos0:pos0 + m] = v.transpose(1, 0, 2)
            y = np.empty((m, H, d), np.float32)
            for r in range(m):
                n = pos0 + r + 1
                for h in range(H):
                    sc = (self.k[li, h, :n] @ q[r, h]) * np.float32(d ** -0.5)
                    p = np.exp(sc - sc.max())
                    y[r, h] = (p @ self.v[li, h, :n]) / p.sum(dtype=np.float32)
            x = (x + linear(y.reshape(m, C), *Lr['attn.c_proj'])).astype(np.float32)
            hn = layernorm(x, *Lr['ln_2'])
            x = (x + linear(gelu(linear(hn, *Lr['mlp.c_fc'])), *Lr['mlp.c_proj'])).astype(np.float32)
        hl = layernorm(x[-1:], *self.ln_f)
        return linear(hl, self.lm_q, self.lm_s, None)[0]

    def generate(self, prompt, count):
        """Greedy decode (decoder.py:45-55): returns (tokens, top-2 margins)."""
        lg = self.forward(prompt, 0)
        pos = len(prompt)
        toks, margins = [], []
        for i in range(count):
            top = np.sort(lg)[-2:]
            margins.append(float(top[1] - top[0]))
            t = int(np.argmax(lg))
            toks.append(t)
            if i != count - 1:
                lg = self.forward([t], pos)
                pos += 1
        return toks, margins
