"""The reference's CPU decode path, restated with torch CPU ops (test infrastructure / timed CPU baseline; see
oracle/__init__.py).

BagelsFun/efficientgpt's int8 path on a host without its Triton kernel is HF transformers' Qwen3 forward
(modeling_qwen3.py) in eager bf16 with every linear computed as the int8 op's arithmetic
bf16((x.float() @ q.float().T) * s) (research/realmodel/int8_linear.py:67-98; the survey's "torch dequant-matmul
decode"), a static KV cache, and argmax on the last row (research/realmodel/fast_decode.py:45-49). This module
runs exactly that per decode token with torch's CPU kernels (eager bf16 rounding, CPU SDPA) on weights copied
from an already-quantised model, so that bench.py can time it on the box's host cores.
"""
import torch
import torch.nn.functional as F


def _linear(x, q, s):
    return ((x.float() @ q.float().t()) * s.float()).to(torch.bfloat16)


def _rmsnorm(x, w, eps):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * y.to(torch.bfloat16)


def _rope(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rot * sin


class TorchCpuQwen3:
    """Decode steps of a Qwen3Engine's quantised weights on the CPU. `engine` is an efficientgpt_b200
    Qwen3Engine (its tensors are copied to host memory once)."""

    def __init__(self, engine, cap):
        cpu = torch.device('cpu')
        self.nq, self.nkv, self.d, self.eps = engine.nq, engine.nkv, engine.d, engine.eps
        self.h_dim, self.inter = engine.hidden, engine.inter
        self.layers = []
        nq_rows, nkv_rows = self.nq * self.d, self.nkv * self.d
        for lay in engine.layers:
            w_qkv, s_qkv = lay['w_qkv'].to(cpu), lay['s_qkv'].to(cpu)
            w_gu, s_gu = lay['w_gu'].to(cpu), lay['s_gu'].to(cpu)
            self.layers.append({
                'q': (w_qkv[:nq_rows], s_qkv[:nq_rows]),
                'k': (w_qkv[nq_rows:nq_rows + nkv_rows], s_qkv[nq_rows:nq_rows + nkv_rows]),
                'v': (w_qkv[nq_rows + nkv_rows:], s_qkv[nq_rows + nkv_rows:]),
                'o': (lay['w_o'].to(cpu), lay['s_o'].to(cpu)),
                'gate': (w_gu[:self.inter], s_gu[:self.inter]), 'up': (w_gu[self.inter:], s_gu[self.inter:]),
                'down': (lay['w_down'].to(cpu), lay['s_down'].to(cpu)),
                'ln_in': lay['ln_in'].to(cpu), 'ln_post': lay['ln_post'].to(cpu),
                'q_norm': lay['q_norm'].to(cpu), 'k_norm': lay['k_norm'].to(cpu)})
        self.embed = engine.embed.to(cpu)
        self.final_norm = engine.final_norm.to(cpu)
        self.lm = (engine.w_lm.to(cpu), engine.s_lm.to(cpu))
        cos, sin = engine.rope_cos.to(cpu), engine.rope_sin.to(cpu)
        self.cos, self.sin = torch.cat([cos, cos], -1), torch.cat([sin, sin], -1)
        self.cap = cap
        self.k = torch.zeros(len(self.layers), 1, self.nkv, cap, self.d, dtype=torch.bfloat16)
        self.v = torch.zeros_like(self.k)

    @torch.inference_mode()
    def step(self, token, pos):
        """One decode token at position `pos`; returns the next greedy token id."""
        h = self.embed[token].view(1, 1, -1)
        cos, sin = self.cos[pos].view(1, 1, 1, -1), self.sin[pos].view(1, 1, 1, -1)
        grp = self.nq // self.nkv
        for i, L in enumerate(self.layers):
            x = _rmsnorm(h, L['ln_in'], self.eps)
            q = _rmsnorm(_linear(x, *L['q']).view(1, 1, self.nq, self.d), L['q_norm'], self.eps).transpose(1, 2)
            k = _rmsnorm(_linear(x, *L['k']).view(1, 1, self.nkv, self.d), L['k_norm'], self.eps).transpose(1, 2)
            v = _linear(x, *L['v']).view(1, 1, self.nkv, self.d).transpose(1, 2)
            q, k = _rope(q, cos, sin), _rope(k, cos, sin)
            self.k[i, :, :, pos] = k[:, :, 0]
            self.v[i, :, :, pos] = v[:, :, 0]
            kk = self.k[i, :, :, :pos + 1].repeat_interleave(grp, 1)
            vv = self.v[i, :, :, :pos + 1].repeat_interleave(grp, 1)
            a = F.scaled_dot_product_attention(q, kk, vv, scale=self.d ** -0.5)
            h = h + _linear(a.transpose(1, 2).reshape(1, 1, -1), *L['o'])
            x = _rmsnorm(h, L['ln_post'], self.eps)
            h = h + _linear(F.silu(_linear(x, *L['gate'])) * _linear(x, *L['up']), *L['down'])
        logits = _linear(_rmsnorm(h, self.final_norm, self.eps)[:, -1], *self.lm)
        return int(logits.argmax(-1))
