"""Tensor-parallel restatement of the Qwen3 int8 decode step in numpy (test infrastructure; see oracle/__init__.py).

The reference decodes on one GPU (research/realmodel/fast_decode.py:45-49 over transformers modeling_qwen3.py);
this restates that step split Megatron-style over `world` ranks, as efficientgpt_b200.tp shards it:
  rank r owns q heads [r nq/g, (r+1) nq/g), kv heads [r nkv/g, (r+1) nkv/g) (their q|k|v rows, KV cache and
  attention), o_proj columns of its q heads, gate/up rows and down_proj columns [r I/g, (r+1) I/g), lm_head rows
  [r V/g, (r+1) V/g).
o_proj and down_proj become per-rank partial dot products over the rank's columns, in fp64 (exact for these
bf16 x int8 sums), exchanged with an `allgather` callable and added in rank order; the sum is rounded to fp32,
scaled and rounded at the reference's bf16 points (modeling_qwen3.py:305-335 residual adds). Row-sharded
projections (q|k|v, gate/up, lm_head) are the one-GPU rows unchanged (int8_linear.py:26-38 arithmetic per row).
The greedy token is the maximum of the per-rank (logit, global index) keys: larger logit, then lower index
(fast_decode.py:48, first index on ties), the order of argmax_key.
"""
import numpy as np

from .attn_ref import REF_KEY_BLOCK, decode_attention_fp32
from .bf16 import round_bf16
from .int8_ref import int8_matmul
from .qwen3_ref import apply_rope, rmsnorm, silu


def argmax_key(value, index):
    """64-bit key of a rank's best logit: ordered float bits above (2^32 - 1 - index); NaN above all, -0 == +0."""
    v = np.float32(value)
    if np.isnan(v):
        u = 0xFFFFFFFF
    elif v == 0:
        u = 0x80000000
    else:
        b = int(np.array(v, np.float32).view(np.uint32))
        u = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    return (u << 32) | (0xFFFFFFFF - int(index))


def key_index(key):
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)


def first_argmax(logits):
    """np.argmax semantics with NaN as the maximum (torch.argmax): first index of the largest value."""
    lg = np.asarray(logits, np.float32)
    nan = np.isnan(lg)
    return int(np.argmax(nan)) if nan.any() else int(np.argmax(lg))


class TPQwen3Ref:
    """Rank `rank` of a `world`-way split of a Qwen3Ref (oracle/qwen3_ref.py) model; `allgather(array)` returns
    the list of every rank's array in rank order (a gloo all_gather in the tests, [array] for world 1)."""

    def __init__(self, full, rank, world, allgather):
        c = full.cfg
        self.full, self.rank, self.world, self.allgather = full, rank, world, allgather
        self.nq, self.nkv, self.d = c['n_q_heads'] // world, c['n_kv_heads'] // world, c['head_dim']
        self.inter, self.vocab = c['intermediate'] // world, c['vocab'] // world
        d = self.d
        self.q_rows = slice(rank * self.nq * d, (rank + 1) * self.nq * d)
        self.kv_rows = slice(rank * self.nkv * d, (rank + 1) * self.nkv * d)
        self.i_rows = slice(rank * self.inter, (rank + 1) * self.inter)
        self.v_rows = slice(rank * self.vocab, (rank + 1) * self.vocab)
        cap = full.cap
        self.k = np.zeros((len(full.layers), self.nkv, cap, d), np.float32)
        self.v = np.zeros((len(full.layers), self.nkv, cap, d), np.float32)

    def _reduce(self, part):
        """Rank-order sum of every rank's fp64 partial."""
        tot = np.zeros_like(part)
        for p in self.allgather(part):
            tot = tot + p
        return tot

    def step(self, tok, pos):
        """One decode token at position pos; returns (this rank's bf16 logits, the greedy token of all ranks)."""
        f, c = self.full, self.full.cfg
        eps, d, nq, nkv = c['eps'], self.d, self.nq, self.nkv
        if pos >= f.cap:
            raise ValueError('position past the cache')
        h = f.embed[[int(tok)]]
        cos, sin = f.cos[pos:pos + 1][:, None, :], f.sin[pos:pos + 1][:, None, :]
        scale = d ** -0.5
        for li, L in enumerate(f.layers):
            x = rmsnorm(h, L['ln_in'], eps)
            q = int8_matmul(x, L['q'][0][self.q_rows], L['q'][1][self.q_rows]).reshape(1, nq, d)
            k = int8_matmul(x, L['k'][0][self.kv_rows], L['k'][1][self.kv_rows]).reshape(1, nkv, d)
            v = int8_matmul(x, L['v'][0][self.kv_rows], L['v'][1][self.kv_rows]).reshape(1, nkv, d)
            q = apply_rope(rmsnorm(q, L['q_norm'], eps), cos, sin)
            k = apply_rope(rmsnorm(k, L['k_norm'], eps), cos, sin)
            self.k[li, :, pos] = k[0]
            self.v[li, :, pos] = v[0]
            o = decode_attention_fp32(q[0], self.k[li], self.v[li], pos + 1, scale, p_bf16=True, block=REF_KEY_BLOCK)
            o = round_bf16(o).reshape(1, nq * d)
            part = o.astype(np.float64) @ L['o'][0][:, self.q_rows].astype(np.float64).T
            y = round_bf16(self._reduce(part).astype(np.float32) * L['o'][1][None, :])
            h = round_bf16(h + y)
            x = rmsnorm(h, L['ln_post'], eps)
            g = int8_matmul(x, L['gate'][0][self.i_rows], L['gate'][1][self.i_rows])
            u = int8_matmul(x, L['up'][0][self.i_rows], L['up'][1][self.i_rows])
            a = round_bf16(round_bf16(silu(g)) * u)
            part = a.astype(np.float64) @ L['down'][0][:, self.i_rows].astype(np.float64).T
            y = round_bf16(self._reduce(part).astype(np.float32) * L['down'][1][None, :])
            h = round_bf16(h + y)
        hn = rmsnorm(h, f.final_norm, eps)
        logits = int8_matmul(hn, f.lm_q[self.v_rows], f.lm_s[self.v_rows])[0]
        best = first_argmax(logits)
        key = argmax_key(logits[best], best + self.rank * self.vocab)
        keys = self.allgather(np.array([key], np.uint64).view(np.int64))  # (bit pattern; gloo has no uint64)
        return logits, key_index(max(int(kk.view(np.uint64)[0]) for kk in keys))

    def feed_and_generate(self, prompt, n_new):
        """Prompt token by token from position 0, then n_new greedy tokens; returns (tokens, per-token logits)."""
        toks, logs = [], []
        pos, nxt = 0, None
        for t in prompt:
            lg, nxt = self.step(t, pos)
            pos += 1
        toks.append(nxt)
        logs.append(lg)
        for _ in range(n_new - 1):
            lg, nxt = self.step(nxt, pos)
            pos += 1
            toks.append(nxt)
            logs.append(lg)
        return toks, logs
