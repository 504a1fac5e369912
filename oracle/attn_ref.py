"""Attention references in numpy (test infrastructure; see oracle/__init__.py).

Semantics: transformers' SDPA call in Qwen3Attention (modeling_qwen3.py:258-291) with the static cache's mask
`slot <= position`, scale d^-0.5 and GQA (q head h reads kv head h // (nq / nkv)); the split-K form follows
BagelsFun/efficientgpt research/phase5/decode_attention.py:22-71 ((m, l, acc) partials and an LSE combine).
"""
import numpy as np

from .bf16 import round_bf16


def decode_attention_truth(q, k, v, length, scale):
    """fp64 truth. q [nq, d]; k, v [nkv, cap, d]; keys [0, length). Returns [nq, d] float64."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)[:, :length]
    v = np.asarray(v, np.float64)[:, :length]
    nq, nkv = q.shape[0], k.shape[0]
    grp = nq // nkv
    out = np.empty_like(q)
    for h in range(nq):
        s = (k[h // grp] @ q[h]) * scale
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ v[h // grp]
    return out


# Keys per softmax block of the SDPA kernel the reference runs for bf16 decode on the GPU
# (fmha_cutlassF_bf16_aligned_64x128_rf_sm80: 64 queries x 128 keys per iteration; the reference's own profile of
# the int8 decode path names it). It walks the cache in 128-key blocks with a running maximum and feeds each
# block's probabilities, rounded to bf16 relative to the running maximum, to the P.V product.
REF_KEY_BLOCK = 128


def decode_attention_fp32(q, k, v, length, scale, p_bf16=False, block=None):
    """fp32 softmax attention, [nq, d] float32: s = (K q) * scale, p = exp(s - m), out = (p @ V) / sum(p).

    With p_bf16 the probabilities enter p @ V rounded to bf16 while the denominator sums the fp32 values: the
    rounding point of the SDPA kernels that serve bf16 inputs (PyTorch's CPU flash attention and the GPU
    memory-efficient kernel both feed bf16 probabilities to the second product). The reference point m of that
    rounding is the maximum over all keys when block is None (one block: what both kernels do while the
    cache fits one of their key blocks), else the running maximum of the kernel's block walk: keys of block
    j = [j*block, (j+1)*block) are rounded relative to max(s[0 : (j+1)*block]), and the blocks' sums are
    brought to the final maximum in fp32 (exp(m_j - M) factors)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)[:, :length]
    v = np.asarray(v, np.float32)[:, :length]
    nq, nkv = q.shape[0], k.shape[0]
    grp = nq // nkv
    out = np.empty_like(q)
    for h in range(nq):
        s = (k[h // grp] @ q[h]) * np.float32(scale)
        if block is None or length <= block:
            p = np.exp(s - s.max())
            num = (round_bf16(p) if p_bf16 else p) @ v[h // grp]
            out[h] = num / p.sum(dtype=np.float32)
            continue
        M = s.max()
        num = np.zeros(v.shape[-1], np.float32)
        den = np.float32(0)
        run = -np.inf
        for a in range(0, length, block):
            b = min(length, a + block)
            run = max(run, s[a:b].max())
            p = np.exp(s[a:b] - run)
            f = np.float32(np.exp(np.float32(run - M)))
            num += f * ((round_bf16(p) if p_bf16 else p) @ v[h // grp, a:b])
            den += f * p.sum(dtype=np.float32)
        out[h] = num / den
    return out


def split_partials(q, k, v, length, scale, nsplit):
    """Per-split (m, l, acc) in fp32 over key ranges of ceil(length / nsplit) keys."""
    q = np.asarray(q, np.float32)
    chunk = -(-length // nsplit)
    parts = []
    for s in range(nsplit):
        a, b = s * chunk, min(length, (s + 1) * chunk)
        if a >= b:
            parts.append((np.full(q.shape[0], -np.inf, np.float32), np.zeros(q.shape[0], np.float32),
                          np.zeros_like(q)))
            continue
        grp = q.shape[0] // k.shape[0]
        m = np.empty(q.shape[0], np.float32)
        l = np.empty(q.shape[0], np.float32)
        acc = np.empty_like(q)
        for h in range(q.shape[0]):
            sc = (np.asarray(k[h // grp, a:b], np.float32) @ q[h]) * np.float32(scale)
            m[h] = sc.max()
            p = np.exp(sc - m[h])
            l[h] = p.sum(dtype=np.float32)
            acc[h] = p @ np.asarray(v[h // grp, a:b], np.float32)
        parts.append((m, l, acc))
    return parts


def lse_combine(parts):
    """decode_attention.py:59-71 combine: out = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s."""
    m = np.stack([p[0] for p in parts])
    l = np.stack([p[1] for p in parts])
    acc = np.stack([p[2] for p in parts])
    M = m.max(axis=0)
    f = np.where(l > 0, np.exp(m - M[None]), 0.0).astype(np.float32)
    return (f[..., None] * acc).sum(0) / (f * l).sum(0)[:, None]
