"""Prompt prefill of the Qwen3 engines: the reference's >16-row int8 branch on this library's tcgen05 GEMM.

replaces: research/realmodel/int8_linear.py:96-97 (`bf16(bf16(x @ bf16(q).T) * s)` for more than 16 rows) inside
the HF Qwen3 forward over the prompt (modeling_qwen3.py:258-335), as GraphGreedyDecoder's prefill runs it
(research/realmodel/fast_decode.py:77-85).

Prompts of more than 16 tokens are GEMMs, not GEMVs: the projections run on `egpt_gemm_i8_tc` (the int8 weights are
widened to bf16 in shared memory on their way to the tensor cores, where the reference materialises `bf16(q)` in HBM
on every call), RMSNorm and the q/k-norm + RoPE + KV-cache write run on this library's kernels, and causal attention
over the prompt runs on this library's tcgen05 flash-attention kernel (egpt_attn_prefill; head_dim 128) in place of
the reference's SDPA call. The one-GPU engine takes the
last prompt row's hidden state (`last_hidden`) to its final norm and lm_head; the tensor-parallel engine fills the
cache of all but the last token and runs that one through its decode step, which exchanges the lm_head keys. With
`allreduce` (tensor parallelism) o_proj and down_proj give per-rank unscaled partial products (the tcgen05 GEMM
with unit scales, bf16(x_r @ bf16(q_r).T)) that are summed across ranks in fp32 (torch.distributed) before the
scale.
"""
import torch
import torch.nn.functional as F

from . import ops


def _proj(x, q, s, residual=None):
    """bf16(bf16(x @ bf16(q).T) * s): the op's >16-row arithmetic (int8_linear.py:96-97), on this library's tcgen05
    GEMM (int8 rows widened to bf16 in shared memory, fp32 accumulation in TMEM). With `residual` the result is
    bf16(residual + y), the HF residual add, done in the GEMM's epilogue into `residual` itself."""
    if x.shape[-1] % 64 == 0:
        if residual is not None:
            return ops.gemm_i8_tc(x.contiguous(), q, s, double_round=True, out=residual, add_out=True)
        return ops.gemm_i8_tc(x.contiguous(), q, s, double_round=True)
    y = torch.matmul(x, q.to(torch.bfloat16).t())  # widths the tcgen05 tiles do not take
    y = (y.float() * s.float()).to(torch.bfloat16)
    return y if residual is None else residual + y


def _attend(q, k_cache, v_cache, pos0, nq, nkv, d):
    """Causal attention of the rows q [m, nq * d] at positions pos0 .. pos0 + m - 1 over the cached keys: this
    library's tcgen05 kernel (egpt_attn_prefill) for head_dim 128, the head size of every Qwen3 model; other head
    sizes (small test models) take PyTorch's SDPA, the reference's own prefill attention."""
    m = q.shape[0]
    if d == 128:
        return ops.attn_prefill(q.contiguous(), k_cache, v_cache, pos0, nq, nkv, d, scale=d ** -0.5)
    n = pos0 + m
    qh = q.view(m, nq, d).transpose(0, 1).unsqueeze(0)
    kh, vh = k_cache[:, :n].unsqueeze(0), v_cache[:, :n].unsqueeze(0)
    mask = None if pos0 == 0 else torch.ones(m, n, dtype=torch.bool, device=q.device).tril(diagonal=pos0)
    a = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, is_causal=mask is None and m > 1,
                                       scale=d ** -0.5, enable_gqa=nq != nkv)
    return a[0].transpose(0, 1).reshape(m, nq * d)


def _proj_partial(x, q, s, allreduce):
    """Row-sharded projection: every rank's bf16(x_r @ bf16(q_r).T), summed over the ranks in fp32, then scaled
    and rounded once more (the one-GPU rounding points with the sum split across ranks)."""
    if x.shape[-1] % 64 == 0:  # bf16(bf16(acc) * 1) = bf16(acc) on the tcgen05 GEMM
        ones = torch.ones(q.shape[0], dtype=torch.bfloat16, device=x.device)
        y = ops.gemm_i8_tc(x.contiguous(), q, ones, double_round=True).float()
    else:
        y = torch.matmul(x, q.to(torch.bfloat16).t()).float()
    allreduce(y)
    return (y.to(torch.bfloat16).float() * s.float()).to(torch.bfloat16)


@torch.no_grad()
def fill_kv(ids, layers, embed, kv, rope_cos, rope_sin, nq, nkv, d, eps, allreduce=None, last_hidden=False):
    """KV cache entries of positions 0 .. len(ids) - 1 for the prompt `ids` (int64 [p] on the device).

    layers: fused per-layer weights (w_qkv, s_qkv, w_o, s_o, w_gu, s_gu, w_down, s_down, ln_in, ln_post, q_norm,
    k_norm), this rank's shard under tensor parallelism (nq, nkv the rank's heads); kv [L, 2, nkv, cap, d] bf16.
    last_hidden: also run the last layer for the last prompt row (its attention over the whole prompt, o_proj and
    MLP with the same >16-row arithmetic) and return that row's hidden state [1, hidden], for the caller's final
    norm and lm_head; otherwise return p.
    """
    p = ids.numel()
    dev = ids.device
    pos0 = torch.zeros(1, dtype=torch.int64, device=dev)
    h = ops.embed(ids, embed)
    inter = layers[0]['w_gu'].shape[0] // 2
    for i, lay in enumerate(layers):
        x = ops.rmsnorm(h, lay['ln_in'], eps)
        qkv = _proj(x, lay['w_qkv'], lay['s_qkv'])
        q = ops.qk_norm_rope_kv_append(qkv, kv[i, 0], kv[i, 1], pos0, nq, nkv, d, q_norm_w=lay['q_norm'],
                                       k_norm_w=lay['k_norm'], eps=eps, rope_cos=rope_cos, rope_sin=rope_sin)
        if i == len(layers) - 1:
            if not last_hidden:  # the last layer's keys and values are all the decode step needs
                break
            # the last layer only matters for the last row: its attention over the prompt, then o_proj and the MLP
            # on that row (the per-element arithmetic of the >16-row branch does not depend on the row count)
            a = _attend(q[p - 1:p], kv[i, 0], kv[i, 1], p - 1, nq, nkv, d)
            hl = _proj(a, lay['w_o'], lay['s_o'], residual=h[p - 1:p])
            x = ops.rmsnorm(hl, lay['ln_post'], eps)
            gu = _proj(x, lay['w_gu'], lay['s_gu'])
            return _proj(ops.silu_mul(gu, inter), lay['w_down'], lay['s_down'], residual=hl)
        a = _attend(q, kv[i, 0], kv[i, 1], 0, nq, nkv, d)
        if allreduce is None:
            h = _proj(a, lay['w_o'], lay['s_o'], residual=h)
        else:
            h = h + _proj_partial(a, lay['w_o'], lay['s_o'], allreduce)
        x = ops.rmsnorm(h, lay['ln_post'], eps)
        gu = _proj(x, lay['w_gu'], lay['s_gu'])
        act = ops.silu_mul(gu, inter)
        if allreduce is None:
            h = _proj(act, lay['w_down'], lay['s_down'], residual=h)
        else:
            h = h + _proj_partial(act, lay['w_down'], lay['s_down'], allreduce)
    return p
