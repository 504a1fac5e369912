"""Long-prompt prefill of the Qwen3 engines: the reference's >16-row int8 branch as a plain library GEMM.

replaces: research/realmodel/int8_linear.py:96-97 (`bf16(bf16(x @ bf16(q).T) * s)` for more than 16 rows) inside
the HF Qwen3 forward over the prompt (modeling_qwen3.py:258-335), as GraphGreedyDecoder's prefill runs it
(research/realmodel/fast_decode.py:77-85).

Prompts of hundreds or thousands of tokens are GEMMs, not GEMVs: the projections run on this library's tcgen05 GEMM
(`egpt_gemm_i8_tc`: the int8 weights are widened to bf16 in shared memory on their way to the tensor cores, where
the reference materialises `bf16(q)` in HBM on every call), RMSNorm and the q/k-norm + RoPE + KV-cache write run on
this library's kernels, and causal attention over the prompt runs through PyTorch's SDPA (the reference's own
prefill attention). Under tensor parallelism the row-sharded projections (o_proj, down_proj) need their unscaled
fp32 partial products for the cross-rank sum and stay on a cuBLAS GEMM of the dequantised shard. Only the KV cache is produced: the caller
runs the prompt's last token through the decode step, which writes the first generated token (and, for tensor
parallelism, exchanges the lm_head keys). With `allreduce` (tensor parallelism) o_proj and down_proj give
per-rank partial products that are summed across ranks in fp32 before the scale.
"""
import torch
import torch.nn.functional as F

from . import ops


def _proj(x, q, s):
    """bf16(bf16(x @ bf16(q).T) * s): the op's >16-row arithmetic (int8_linear.py:96-97), on this library's tcgen05
    GEMM (int8 rows widened to bf16 in shared memory, fp32 accumulation in TMEM)."""
    if x.shape[-1] % 64 == 0:
        return ops.gemm_i8_tc(x.contiguous(), q, s, double_round=True)
    y = torch.matmul(x, q.to(torch.bfloat16).t())  # widths the tcgen05 tiles do not take
    return (y.float() * s.float()).to(torch.bfloat16)


def _proj_partial(x, q, s, allreduce):
    """Row-sharded projection: every rank's bf16(x_r @ bf16(q_r).T), summed over the ranks in fp32, then scaled
    and rounded once more (the one-GPU rounding points with the sum split across ranks)."""
    y = torch.matmul(x, q.to(torch.bfloat16).t()).float()
    allreduce(y)
    return (y.to(torch.bfloat16).float() * s.float()).to(torch.bfloat16)


@torch.no_grad()
def fill_kv(ids, layers, embed, kv, rope_cos, rope_sin, nq, nkv, d, eps, allreduce=None):
    """KV cache entries of positions 0 .. len(ids) - 1 for the prompt `ids` (int64 [p] on the device).

    layers: fused per-layer weights (w_qkv, s_qkv, w_o, s_o, w_gu, s_gu, w_down, s_down, ln_in, ln_post, q_norm,
    k_norm), this rank's shard under tensor parallelism (nq, nkv the rank's heads); kv [L, 2, nkv, cap, d] bf16.
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
        if i == len(layers) - 1:  # the last layer's keys and values are all the decode step needs
            break
        qh = q.view(p, nq, d).transpose(0, 1).unsqueeze(0)
        kh, vh = kv[i, 0, :, :p].unsqueeze(0), kv[i, 1, :, :p].unsqueeze(0)
        a = F.scaled_dot_product_attention(qh, kh, vh, is_causal=True, scale=d ** -0.5, enable_gqa=nq != nkv)
        a = a[0].transpose(0, 1).reshape(p, nq * d)
        o = _proj(a, lay['w_o'], lay['s_o']) if allreduce is None else _proj_partial(a, lay['w_o'], lay['s_o'], allreduce)
        h = h + o
        x = ops.rmsnorm(h, lay['ln_post'], eps)
        gu = _proj(x, lay['w_gu'], lay['s_gu'])
        act = F.silu(gu[:, :inter]) * gu[:, inter:]
        dn = (_proj(act, lay['w_down'], lay['s_down']) if allreduce is None
              else _proj_partial(act, lay['w_down'], lay['s_down'], allreduce))
        h = h + dn
    return p
