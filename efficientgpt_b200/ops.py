"""Tensor-level wrappers over the C-ABI (one function per entry point of include/egpt_b200.h).

PyTorch only provides device memory and the current stream here: every op checks its tensors, passes raw
pointers to libegpt_b200.so and launches on `torch.cuda.current_stream()`, so the calls can be captured in a
CUDA graph. Nothing here computes on the CPU; non-CUDA tensors are rejected.
"""
import ctypes

import torch

from . import _lib as L

MAX_KERNEL_ROWS = 16


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dt(t):
    if t.dtype == torch.bfloat16:
        return L.EGPT_BF16
    if t.dtype == torch.float32:
        return L.EGPT_F32
    raise ValueError(f'unsupported dtype {t.dtype}')


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError('efficientgpt_b200 ops need CUDA tensors (there is no CPU path)')


def _contig_rows(t, name):
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f'{name} must be a 2-D tensor with unit column stride')


def version():
    return L.load().egpt_version().decode()


def quantize_rows(w, scale_dtype=torch.float32):
    """Per-row symmetric int8 of a [N, K] fp32/bf16 CUDA tensor -> (q int8 [N, K], s [N] of scale_dtype)."""
    _cuda(w)
    w = w.detach().contiguous()
    n, k = w.shape
    q = torch.empty((n, k), dtype=torch.int8, device=w.device)
    s = torch.empty(n, dtype=scale_dtype, device=w.device)
    if n == 0 or k == 0:
        raise ValueError('quantize_rows: empty weight')
    L.check(L.load().egpt_quantize_rows(_p(q), _p(s), _dt(s), _p(w), _dt(w), n, k, _stream()), 'quantize_rows')
    return q, s


def gemv_i8(x, w, s, *, out=None, epilogue=L.EPI_NONE, bias=None, residual=None, norm_w=None, eps=1e-6,
            double_round=False, pdl=False, no_tma=False, exact=False):
    """out[m, :] = epilogue(s * (x[m] @ q.T)) for x [M <= 16, K] (bf16 or fp32), q int8 [N, K].

    EPI_SILU_MUL takes q = cat(gate, up) rows ([2I, K]) and returns [M, I]. exact (one bf16 row): the int8
    tensor-core kernel with exact row sums, rounded once (EGPT_FLAG_EXACT)."""
    _cuda(x, w, s, bias, residual, norm_w, out)
    _contig_rows(x, 'x')
    m, k = x.shape
    n = w.shape[0]
    if w.shape[1] != k or not w.is_contiguous() or w.dtype != torch.int8:
        raise ValueError('gemv_i8: w must be a contiguous int8 [N, K] tensor')
    if s.shape != (n,) or not s.is_contiguous():
        raise ValueError('gemv_i8: s must be a contiguous [N] tensor')
    ncols = n // 2 if epilogue == L.EPI_SILU_MUL else n
    if out is None:
        out = torch.empty((m, ncols), dtype=x.dtype, device=x.device) if residual is None else residual
    _contig_rows(out, 'out')
    if residual is not None and (residual.stride() != out.stride() or residual.shape != out.shape):
        raise ValueError('gemv_i8: residual must have the output layout')
    flags = (L.FLAG_DOUBLE_ROUND if double_round else 0) | (L.FLAG_RMSNORM if norm_w is not None else 0) \
        | (L.FLAG_PDL if pdl else 0) | (L.FLAG_NO_TMA if no_tma else 0) | (L.FLAG_EXACT if exact else 0)
    L.check(L.load().egpt_gemv_i8(_p(out), _p(x), _dt(x), m, x.stride(0), out.stride(0), _p(w), _p(s), _dt(s), n, k,
                                  _p(bias), _p(residual), epilogue, _p(norm_w), float(eps), None, flags, _stream()),
            'gemv_i8')
    return out


def gemv_i8_rows(x, w, s, *, double_round, epilogue=L.EPI_NONE, residual=None, bias=None, out=None):
    """Any number of rows: 16-row launches of gemv_i8 (the kernel holds at most 16 rows of x)."""
    m = x.shape[0]
    n = w.shape[0]
    ncols = n // 2 if epilogue == L.EPI_SILU_MUL else n
    if out is None:
        out = residual if residual is not None else torch.empty((m, ncols), dtype=x.dtype, device=x.device)
    for i in range(0, m, MAX_KERNEL_ROWS):
        j = min(m, i + MAX_KERNEL_ROWS)
        gemv_i8(x[i:j], w, s, out=out[i:j], epilogue=epilogue, bias=bias,
                residual=None if residual is None else residual[i:j], double_round=double_round)
    return out


def lm_head_ws(n, device):
    return torch.zeros(int(L.load().egpt_lm_head_ws_bytes(n)), dtype=torch.uint8, device=device)


def lm_head_argmax(x, w, s, ws, *, norm_w=None, eps=1e-6, logits=None, token=None, position=None, advance=False,
                   pdl=False, exact=False):
    """token = argmax(bf16(s * (RMSNorm(x) @ q.T))) on the device; x bf16 [K] (one row). fp32 x (nanoGPT): the
    logits are fp32 s * (x @ q.T) without rounding, written fp32 to `logits`."""
    _cuda(x, w, s, ws, norm_w, logits, token, position)
    n, k = w.shape
    if x.numel() != k or x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError('lm_head_argmax: x must be one bf16 or fp32 row of K elements')
    if logits is not None and logits.dtype != x.dtype:
        raise ValueError('lm_head_argmax: logits must have the dtype of x')
    if token is None:
        token = torch.empty(1, dtype=torch.int64, device=x.device)
    flags = (L.FLAG_RMSNORM if norm_w is not None else 0) | (L.FLAG_ADVANCE if advance else 0) \
        | (L.FLAG_PDL if pdl else 0) | (L.FLAG_X_F32 if x.dtype == torch.float32 else 0) \
        | (L.FLAG_EXACT if exact else 0)
    L.check(L.load().egpt_lm_head_argmax(_p(token), _p(position), _p(logits), _p(x), _p(w), _p(s), _dt(s), n, k,
                                         _p(norm_w), float(eps), _p(ws), ws.numel(), flags, _stream()),
            'lm_head_argmax')
    return token


def rmsnorm(x, w, eps=1e-6, out=None):
    _cuda(x, w, out)
    x2 = x.reshape(-1, x.shape[-1])
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or not x2.is_contiguous():
        raise ValueError('rmsnorm: bf16 contiguous rows expected')
    out = torch.empty_like(x2) if out is None else out
    L.check(L.load().egpt_rmsnorm(_p(out), _p(x2), _p(w), x2.shape[0], x2.shape[1], float(eps), _stream()), 'rmsnorm')
    return out.reshape(x.shape)


def layernorm_f32(x, w, b, eps=1e-5, out=None):
    _cuda(x, w, b, out)
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    out = torch.empty_like(x2) if out is None else out
    L.check(L.load().egpt_layernorm_f32(_p(out), _p(x2), _p(w), _p(b), x2.shape[0], x2.shape[1], float(eps),
                                        _stream()), 'layernorm_f32')
    return out.reshape(x.shape)


def embed(ids, table, pos_table=None, pos0=0, out=None, position=None):
    """out[i] = table[ids[i]] (+ pos_table[pos0 + i], + *position when the device position is given)."""
    _cuda(ids, table, pos_table, out, position)
    ids = ids.reshape(-1).contiguous()
    if ids.dtype != torch.int64:
        raise ValueError('embed: ids must be int64')
    out = torch.empty((ids.numel(), table.shape[1]), dtype=table.dtype, device=table.device) if out is None else out
    L.check(L.load().egpt_embed(_p(out), _p(ids), ids.numel(), _p(table), _p(pos_table), int(pos0), _p(position),
                                table.shape[0], table.shape[1], _dt(table), _stream()), 'embed')
    return out


def qk_norm_rope_kv_append(qkv, k_cache, v_cache, position, nq, nkv, d, *, q_norm_w=None, k_norm_w=None, eps=1e-6,
                           rope_cos=None, rope_sin=None, q_out=None):
    """Rows i of qkv [M, (nq+2nkv)d] at positions *position + i: returns rotated q [M, nq d], fills the caches."""
    _cuda(qkv, k_cache, v_cache, position, q_norm_w, k_norm_w, rope_cos, rope_sin, q_out)
    _contig_rows(qkv, 'qkv')
    m = qkv.shape[0]
    cap = k_cache.shape[-2]
    if q_out is None:
        q_out = torch.empty((m, nq * d), dtype=qkv.dtype, device=qkv.device)
    L.check(L.load().egpt_qk_norm_rope_kv_append(_p(q_out), _p(qkv), qkv.stride(0), _p(k_cache), _p(v_cache), cap,
                                                 _p(position), m, nq, nkv, d, _p(q_norm_w), _p(k_norm_w), float(eps),
                                                 _p(rope_cos), _p(rope_sin), _dt(qkv), _stream()),
            'qk_norm_rope_kv_append')
    return q_out


def attn_ws(m, nq, nkv, d, max_split, device):
    return torch.zeros(int(L.load().egpt_attn_ws_bytes(m, nq, nkv, d, max_split)), dtype=torch.uint8, device=device)


def attn_decode(q, k_cache, v_cache, position, nq, nkv, d, *, scale, max_split=16, ws=None, out=None, append=False,
                q_norm_w=None, k_norm_w=None, eps=1e-6, rope_cos=None, rope_sin=None, pdl=False, ref_softmax=False,
                ragged=False):
    """Split-K decode attention for rows i of q (L_i = *position + i + 1 keys); caches [nkv, cap, d].
    ref_softmax: round the bf16 probabilities as the reference's GPU SDPA kernel does (128-key block walk).
    ragged: row i is its own sequence at position[i] (int64 [m]) with caches [m * nkv, cap, d]."""
    _cuda(q, k_cache, v_cache, position, ws, out, q_norm_w, k_norm_w, rope_cos, rope_sin)
    _contig_rows(q, 'q')
    m = q.shape[0]
    cap = k_cache.shape[-2]
    if out is None:
        out = torch.empty((m, nq * d), dtype=q.dtype, device=q.device)
    if ws is None:
        ws = attn_ws(m, nq, nkv, d, max_split, q.device)
    flags = ((L.FLAG_APPEND if append else 0) | (L.FLAG_PDL if pdl else 0) | (L.FLAG_REF_SOFTMAX if ref_softmax else 0)
             | (L.FLAG_RAGGED if ragged else 0))
    L.check(L.load().egpt_attn_decode(_p(out), out.stride(0), _p(q), q.stride(0), _p(k_cache), _p(v_cache), cap,
                                      _p(position), m, nq, nkv, d, _p(q_norm_w), _p(k_norm_w), float(eps), _p(rope_cos),
                                      _p(rope_sin), float(scale), int(max_split), _p(ws), ws.numel(), _dt(q), flags,
                                      _stream()), 'attn_decode')
    return out


def attn_prefill(q, k_cache, v_cache, pos0, nq, nkv, d, *, scale, out=None):
    """Causal attention of the prompt rows q bf16 [m, nq * d] (row i at position pos0 + i, normed and rotated) over
    the cached keys 0 .. pos0 + i of caches [nkv, cap, d] -> bf16 [m, nq * d], on the tcgen05 tensor cores."""
    _cuda(q, k_cache, v_cache, out)
    _contig_rows(q, 'q')
    if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise ValueError('attn_prefill: bf16 q and caches')
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()) or k_cache.shape != v_cache.shape:
        raise ValueError('attn_prefill: caches must be contiguous [nkv, cap, d]')
    m = q.shape[0]
    cap = k_cache.shape[-2]
    if out is None:
        out = torch.empty((m, nq * d), dtype=q.dtype, device=q.device)
    _contig_rows(out, 'out')
    L.check(L.load().egpt_attn_prefill(_p(out), out.stride(0), _p(q), q.stride(0), _p(k_cache), _p(v_cache), cap,
                                       int(pos0), m, nq, nkv, d, float(scale), _stream()), 'attn_prefill')
    return out


def argmax_rows(logits):
    _cuda(logits)
    x2 = logits.reshape(-1, logits.shape[-1])
    _contig_rows(x2, 'logits')
    out = torch.empty(x2.shape[0], dtype=torch.int64, device=logits.device)
    L.check(L.load().egpt_argmax_rows(_p(out), _p(x2), x2.shape[0], x2.shape[1], x2.stride(0), _dt(x2), _stream()),
            'argmax_rows')
    return out.reshape(logits.shape[:-1])


def gemm_i8_tc(x, w, s, *, double_round=True, out=None, ws=None, add_out=False):
    """bf16 [M, K] x int8 [N, K]^T on the tcgen05 tensor cores -> bf16 [M, N]: bf16(bf16(acc) * s) (the reference's
    >16-row arithmetic) or, with double_round=False, bf16(acc * s). K a multiple of 64. Few rows split K over
    several CTAs per tile with an fp32 workspace (allocated here unless `ws` is given). add_out: `out` holds the
    residual and becomes bf16(out + result) (the HF residual add, fused)."""
    if add_out and out is None:
        raise ValueError('gemm_i8_tc: add_out needs out (the residual)')
    _cuda(x, w, s)
    if x.dtype != torch.bfloat16 or w.dtype != torch.int8 or x.dim() != 2 or w.dim() != 2:
        raise ValueError('gemm_i8_tc: x bf16 [M, K], w int8 [N, K]')
    m, k = x.shape
    n = w.shape[0]
    if w.shape[1] != k or x.stride(1) != 1 or not w.is_contiguous():
        raise ValueError('gemm_i8_tc: shapes or strides')
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    need = int(L.load().egpt_gemm_i8_tc_ws_bytes(m, n, k))
    if ws is None and need:
        ws = torch.empty(need, dtype=torch.uint8, device=x.device)
    L.check(L.load().egpt_gemm_i8_tc(_p(out), out.stride(0), _p(x), x.stride(0), m, _p(w), _p(s), _dt(s), n, k,
                                     (L.FLAG_DOUBLE_ROUND if double_round else 0) | (L.FLAG_ADD_OUT if add_out else 0),
                                     _p(ws),
                                     0 if ws is None else ws.numel(), _stream()), 'gemm_i8_tc')
    return out


def silu_mul(gu, inter, out=None):
    """bf16(bf16(silu(gate)) * up) over rows of the gate|up output gu bf16 [M, >= 2 inter] (gate columns first)."""
    _cuda(gu, out)
    _contig_rows(gu, 'gu')
    if gu.dtype != torch.bfloat16:
        raise ValueError('silu_mul: bf16 rows')
    m = gu.shape[0]
    if out is None:
        out = torch.empty(m, inter, dtype=torch.bfloat16, device=gu.device)
    _contig_rows(out, 'out')
    L.check(L.load().egpt_silu_mul(_p(out), out.stride(0), _p(gu), gu.stride(0), m, int(inter), _stream()), 'silu_mul')
    return out
