"""GPU parity of the causal prefill attention (egpt_attn_prefill, tcgen05) against fp64 truth and PyTorch's SDPA:
the attention over the prompt that the reference's prefill runs through SDPA with is_causal
(modeling_qwen3.py:258-291 under research/realmodel/fast_decode.py:77-85). The rule is PyTorch's own bf16 SDPA on the
same inputs (at most twice its largest and 1.25 times its mean error against fp64) and the north star's attention
rule (within 2e-3 of fp64) on rows that see at least 512 keys."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

D = 128


def _ops():
    from efficientgpt_b200 import ops
    return ops


def _inputs(m, pos0, cap, nq, nkv, seed, cuda):
    g = torch.Generator(device='cuda').manual_seed(seed)
    q = torch.randn(m, nq * D, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(nkv, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(nkv, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    # cache rows past the prompt hold NaN: the kernel must never read them
    k[:, pos0 + m:] = float('nan')
    v[:, pos0 + m:] = float('nan')
    return q, k, v


def _reference(q, k, v, pos0, nq, nkv, dtype):
    """Causal attention of rows at positions pos0 .. pos0 + m - 1 over keys 0 .. pos0 + m - 1 in `dtype`, one kv
    group at a time (keeps the fp64 score matrices small)."""
    m = q.shape[0]
    n = pos0 + m
    grp = nq // nkv
    mask = torch.ones(m, n, dtype=torch.bool, device=q.device).tril(diagonal=pos0)
    out = torch.empty(m, nq, D, dtype=dtype, device=q.device)
    for j in range(nkv):
        qq = q.view(m, nq, D)[:, j * grp:(j + 1) * grp].transpose(0, 1).to(dtype)[None]
        kk = k[j, :n].to(dtype)[None, None].expand(1, grp, n, D)
        vv = v[j, :n].to(dtype)[None, None].expand(1, grp, n, D)
        o = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, scale=D ** -0.5)
        out[:, j * grp:(j + 1) * grp] = o[0].transpose(0, 1)
    return out.reshape(m, nq * D)


@pytest.mark.parametrize('m,pos0,nq,nkv', [
    (32, 0, 16, 8),      # config 2's prompt
    (129, 0, 16, 8),     # one row past a query block
    (300, 0, 16, 8),     # ragged last query and key blocks
    (1000, 0, 32, 8),    # the 8B head grouping
    (4096, 0, 32, 8),    # config 5's prompt
    (200, 77, 16, 8),    # a continued prompt: 77 keys already cached
    (1, 1023, 16, 8),    # one row over a long cache (the last prompt row)
    (64, 0, 8, 8),       # no head grouping
])
def test_prefill_attention_vs_fp64_and_sdpa(cuda, m, pos0, nq, nkv):
    ops = _ops()
    cap = pos0 + m + 37
    q, k, v = _inputs(m, pos0, cap, nq, nkv, m + pos0, cuda)
    out = ops.attn_prefill(q, k, v, pos0, nq, nkv, D, scale=D ** -0.5)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(out).all())
    truth = _reference(q, k, v, pos0, nq, nkv, torch.float64)
    sdpa = _reference(q, k, v, pos0, nq, nkv, torch.bfloat16)
    err = float((out.double() - truth).abs().max())
    sdpa_err = float((sdpa.double() - truth).abs().max())
    # no worse than PyTorch's bf16 SDPA: twice its largest error, 1.25 times its mean error (rows with few keys have
    # O(1) outputs whose bf16 probabilities and rounding alone cost up to ~1e-2, in SDPA as here)
    assert err <= max(2 * sdpa_err, 1e-3), (m, pos0, err, sdpa_err)
    mean, sdpa_mean = float((out.double() - truth).abs().mean()), float((sdpa.double() - truth).abs().mean())
    assert mean <= 1.25 * sdpa_mean + 1e-6, (m, pos0, mean, sdpa_mean)
    # the north star's attention rule, within 2e-3 of fp64, on the rows that see at least 512 keys (config 4's
    # shortest context)
    long_rows = torch.arange(m, device=cuda) + pos0 >= 511
    if bool(long_rows.any()):
        long_err = float((out.double() - truth)[long_rows].abs().max())
        assert long_err <= 2e-3, (m, pos0, long_err)


def test_prefill_attention_chunks_match_one_call(cuda):
    """A prompt attended in two calls (the second continuing at pos0) gives the rows of one call."""
    ops = _ops()
    m, nq, nkv = 384, 16, 8
    q, k, v = _inputs(m, 0, m, nq, nkv, 5, cuda)
    whole = ops.attn_prefill(q, k, v, 0, nq, nkv, D, scale=D ** -0.5)
    first = ops.attn_prefill(q[:200].contiguous(), k, v, 0, nq, nkv, D, scale=D ** -0.5)
    second = ops.attn_prefill(q[200:].contiguous(), k, v, 200, nq, nkv, D, scale=D ** -0.5)
    assert torch.equal(torch.cat([first, second]), whole)


def test_prefill_attention_last_row_matches_decode_attention(cuda):
    """m = 1 at pos0 = L - 1 is one decode row: within 2e-3 of the split-K decode attention kernel."""
    ops = _ops()
    L, nq, nkv = 777, 16, 8
    q, k, v = _inputs(1, L - 1, L + 64, nq, nkv, 9, cuda)
    a = ops.attn_prefill(q, k, v, L - 1, nq, nkv, D, scale=D ** -0.5)
    b = ops.attn_decode(q, k, v, torch.tensor([L - 1], device=cuda), nq, nkv, D, scale=D ** -0.5)
    assert float((a.float() - b.float()).abs().max()) <= 2e-3


def test_prefill_attention_argument_errors(cuda):
    from efficientgpt_b200 import _lib as L
    ops = _ops()
    q, k, v = _inputs(16, 0, 16, 16, 8, 0, cuda)
    with pytest.raises(ValueError, match='head_dim'):
        L.check(L.load().egpt_attn_prefill(ops._p(q), 16 * 64, ops._p(q), 16 * 64, ops._p(k), ops._p(v), 16, 0, 16,
                                           16, 8, 64, 0.1, ops._stream()), 'attn_prefill')
    with pytest.raises(ValueError, match='pos0 \\+ m <= cap'):
        ops.attn_prefill(q, k, v, 1, 16, 8, D, scale=D ** -0.5)
    with pytest.raises(ValueError, match='multiple of nkv'):
        ops.attn_prefill(q[:, :12 * D].contiguous(), k, v, 0, 12, 8, D, scale=D ** -0.5)
