"""GPU parity of the decode attention kernels (egpt_attn_decode, egpt_qk_norm_rope_kv_append)
against fp64 truth, the reference's masked-SDPA error rule (research/phase5/test_graph_gpu.py:202-261) and the
oracle's norm/RoPE restatement."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import attn_ref
from oracle.bf16 import from_torch, round_bf16
from oracle.qwen3_ref import apply_rope, rmsnorm

pytestmark = pytest.mark.gpu

NQ, NKV, D = 16, 8, 128
SCALE = D ** -0.5


def _ops():
    from efficientgpt_b200 import _lib as L, ops
    return L, ops


def _inputs(L, cap, seed, cuda, dtype=torch.bfloat16):
    g = torch.Generator(device='cuda').manual_seed(seed)
    q = torch.randn(1, NQ * D, device=cuda, generator=g).to(dtype)
    k = torch.randn(NKV, cap, D, device=cuda, generator=g).to(dtype)
    v = torch.randn(NKV, cap, D, device=cuda, generator=g).to(dtype)
    return q, k, v


def _sdpa_err(q, k, v, length):
    qq = q.view(1, NQ, 1, D)
    kk = k[:, :length].repeat_interleave(NQ // NKV, 0)[None]
    vv = v[:, :length].repeat_interleave(NQ // NKV, 0)[None]
    ref = F.scaled_dot_product_attention(qq.double(), kk.double(), vv.double(), scale=SCALE)
    out = F.scaled_dot_product_attention(qq, kk, vv, scale=SCALE)
    return float((out.double() - ref).abs().max())


@pytest.mark.parametrize('length', [512, 2048, 8192, 32768])
@pytest.mark.parametrize('max_split', [1, 19, 64])
def test_decode_attention_vs_fp64(cuda, length, max_split):
    L, ops = _ops()
    q, k, v = _inputs(L, length, length, cuda)
    pos = torch.tensor([length - 1], device=cuda)
    out = ops.attn_decode(q, k, v, pos, NQ, NKV, D, scale=SCALE, max_split=max_split)
    truth = attn_ref.decode_attention_truth(from_torch(q).reshape(NQ, D), from_torch(k), from_torch(v), length, SCALE)
    err = float(np.abs(from_torch(out).reshape(NQ, D) - truth).max())
    assert err <= 2e-3, (length, max_split, err)
    assert err <= max(2 * _sdpa_err(q, k, v, length), 1e-3), (length, max_split, err)


def test_split_count_does_not_change_much(cuda):
    L, ops = _ops()
    q, k, v = _inputs(L, 4096, 1, cuda)
    pos = torch.tensor([3000], device=cuda)
    outs = [ops.attn_decode(q, k, v, pos, NQ, NKV, D, scale=SCALE, max_split=ms).float() for ms in (1, 2, 7, 24, 64)]
    for o in outs[1:]:
        torch.testing.assert_close(o, outs[0], atol=4e-3, rtol=1e-2)


@pytest.mark.parametrize('length', [100, 128, 129, 300, 1000, 3000])
@pytest.mark.parametrize('max_split', [1, 3, 18])
def test_ref_softmax_matches_oracle_block_walk(cuda, length, max_split):
    """EGPT_FLAG_REF_SOFTMAX: probabilities rounded relative to the running maximum of the reference GPU
    kernel's 128-key blocks (oracle attn_ref, block=REF_KEY_BLOCK). What remains is fp32 noise: sums in
    another order, and exp() of CUDA vs numpy one fp32 ulp apart, which now and then moves a probability
    across a bf16 rounding boundary (one bf16 ulp of p, i.e. at most 2^-8 max|V| / sum(p) on the output).
    Outputs agree to one bf16 ulp plus a few such moves; nearly all of them exactly."""
    L, ops = _ops()
    q, k, v = _inputs(L, 3072, 7 + length, cuda)
    pos = torch.tensor([length - 1], device=cuda)
    out = from_torch(ops.attn_decode(q, k, v, pos, NQ, NKV, D, scale=SCALE, max_split=max_split,
                                     ref_softmax=True)).reshape(NQ, D)
    qn, kn, vn = from_torch(q).reshape(NQ, D), from_torch(k), from_torch(v)
    want = round_bf16(attn_ref.decode_attention_fp32(qn, kn, vn, length, SCALE, p_bf16=True,
                                                     block=attn_ref.REF_KEY_BLOCK))
    grp = NQ // NKV
    tol = np.empty((NQ, 1))
    for h in range(NQ):
        sc = (kn[h // grp, :length].astype(np.float64) @ qn[h]) * SCALE
        den = np.exp(sc - sc.max()).sum()
        tol[h] = 4 * 2.0 ** -8 * np.abs(vn[h // grp, :length]).max() / den
    diff = np.abs(out - want)
    assert (diff <= np.abs(want) * 2.0 ** -7 + tol).all(), (length, max_split)
    assert (diff == 0).mean() > 0.98, (length, max_split, float((diff == 0).mean()))


def test_never_reads_past_position(cuda):
    L, ops = _ops()
    q, k, v = _inputs(L, 300, 2, cuda)
    for p in (0, 17, 127, 128, 250, 299):
        pos = torch.tensor([p], device=cuda)
        clean = ops.attn_decode(q, k, v, pos, NQ, NKV, D, scale=SCALE, max_split=8)
        kp, vp = k.clone(), v.clone()
        kp[:, p + 1:] = float('nan')
        vp[:, p + 1:] = float('nan')
        assert torch.equal(clean, ops.attn_decode(q, kp, vp, pos, NQ, NKV, D, scale=SCALE, max_split=8)), p


def test_multi_row_causal_matches_rowwise(cuda):
    """Prefill rows: row i attends to [0, pos0 + i]; equals one decode call per row. The one-row calls take the
    streamed kernels and the multi-row call the split kernel (fp32 sums in other orders, and without the
    reference-rounding flag bf16 probabilities against other running maxima): within the tolerance that split
    counts are held to, with and without the flag."""
    L, ops = _ops()
    cap, m = 96, 9
    g = torch.Generator(device='cuda').manual_seed(4)
    q = torch.randn(m, NQ * D, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(NKV, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(NKV, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    pos0 = torch.tensor([40], device=cuda)
    out = ops.attn_decode(q, k, v, pos0, NQ, NKV, D, scale=SCALE, max_split=4)
    ref = ops.attn_decode(q, k, v, pos0, NQ, NKV, D, scale=SCALE, max_split=4, ref_softmax=True)
    for i in range(m):
        one = ops.attn_decode(q[i:i + 1].contiguous(), k, v, pos0 + i, NQ, NKV, D, scale=SCALE, max_split=4)
        torch.testing.assert_close(out[i:i + 1].float(), one.float(), atol=4e-3, rtol=1e-2)
        one_ref = ops.attn_decode(q[i:i + 1].contiguous(), k, v, pos0 + i, NQ, NKV, D, scale=SCALE, max_split=4,
                                  ref_softmax=True)
        torch.testing.assert_close(ref[i:i + 1].float(), one_ref.float(), atol=4e-3, rtol=1e-2)


def _norm_rope_setup(cuda, cap=64):
    g = torch.Generator(device='cuda').manual_seed(5)
    qkv = torch.randn(3, (NQ + 2 * NKV) * D, device=cuda, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)).to(torch.bfloat16)
    inv = (1.0 / (1e6 ** (torch.arange(0, D, 2, device=cuda).float() / D))).to(torch.bfloat16).float()
    fr = torch.arange(cap, device=cuda).float()[:, None] * inv[None]
    cos, sin = fr.cos().to(torch.bfloat16).contiguous(), fr.sin().to(torch.bfloat16).contiguous()
    return qkv, qn, kn, cos, sin


def test_qk_norm_rope_append_vs_oracle(cuda):
    L, ops = _ops()
    cap = 64
    qkv, qn, kn, cos, sin = _norm_rope_setup(cuda, cap)
    kc = torch.zeros(NKV, cap, D, device=cuda, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    pos0 = torch.tensor([10], device=cuda)
    q = ops.qk_norm_rope_kv_append(qkv, kc, vc, pos0, NQ, NKV, D, q_norm_w=qn, k_norm_w=kn, eps=1e-6, rope_cos=cos,
                                   rope_sin=sin)
    x = from_torch(qkv)
    c = np.concatenate([from_torch(cos)] * 2, -1)[10:13][:, None, :]
    s = np.concatenate([from_torch(sin)] * 2, -1)[10:13][:, None, :]
    q_ref = apply_rope(rmsnorm(x[:, :NQ * D].reshape(3, NQ, D), from_torch(qn), 1e-6), c, s).reshape(3, NQ * D)
    k_ref = apply_rope(rmsnorm(x[:, NQ * D:(NQ + NKV) * D].reshape(3, NKV, D), from_torch(kn), 1e-6), c, s)
    v_ref = x[:, (NQ + NKV) * D:].reshape(3, NKV, D)
    # rsqrtf vs 1/sqrt: rare one-ulp differences
    assert (from_torch(q) != q_ref).mean() < 0.01
    np.testing.assert_allclose(from_torch(q), q_ref, rtol=2 ** -7, atol=1e-6)
    np.testing.assert_allclose(from_torch(kc)[:, 10:13].transpose(1, 0, 2), k_ref, rtol=2 ** -7, atol=1e-6)
    np.testing.assert_array_equal(from_torch(vc)[:, 10:13].transpose(1, 0, 2), v_ref)
    assert float(kc[:, :10].abs().sum()) == 0 and float(kc[:, 13:].abs().sum()) == 0


def test_fused_append_equals_separate_kernels(cuda):
    """The in-kernel q/k-norm + RoPE + append (EGPT_FLAG_APPEND) writes the same cache rows as the separate kernel,
    bit for bit, and gives the same output within the split-count tolerance (the separate one-row call takes the
    streamed kernels, the fused one the split kernel), with and without the reference rounding."""
    L, ops = _ops()
    cap = 200
    qkv, qn, kn, cos, sin = _norm_rope_setup(cuda, cap)
    g = torch.Generator(device='cuda').manual_seed(9)
    k0 = torch.randn(NKV, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    v0 = torch.randn(NKV, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    for p, ms in ((0, 4), (130, 4), (130, 1), (199, 19)):
        pos = torch.tensor([p], device=cuda)
        ka, va = k0.clone(), v0.clone()
        kw = dict(q_norm_w=qn, k_norm_w=kn, eps=1e-6, rope_cos=cos, rope_sin=sin)
        fused = ops.attn_decode(qkv[:1].contiguous(), ka, va, pos, NQ, NKV, D, scale=SCALE, max_split=ms, append=True,
                                **kw)
        fused_ref = ops.attn_decode(qkv[:1].contiguous(), ka, va, pos, NQ, NKV, D, scale=SCALE, max_split=ms,
                                    append=True, ref_softmax=True, **kw)
        kb, vb = k0.clone(), v0.clone()
        q = ops.qk_norm_rope_kv_append(qkv[:1].contiguous(), kb, vb, pos, NQ, NKV, D, **kw)
        sep = ops.attn_decode(q, kb, vb, pos, NQ, NKV, D, scale=SCALE, max_split=ms)
        sep_ref = ops.attn_decode(q, kb, vb, pos, NQ, NKV, D, scale=SCALE, max_split=ms, ref_softmax=True)
        assert torch.equal(ka, kb) and torch.equal(va, vb), p
        torch.testing.assert_close(fused_ref.float(), sep_ref.float(), atol=4e-3, rtol=1e-2)
        torch.testing.assert_close(fused.float(), sep.float(), atol=4e-3, rtol=1e-2)


def test_fp32_mha_path(cuda):
    """nanoGPT attention: fp32 caches, 6 heads of 64, no norm / RoPE."""
    L, ops = _ops()
    g = torch.Generator(device='cuda').manual_seed(6)
    cap, nh, d = 256, 6, 64
    q = torch.randn(1, nh * d, device=cuda, generator=g)
    k = torch.randn(nh, cap, d, device=cuda, generator=g)
    v = torch.randn(nh, cap, d, device=cuda, generator=g)
    pos = torch.tensor([200], device=cuda)
    out = ops.attn_decode(q, k, v, pos, nh, nh, d, scale=d ** -0.5, max_split=8)
    truth = attn_ref.decode_attention_truth(from_torch(q).reshape(nh, d), from_torch(k), from_torch(v), 201, d ** -0.5)
    assert np.abs(from_torch(out).reshape(nh, d) - truth).max() < 1e-5


@pytest.mark.parametrize('nq,nkv', [(8, 8), (32, 8)])
@pytest.mark.parametrize('length', [1, 130, 5000])
def test_single_row_group_sizes_vs_fp64(cuda, nq, nkv, length):
    """The one-row bf16 path (K/V streamed through shared memory by bulk copies) with 1 and 4 q heads per kv head,
    a single key, a ragged last block and many ranges: within 2e-3 of fp64 and 2x PyTorch's SDPA error; cache rows
    past the position hold NaN and are never read."""
    L, ops = _ops()
    g = torch.Generator(device='cuda').manual_seed(length + nq)
    cap = length + 64
    q = torch.randn(1, nq * D, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(nkv, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(nkv, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    k[:, length:] = float('nan')
    v[:, length:] = float('nan')
    pos = torch.tensor([length - 1], device=cuda)
    out = ops.attn_decode(q, k, v, pos, nq, nkv, D, scale=SCALE, max_split=64)
    qq = q.view(1, nq, 1, D)
    kk = k[:, :length].repeat_interleave(nq // nkv, 0)[None]
    vv = v[:, :length].repeat_interleave(nq // nkv, 0)[None]
    truth = F.scaled_dot_product_attention(qq.double(), kk.double(), vv.double(), scale=SCALE).reshape(1, nq * D)
    sdpa = F.scaled_dot_product_attention(qq, kk, vv, scale=SCALE).reshape(1, nq * D)
    err = float((out.double() - truth).abs().max())
    assert err <= 2e-3 or length < 512, (nq, length, err)  # short contexts: O(1) outputs, bf16 output rounding
    assert err <= max(2 * float((sdpa.double() - truth).abs().max()), 1e-3), (nq, length, err)


@pytest.mark.parametrize('nq,nkv', [(8, 8), (32, 8)])
@pytest.mark.parametrize('length', [130, 3000])
def test_single_row_ref_softmax_group_sizes_vs_oracle(cuda, nq, nkv, length):
    """The reference rounding on the one-row streamed kernels (block-maximum pass, then the attention pass) with 1
    and 4 q heads per kv head: the oracle's 128-key block walk to one bf16 ulp plus the fp32-noise allowance of
    test_ref_softmax_matches_oracle_block_walk, nearly all outputs identical."""
    L, ops = _ops()
    g = torch.Generator(device='cuda').manual_seed(3 * length + nq)
    cap = 3072
    q = torch.randn(1, nq * D, device=cuda, generator=g).to(torch.bfloat16)
    k = torch.randn(nkv, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(nkv, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    pos = torch.tensor([length - 1], device=cuda)
    out = from_torch(ops.attn_decode(q, k, v, pos, nq, nkv, D, scale=SCALE, max_split=64,
                                     ref_softmax=True)).reshape(nq, D)
    qn, kn, vn = from_torch(q).reshape(nq, D), from_torch(k), from_torch(v)
    want = round_bf16(attn_ref.decode_attention_fp32(qn, kn, vn, length, SCALE, p_bf16=True,
                                                     block=attn_ref.REF_KEY_BLOCK))
    grp = nq // nkv
    tol = np.empty((nq, 1))
    for h in range(nq):
        sc = (kn[h // grp, :length].astype(np.float64) @ qn[h]) * SCALE
        tol[h] = 4 * 2.0 ** -8 * np.abs(vn[h // grp, :length]).max() / np.exp(sc - sc.max()).sum()
    diff = np.abs(out - want)
    assert (diff <= np.abs(want) * 2.0 ** -7 + tol).all(), (nq, length)
    assert (diff == 0).mean() > 0.98, (nq, length, float((diff == 0).mean()))
