"""CPU tests: the oracle against the golden vectors produced by the reference (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import attn_ref, int8_ref, parity
from oracle.bf16 import from_bits, from_torch, round_bf16, to_bits
from oracle.qwen3_ref import Qwen3Ref, rmsnorm, rope_table

GOLD = gi.sha  # noqa


def _npz(name):
    from conftest import ROOT
    return np.load(ROOT / 'tests' / 'golden' / name)


def test_bf16_rounding_matches_torch():
    g = torch.Generator().manual_seed(3)
    x = torch.cat([torch.randn(10000, generator=g) * 10 ** torch.randint(-30, 30, (10000,), generator=g).float(),
                   torch.tensor([0.0, -0.0, 1e-40, 3.4e38, float('inf'), -float('inf'), 1.00390625, 1.01171875])])
    ref = x.to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(round_bf16(x.numpy()), ref)
    np.testing.assert_array_equal(from_bits(to_bits(x.numpy())), ref)


def test_quantize_matches_reference_golden(golden):
    z = _npz('quantize.npz')
    w = gi.quantize_input()
    assert gi.sha(w) == golden['quantize']['w_sha256'], 'torch CPU generator changed: golden inputs differ'
    q, s = int8_ref.quantize_weight(from_torch(w), 'cpu')  # the golden ran on CPU
    np.testing.assert_array_equal(q, z['q'])
    np.testing.assert_array_equal(s, z['s'])
    e = gi.quantize_edge_rows()
    assert gi.sha(e) == golden['quantize']['edge_sha256']
    qe, se = int8_ref.quantize_weight(e.numpy(), 'cpu')
    np.testing.assert_array_equal(qe, z['edge_q'])
    np.testing.assert_array_equal(se, z['edge_s'])


def test_prefill_branch_matches_reference_golden(golden):
    z = _npz('prefill_linear.npz')
    for i, (m, k, n) in enumerate(gi.PREFILL_SHAPES):
        x, q, s = gi.prefill_case(i)
        assert [gi.sha(x), gi.sha(q), gi.sha(s)] == golden['prefill_linear']['input_sha256'][i]
        y = int8_ref.int8_linear(from_torch(x), q.numpy(), s.numpy())
        ref = from_bits(z[f'y{i}'])
        # the reference's CPU bf16 GEMM sums in another order: at most one bf16 ulp on rare elements
        diff = np.abs(y - ref)
        ulp = np.maximum(np.abs(ref), 1e-30) * 2.0 ** -7
        assert np.all(diff <= ulp), (m, k, n)
        assert (diff > 0).mean() < 0.01, (m, k, n)


def test_cuda_and_cpu_quantiser_semantics_differ_only_by_the_scalar_division():
    w = from_torch(gi.quantize_input())
    qc, sc = int8_ref.quantize_weight(w, 'cuda')
    qh, sh = int8_ref.quantize_weight(w, 'cpu')
    amax = np.abs(w).max(axis=1)
    np.testing.assert_array_equal(sc, np.maximum(amax * np.float32(1 / 127), np.float32(1e-12)))
    diff = sc != sh
    assert diff.mean() < 0.5  # the reciprocal product is off by one ulp on a minority of rows
    np.testing.assert_array_equal(qc[~diff], qh[~diff])


def test_decode_branch_refuses_more_than_16_rows():
    with pytest.raises(ValueError):
        int8_ref.int8_matmul(np.zeros((17, 32), np.float32), np.zeros((8, 32), np.int8), np.ones(8, np.float32))


def test_int8_matmul_close_to_fp64_truth():
    for n, k in [(64, 2048), (96, 6144)]:
        x, q, s = int8_ref.gemv_inputs(n, k, seed=0)
        y = int8_ref.int8_matmul(x, q, s)
        truth = int8_ref.int8_truth(x, q, s)
        assert np.abs(y - truth).max() <= np.abs(truth).max() * 2.0 ** -8 + 1e-6


def test_split_lse_combine_equals_single_pass():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((16, 128)).astype(np.float32)
    k = rng.standard_normal((8, 300, 128)).astype(np.float32)
    v = rng.standard_normal((8, 300, 128)).astype(np.float32)
    one = attn_ref.decode_attention_fp32(q, k, v, 257, 128 ** -0.5)
    for ns in (1, 3, 7, 40):
        comb = attn_ref.lse_combine(attn_ref.split_partials(q, k, v, 257, 128 ** -0.5, ns))
        np.testing.assert_allclose(comb, one, rtol=2e-5, atol=2e-6)
    truth = attn_ref.decode_attention_truth(q, k, v, 257, 128 ** -0.5)
    assert np.abs(one - truth).max() < 1e-5


def test_rope_table_matches_hf():
    model = gi.build_model(gi.tiny_config())
    cos, sin = model.model.rotary_emb(torch.zeros(1, dtype=torch.bfloat16), torch.arange(128)[None])
    c, s = rope_table(128, from_torch(model.model.rotary_emb.inv_freq))
    np.testing.assert_array_equal(c, from_torch(cos[0]))
    np.testing.assert_array_equal(s, from_torch(sin[0]))


def test_rmsnorm_matches_hf():
    model = gi.build_model(gi.tiny_config())
    x = torch.randn(7, 128, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    blk = model.model.layers[0]
    with torch.no_grad():
        ref = blk.input_layernorm(x)
    y = rmsnorm(from_torch(x), from_torch(blk.input_layernorm.weight), model.config.rms_norm_eps)
    np.testing.assert_array_equal(y, from_torch(ref))


@pytest.mark.parametrize('scale_dtype', ['fp32', 'bf16'])
def test_tiny_model_greedy_tokens_match_reference(golden, scale_dtype):
    model = gi.build_model(gi.tiny_config())
    assert gi.state_hash(model) == golden['tiny_qwen3']['state_sha256'], 'HF random init changed'
    exact = 0
    for p, x in gi.tiny_prompts().items():
        run = golden['tiny_qwen3']['runs'][scale_dtype][str(p)]
        ref = Qwen3Ref.from_hf(model, 128, scale_dtype, semantics='cpu')
        toks, _ = ref.generate(x[0].tolist(), 40)
        ok, first, detail = parity.near_tie_match(run['tokens'], run['margins'], run['tops'], toks)
        assert ok, (scale_dtype, p, detail)
        exact += first is None
        assert len(set(toks)) > 8
    assert exact >= 1


@pytest.mark.parametrize('scale_dtype', ['fp32', 'bf16'])
def test_tiny_model_first_logits_match_reference(scale_dtype):
    z = _npz('tiny_qwen3.npz')
    model = gi.build_model(gi.tiny_config())
    ref = Qwen3Ref.from_hf(model, 128, scale_dtype, semantics='cpu')
    x = gi.tiny_prompts()[5]
    lg = ref.forward(x[0].tolist(), 0)
    gold = from_bits(z[f'logits_p5_{scale_dtype}'])
    np.testing.assert_allclose(lg, gold, atol=1e-2, rtol=1e-2)


def test_near_tie_rule():
    assert parity.near_tie_match([1, 2, 3], [1.0, 1.0, 1.0], [5.0] * 3, [1, 2, 3])[0]
    assert parity.near_tie_match([1, 2, 3], [1.0, 0.0, 1.0], [5.0] * 3, [1, 7, 9])[0]
    assert parity.near_tie_match([1, 2, 3], [1.0, 0.0625, 1.0], [5.0] * 3, [1, 7, 9])[0]  # 2 ulps at 5.0
    assert not parity.near_tie_match([1, 2, 3], [1.0, 0.5, 1.0], [5.0] * 3, [1, 7, 9])[0]
    assert not parity.near_tie_match([1, 2], [1.0, 0.0], [5.0] * 2, [1])[0]


def test_nanogpt_oracle_matches_reference_golden():
    """oracle/nanogpt_ref.py against the reference's own nanoGPT int8 decode (tests/golden/make_golden_nanogpt.py):
    every greedy token equal and the first-step fp32 logits within 1e-6."""
    import json
    from conftest import ROOT
    from oracle.nanogpt_ref import NanoGPTRef
    z = np.load(ROOT / 'tests' / 'golden' / 'nanogpt_tiny.npz')
    meta = json.loads((ROOT / 'tests' / 'golden' / 'nanogpt.json').read_text())
    params = {k[len('param.'):]: z[k] for k in z.files if k.startswith('param.')}
    for run in meta['runs']:
        toks, _ = NanoGPTRef(params, meta['config']).generate(run['prompt'], len(run['tokens']))
        assert toks == run['tokens']
        lg = NanoGPTRef(params, meta['config']).forward(run['prompt'], 0)
        np.testing.assert_allclose(lg, z[f"logits_first_{len(run['prompt'])}"], atol=1e-6, rtol=0)


@pytest.mark.parametrize('n,k,edge', [(512, 2048, None), (256, 6144, 'large'), (128, 12288, 'extreme_w')])
def test_fixed_point_staging_is_exact(n, k, edge):
    """The exact GEMV's staging: balanced digits rebuild X, |X| < 2^30 and every digit in [-128, 127] (digit 3 too),
    and the int64 dot product on X rounded once equals the exact-sum oracle int8_exact (x values of N(0, 1) sit on
    the fixed-point grid: bf16 values at least 2^-29 of the largest)."""
    x, q, s = int8_ref.gemv_inputs(n, k, 4, edge=edge)
    e, big, d = int8_ref.fixed_point_stage(x[0])
    assert np.all(np.abs(big) < 2 ** 30)
    assert d.min() >= -128 and d.max() <= 127
    assert np.array_equal(d[0] + 256 * d[1] + 65536 * d[2] + 16777216 * d[3], big)
    assert np.array_equal(big.astype(np.float64) * 2.0 ** e, x[0].astype(np.float64))  # on the grid
    np.testing.assert_array_equal(int8_ref.int8_fixed_point(x, q, s), int8_ref.int8_exact(x, q, s))
