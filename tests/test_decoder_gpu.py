"""GPU parity of the whole decode path (egpt_decode_step in a CUDA graph behind GraphGreedyDecoder) against the
reference's greedy tokens (golden fixtures) and the oracle. Mirrors research/realmodel/test_fast_decode.py."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import parity
from oracle.bf16 import from_bits, from_torch
from oracle.qwen3_ref import Qwen3Ref

pytestmark = pytest.mark.gpu


def _quantize(model, scale_dtype, semantics):
    """quantize_model, then (semantics='cpu') overwrite q/s with the quantiser evaluated as the golden run did:
    the goldens come from the reference on CPU, where `max|w| / 127.0` is a true division, while on the GPU
    PyTorch (and the product) multiply by fl32(1/127); a few q elements differ between the two."""
    from efficientgpt_b200.int8_linear import Int8Linear, quantize_model
    orig = {n: m.weight.detach().clone() for n, m in model.named_modules() if isinstance(m, torch.nn.Linear)}
    quantize_model(model, scale_dtype=scale_dtype)
    if semantics == 'cpu':
        for n, m in model.named_modules():
            if isinstance(m, Int8Linear):
                w = orig[n].float()
                amax = w.abs().amax(1)
                s = (amax / torch.full_like(amax, 127.0)).clamp_min(1e-12)  # tensor divisor: true division
                m.qweight.copy_(torch.round(w / s[:, None]).clamp(-127, 127).to(torch.int8))
                m.scale.copy_(s.to(m.scale.dtype))
    return model


def _cfg05():
    """The tiny config with N(0, 0.05) weights (fresh each time: quantize_model unties the lm_head in the config
    it is given)."""
    c = gi.tiny_config()
    c.initializer_range = 0.05
    return c


def _tiny(scale_dtype=torch.float32, quantize=True, semantics='cuda'):
    model = gi.build_model(gi.tiny_config())
    cpu_hash = gi.state_hash(model)
    model = model.cuda()
    if quantize:
        _quantize(model, scale_dtype, semantics)
    return model, cpu_hash


@pytest.mark.parametrize('semantics', ['cpu', 'cuda'])
@pytest.mark.parametrize('scale_dtype', [torch.float32, torch.bfloat16])
def test_tokens_match_reference_golden(cuda, golden, scale_dtype, semantics):
    """semantics='cpu': the golden's exact weights; 'cuda': the product's own quantiser (a few q differ)."""
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    model, h = _tiny(scale_dtype, semantics=semantics)
    assert h == golden['tiny_qwen3']['state_sha256'], 'HF random init changed: golden tokens do not apply'
    key = 'fp32' if scale_dtype == torch.float32 else 'bf16'
    dec = GraphGreedyDecoder(model, max_cache_len=128)
    report = []
    for p, x in gi.tiny_prompts().items():
        run = golden['tiny_qwen3']['runs'][key][str(p)]
        got, st = dec.generate(x.cuda(), 40)
        assert st['tokens'] == 40
        assert len(set(got)) > 8, 'degenerate model output would make equality trivial'
        ok, first, detail = parity.near_tie_match(run['tokens'], run['margins'], run['tops'], got)
        assert ok, (key, p, detail)
        report.append((p, first, None if first is None else run['margins'][first],
                       None if first is None else parity.bf16_ulp(run['tops'][first])))
    import warnings
    warnings.warn(f'tiny Qwen3 {key} scales, {semantics} quantiser: (prompt length, first divergence, reference '
                  f'top-2 margin there, one bf16 ulp of its top-1 logit) = {report}')
    # Every prompt identical over all 40 tokens, or its first divergence where the reference's own bf16 logits are
    # tied to within ONE ulp: the reference's near-tie rule (research/phase5/benchmark_review.py:54-67, margin
    # < 1e-2) was written for fp32 logits; these logits are bf16, whose spacing above |4| is 0.03125, so the
    # smallest non-zero margin there is already three times 1e-2, and one rounding step anywhere in the forward
    # can swap a one-ulp pair. Measured: one or two of the three prompts diverge, at margins 0 or one ulp.
    assert all(first is None or margin < 1e-2 or margin <= ulp for _, first, margin, ulp in report), report
    assert sum(first is None for _, first, _, _ in report) >= 1


def test_quantized_weights_equal_oracle(cuda):
    model, _ = _tiny()
    ref_model = gi.build_model(gi.tiny_config())
    ref = Qwen3Ref.from_hf(ref_model, 128, 'fp32')
    blk = model.model.layers[1].mlp.down_proj
    q, s = ref.layers[1]['down']
    np.testing.assert_array_equal(blk.qweight.cpu().numpy(), q)
    np.testing.assert_array_equal(blk.scale.cpu().numpy(), s)


@pytest.mark.parametrize('scale_dtype', ['fp32', 'bf16'])
def test_logits_match_reference_and_oracle(cuda, scale_dtype):
    """Prefill logits vs the reference's golden logits, then 12 teacher-forced decode steps vs the oracle
    (bf16 logits within 1e-2 abs / 1e-2 rel)."""
    from conftest import ROOT
    from efficientgpt_b200.engine import Qwen3Engine
    sd = torch.float32 if scale_dtype == 'fp32' else torch.bfloat16
    model, _ = _tiny(sd, semantics='cpu')  # the golden's quantisation (see _quantize)
    eng = Qwen3Engine(model, 128, keep_logits=True)
    x = gi.tiny_prompts()[5]
    eng.prefill(x.cuda())
    z = np.load(ROOT / 'tests' / 'golden' / 'tiny_qwen3.npz')
    np.testing.assert_allclose(from_torch(eng.logits), from_bits(z[f'logits_p5_{scale_dtype}']), atol=1e-2, rtol=1e-2)
    ref = Qwen3Ref.from_hf(gi.build_model(gi.tiny_config()), 128, scale_dtype, semantics='cpu')
    lg = ref.forward(x[0].tolist(), 0)
    np.testing.assert_allclose(from_torch(eng.logits), lg, atol=1e-2, rtol=1e-2)
    pos = 5
    for i in range(12):
        tok = int(np.argmax(lg))
        eng.token.fill_(tok)
        eng.step()
        lg = ref.forward([tok], pos)
        pos += 1
        assert int(eng.position) == pos
        np.testing.assert_allclose(from_torch(eng.logits), lg, atol=1e-2, rtol=1e-2, err_msg=f'step {i}')
        if int(eng.token) != int(np.argmax(lg)):  # only at a near-tie of the oracle's own logits
            top = np.sort(lg)[-2:]
            assert top[1] - top[0] <= parity.near_tie_threshold(top[1]), i


@pytest.mark.parametrize('scale_dtype', [torch.float32, torch.bfloat16])
def test_persistent_step_matches_launch_sequence(cuda, scale_dtype):
    """egpt_decode_step_persistent (one cooperative kernel) vs egpt_decode_step (launch sequence), teacher-forced
    for 600 steps (past 512 keys, where attention splits over several ranges and the persistent kernel exchanges
    range maxima). Attention, norms and RoPE are the same code; the GEMVs differ in summation: the persistent
    kernel's int8 tensor-core dot products are exact (one rounding), the per-stage kernels sum in fp32. Logits
    agree under the long-sequence rule and tokens differ only at near-ties of the launch sequence's logits."""
    from efficientgpt_b200 import _lib
    from efficientgpt_b200.engine import Qwen3Engine
    model = gi.build_model(_cfg05(), seed=3).cuda()  # moderate gain: flips do not snowball over 600 steps
    _quantize(model, scale_dtype, 'cuda')
    a = Qwen3Engine(model, 640, keep_logits=True, persistent=False)
    b = Qwen3Engine(model, 640, keep_logits=True, step='persistent')
    assert b.persistent and not a.persistent and a.attn_max_split == b.attn_max_split
    x = gi.tiny_prompts()[37].cuda()
    a.prefill(x)
    b.prefill(x)
    same = 0
    for i in range(600):
        b.token.copy_(a.token)  # teacher-force b onto a's tokens
        a.step()
        b.step()
        assert int(a.position) == int(b.position) == 38 + i
        la, lb = from_torch(a.logits), from_torch(b.logits)
        ok, detail = parity.logits_close(lb, la)
        assert ok, (i, detail)
        if int(a.token) != int(b.token):
            top = np.sort(la)[-2:]
            assert top[1] - top[0] <= parity.near_tie_threshold(top[1]), i
        else:
            same += 1
    assert same >= 590
    assert _lib.device_error() == 0


def test_persistent_wide_mlp_matches_launch_sequence(cuda):
    """An intermediate wider than the persistent kernel's register staging (the 8B shape's 12288; here 8192 with
    head_dim 128 and 4 q heads per kv head) takes the two-pass staging of the down_proj input; teacher-forced
    against the launch sequence under the same rules as above."""
    from transformers import Qwen3Config
    from efficientgpt_b200 import _lib
    from efficientgpt_b200.engine import Qwen3Engine
    cfg = Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=8192, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=256,
                      tie_word_embeddings=True, initializer_range=0.05)
    model = gi.build_model(cfg, seed=5).cuda()
    _quantize(model, torch.bfloat16, 'cuda')
    a = Qwen3Engine(model, 160, keep_logits=True, persistent=False)
    b = Qwen3Engine(model, 160, keep_logits=True, step='persistent')
    assert b.step_kind == 'persistent'
    x = gi.tiny_prompts()[5].cuda()
    a.prefill(x)
    b.prefill(x)
    same = 0
    for i in range(120):
        b.token.copy_(a.token)
        a.step()
        b.step()
        la, lb = from_torch(a.logits), from_torch(b.logits)
        ok, detail = parity.logits_close(lb, la)
        assert ok, (i, detail)
        if int(a.token) != int(b.token):
            top = np.sort(la)[-2:]
            assert top[1] - top[0] <= parity.near_tie_threshold(top[1]), i
        else:
            same += 1
    assert same >= 115
    assert _lib.device_error() == 0


def _dataflow_vs_persistent(model, cap, prompt, steps):
    """Teacher-forced: the dataflow step against the persistent step. Their GEMVs, norms, rope and lm_head are the
    same arithmetic; attention differs in summation order only when the dataflow step holds the K/V rows in shared
    memory (its own score and P.V loops, same 128-key-block probability rounding). So: logits within the north
    star's 1e-2 abs + 1e-2 rel for 99.5% of the entries on average and 97% at every step (all within the hard bound
    of parity.logits_close), every step's token agrees unless the persistent step's top-2 margin is within twice the
    tolerance, and at least 95% of the steps agree. (Against the numpy oracle, on the wide-MLP model below, the
    persistent and launch-sequence steps themselves dip to 98.3% at their worst step, the dataflow step to 98.0%.)"""
    from efficientgpt_b200 import _lib
    from efficientgpt_b200.engine import Qwen3Engine
    a = Qwen3Engine(model, cap, keep_logits=True, step='persistent')
    b = Qwen3Engine(model, cap, keep_logits=True, step='dataflow')
    assert b.step_kind == 'dataflow' and a.step_kind == 'persistent'
    a.prefill(prompt)
    b.prefill(prompt)
    same, fracs = 0, []
    for i in range(steps):
        b.token.copy_(a.token)
        a.step()
        b.step()
        assert int(a.position) == int(b.position)
        la, lb = a.logits.float().cpu().numpy().ravel(), b.logits.float().cpu().numpy().ravel()
        ok, detail = parity.logits_close(lb, la, frac=0.97)
        assert ok, f'step {i}: {detail}'
        fracs.append(float(np.mean(np.abs(lb - la) <= 1e-2 + 1e-2 * np.abs(la))))
        if int(a.token) == int(b.token):
            same += 1
        else:
            top2 = np.sort(la)[-2:]
            assert top2[1] - top2[0] <= 2 * (1e-2 + 1e-2 * abs(top2[1])), f'step {i}'
    assert same >= 0.95 * steps, same
    assert np.mean(fracs) >= 0.995, np.mean(fracs)
    assert _lib.device_error() == 0


def test_dataflow_step_tiny(cuda):
    """head_dim 32, 2 q heads per kv head (the reference's tiny test model at N(0, 0.05)), 400 steps."""
    model = gi.build_model(_cfg05(), seed=3).cuda()
    _quantize(model, torch.bfloat16, 'cuda')
    _dataflow_vs_persistent(model, 512, gi.tiny_prompts()[37].cuda(), 400)


@pytest.mark.parametrize('grp', [2, 4])
def test_dataflow_step_head128(cuda, grp):
    """head_dim 128 with 2 (Qwen3-1.7B) or 4 (Qwen3-8B) q heads per kv head, the full 151936-row lm_head."""
    from transformers import Qwen3Config
    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=3,
                      num_attention_heads=4 * grp, num_key_value_heads=4, head_dim=128, max_position_embeddings=512,
                      tie_word_embeddings=True, initializer_range=0.02)
    model = gi.build_model(cfg, seed=7).cuda()
    _quantize(model, torch.bfloat16, 'cuda')
    x = torch.randint(0, cfg.vocab_size, (1, 9), generator=torch.Generator().manual_seed(4)).cuda()
    _dataflow_vs_persistent(model, 300, x, 120)


def test_dataflow_step_wide_mlp(cuda):
    """An intermediate of 8192 (the dataflow step stages inputs up to 8192 wide) with head_dim 128 and 4 q heads
    per kv head, against the persistent step."""
    from transformers import Qwen3Config
    cfg = Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=8192, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128, max_position_embeddings=256,
                      tie_word_embeddings=True, initializer_range=0.05)
    model = gi.build_model(cfg, seed=5).cuda()
    _quantize(model, torch.bfloat16, 'cuda')
    _dataflow_vs_persistent(model, 160, gi.tiny_prompts()[5].cuda(), 120)


def test_dataflow_trace_stamps(cuda):
    """plan->trace on the dataflow step: stamps in order (start, each stage's input ready in CTA 0, the first
    kv head's attention done, token written) and the same tokens as the untraced kernel."""
    from efficientgpt_b200 import _lib
    from efficientgpt_b200.engine import Qwen3Engine
    model = gi.build_model(_cfg05(), seed=3).cuda()
    _quantize(model, torch.bfloat16, 'cuda')
    a = Qwen3Engine(model, 96, step='dataflow')
    b = Qwen3Engine(model, 96, step='dataflow')
    L = a.n_layers
    tr = torch.zeros(5 + 15 * L, dtype=torch.int64, device=cuda)
    b.plan.trace = tr.data_ptr()
    x = gi.tiny_prompts()[5].cuda()
    a.prefill(x)
    b.prefill(x)
    for _ in range(8):
        tr.zero_()
        a.step()
        b.step()
        assert int(a.token) == int(b.token)
        t = tr.cpu().tolist()
        # CTA 0 holds q|k|v tiles of the tiny model; o_proj, gate|up and down_proj tiles too
        stamps = [t[0]] + [t[1 + 5 * l] for l in range(L)] + [t[1 + 5 * L], t[2 + 5 * L]]
        assert all(v > 0 for v in stamps) and stamps == sorted(stamps)
        assert all(t[2 + 5 * l] > 0 for l in range(L))  # attention of kv head 0
    assert _lib.device_error() == 0


def test_gemm_prefill_matches_block_prefill(cuda, monkeypatch):
    """A 300-token prompt through the GEMM prefill (cuBLAS projections with the >16-row rounding, SDPA over the
    prompt, then the last token through the decode step) against the per-stage kernels on 16-row blocks. The two
    round the prompt differently (summation order of the projections, the attention's probability rounding, and
    the last token's single rounding in the decode step against the prefill branch's double rounding), so the
    first logits are held to the hard bound of the long-sequence rule with 95% inside 1e-2; KV caches agree within
    bf16 rounding and the greedy tokens under the near-tie rule."""
    from efficientgpt_b200 import engine as E
    cfg = _cfg05()
    model = gi.build_model(cfg, seed=3).cuda()
    _quantize(model, torch.bfloat16, 'cuda')
    a = E.Qwen3Engine(model, 400, keep_logits=True)
    b = E.Qwen3Engine(model, 400, keep_logits=True)
    x = torch.randint(0, cfg.vocab_size, (1, 300), generator=torch.Generator().manual_seed(11)).cuda()
    monkeypatch.setattr(E, 'PREFILL_GEMM_MIN', 10 ** 9)
    a.prefill(x)
    monkeypatch.setattr(E, 'PREFILL_GEMM_MIN', 256)
    b.prefill(x)
    assert int(a.position) == int(b.position) == 300
    ka, kb = a.kv[:, :, :, :300].float(), b.kv[:, :, :, :300].float()
    assert float((ka - kb).abs().max()) <= 0.05 * float(ka.abs().max())
    ok, detail = parity.logits_close(from_torch(b.logits), from_torch(a.logits), frac=0.95)
    assert ok, detail
    ta, tb, la = [], [], []
    for _ in range(40):
        ta.append(int(a.token))
        tb.append(int(b.token))
        la.append(from_torch(a.logits).copy())
        a.step()
        b.step()
    margins = [float(np.sort(l)[-1] - np.sort(l)[-2]) for l in la]
    tops = [float(l.max()) for l in la]
    ok, first, detail = parity.near_tie_match(ta, margins, tops, tb)
    assert ok, detail


def test_trace_stamps_and_same_tokens(cuda):
    """plan->trace runs the traced instantiation of the persistent kernel: %globaltimer stamps in order (start,
    barrier arrivals and releases, token written) and the same tokens as the untraced kernel."""
    from efficientgpt_b200 import _lib
    from efficientgpt_b200.engine import Qwen3Engine
    model = gi.build_model(_cfg05(), seed=3).cuda()
    _quantize(model, torch.bfloat16, 'cuda')
    a = Qwen3Engine(model, 96, step='persistent')
    b = Qwen3Engine(model, 96, step='persistent')
    L = a.n_layers
    tr = torch.zeros(5 + 15 * L, dtype=torch.int64, device=cuda)
    b.plan.trace = tr.data_ptr()
    x = gi.tiny_prompts()[5].cuda()
    a.prefill(x)
    b.prefill(x)
    for _ in range(8):
        tr.zero_()
        a.step()
        b.step()
        assert int(a.token) == int(b.token)
        t = tr.cpu().tolist()
        stamps = [t[0]] + [t[2 * i - 1] for i in range(1, 3 * L + 1)] + [t[2 + 10 * L]]
        assert all(v > 0 for v in stamps) and stamps == sorted(stamps)
    assert _lib.device_error() == 0


def test_logits_past_one_softmax_block_match_oracle(cuda):
    """Teacher-forced decode from position 120 to 140 (crossing the reference kernel's first 128-key softmax
    block) vs the oracle's block-walk rounding, under the long-sequence logit rule (parity.logits_close: 99%
    within 1e-2 abs / 1e-2 rel, all within 4e-2). The tiny model is re-initialised with N(0, 0.05) weights:
    at the golden's N(0, 0.2) one bf16 rounding flip (CUDA's expf / rsqrtf one fp32 ulp away from numpy's)
    is amplified well past that over a 120-token prompt."""
    from efficientgpt_b200.engine import Qwen3Engine

    model = gi.build_model(_cfg05(), seed=3).cuda()
    _quantize(model, torch.bfloat16, 'cpu')
    eng = Qwen3Engine(model, 192, keep_logits=True)
    x = torch.randint(0, 512, (1, 120), generator=torch.Generator().manual_seed(11))
    eng.prefill(x.cuda())
    ref = Qwen3Ref.from_hf(gi.build_model(_cfg05(), seed=3), 192, 'bf16', semantics='cpu')
    lg = ref.forward(x[0].tolist(), 0)
    ok, detail = parity.logits_close(from_torch(eng.logits), lg)
    assert ok, ('prefill', detail)
    pos = 120
    for i in range(20):
        tok = int(np.argmax(lg))
        eng.token.fill_(tok)
        eng.step()
        lg = ref.forward([tok], pos)
        pos += 1
        ok, detail = parity.logits_close(from_torch(eng.logits), lg)
        assert ok, (pos, detail)
        if int(eng.token) != int(np.argmax(lg)):
            top = np.sort(lg)[-2:]
            assert top[1] - top[0] <= parity.near_tie_threshold(top[1]), pos


@pytest.mark.parametrize('step', ['dataflow', 'persistent'])
def test_persistent_step_in_graph_many_tokens(cuda, step):
    """Many graph replays of a one-kernel step (barrier epochs / LL tags advance every token) stay consistent."""
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    model, _ = _tiny()
    p = GraphGreedyDecoder(model, max_cache_len=256, step=step)
    k = GraphGreedyDecoder(model, max_cache_len=256, persistent=False)
    x = gi.tiny_prompts()[5].cuda()
    for _ in range(3):
        got_p, _ = p.generate(x, 200)
        got_k, _ = k.generate(x, 200)
        n = next((i for i, (u, v) in enumerate(zip(got_p, got_k)) if u != v), len(got_p))
        assert n >= 20, n
    from efficientgpt_b200 import _lib
    assert _lib.device_error() == 0


def test_graph_replay_equals_eager_steps(cuda):
    from efficientgpt_b200.engine import Qwen3Engine
    model, _ = _tiny()
    eng = Qwen3Engine(model, 128)
    x = gi.tiny_prompts()[37].cuda()
    eng.prefill(x)
    eager = []
    for _ in range(20):
        eager.append(int(eng.token))
        eng.step()
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    dec = GraphGreedyDecoder(model, max_cache_len=128)
    got, _ = dec.generate(x, 20)
    assert got == eager


def test_eos_stops_exactly_and_never_leaks_lookahead_tokens(cuda):
    """research/realmodel/test_fast_decode.py:42-56."""
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    model, _ = _tiny()
    dec = GraphGreedyDecoder(model, max_cache_len=128, lookahead=8)
    x = torch.randint(0, 512, (1, 7), generator=torch.Generator().manual_seed(2)).cuda()
    full, _ = dec.generate(x, 60)
    k = max(i for i in range(len(full)) if full[i] not in full[:i])
    assert k > 10, 'EOS must fall well past the first lookahead window'
    streamed = []
    got, st = dec.generate(x, 60, eos_ids={full[k]}, on_token=streamed.append)
    assert got == full[:k + 1]
    assert streamed == got
    again, _ = dec.generate(x, 60)
    assert again == full


def test_guards(cuda):
    """research/realmodel/test_fast_decode.py:58-70."""
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    model, _ = _tiny()
    dec = GraphGreedyDecoder(model, max_cache_len=32)
    with pytest.raises(ValueError):
        dec.generate(torch.zeros((1, 20), dtype=torch.long, device='cuda'), 20)
    with pytest.raises(ValueError):
        dec.generate(torch.zeros((2, 4), dtype=torch.long, device='cuda'), 4)
    with pytest.raises(ValueError):
        dec.generate(torch.zeros((1, 4), dtype=torch.long, device='cuda'), 0)
    out, st = dec.generate(torch.zeros((1, 4), dtype=torch.long, device='cuda'), 3)
    assert (len(out), st['tokens']) == (3, 3)
    assert 'capture_s' in st
    with pytest.raises(ValueError):  # unquantised models are refused (no silent bf16 fallback)
        GraphGreedyDecoder(_tiny(quantize=False)[0], max_cache_len=32)


def test_qwen3_1p7b_shape_matches_reference_golden(cuda, golden):
    """BASELINE config 2 at full size: the reference's 16 greedy tokens (CPU, bf16 scales) vs the native path."""
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    g = golden['qwen3_1p7b']
    model = gi.build_model(gi.qwen3_1p7b_config())
    assert gi.state_hash(model) == g['state_sha256'], 'HF random init changed: golden tokens do not apply'
    model = model.cuda()
    _quantize(model, torch.bfloat16, 'cpu')
    dec = GraphGreedyDecoder(model, max_cache_len=64)
    got, st = dec.generate(gi.big_prompt().cuda(), 16)
    ok, first, detail = parity.near_tie_match(g['tokens'], g['margins'], g['tops'], got)
    assert ok, detail


def _teacher_forced(eng, prompt, tokens, logits_at=None):
    """Feed `tokens` (the reference's greedy sequence) one by one after the prompt; returns the engine's own argmax at
    every step (step 0 = after the prompt) and, with logits_at (per step a list of vocabulary ids), its logits there."""
    eng.prefill(prompt)
    got, at = [int(eng.token)], []
    if logits_at is not None:
        at.append(eng.logits[logits_at[0]].float().cpu().numpy())
    for i, tok in enumerate(tokens[:-1]):
        eng.token.fill_(tok)
        eng.step()
        got.append(int(eng.token))
        if logits_at is not None:
            at.append(eng.logits[logits_at[i + 1]].float().cpu().numpy())
    return got, at


def test_qwen3_1p7b_256_steps_against_reference_golden(cuda):
    """BASELINE config 2 at full size, all 256 greedy steps, against the reference's own run (tests/golden/
    qwen3_1p7b_256.json: HF Qwen3 + the reference's quantize_model, bf16 scales, fp32-accumulated int8 decode branch).
    Teacher-forced along the reference's tokens, so every step is compared at the reference's own context.

    The golden's diagnostic calibrates the rule: the reference forward itself, with only the decode GEMV's fp32
    summation replaced by the exact sum, moves the two decisive logits of a step (the reference's top-1 and
    runner-up, bf16 values in [3.5, 5]) by up to 5 bf16 ulps (0.078), keeps 94% of them within the north star's
    1e-2 abs + 1e-2 rel, and picks a different token at 18 of 256 steps, all at top-2 margins <= 2 ulps. This
    model's greedy choices are that close to ties. The rule:
    * every decisive logit within 8 bf16 ulps (of the reference value's binade) of the reference's;
    * at least 224 of 256 steps (87.5%) pick the reference's token;
    * a step may pick a different token only where it picks the reference's runner-up, or where the reference's
      top-2 margin is within twice the north star tolerance (logits that meet it can swap the order).
    Free-running, the first divergence must sit at such a step. The identical-step count and the fraction within
    the north star tolerance are reported as warnings."""
    import json
    import warnings
    from pathlib import Path
    from efficientgpt_b200.engine import Qwen3Engine
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder
    g = json.loads(Path(gi.__file__).with_name('qwen3_1p7b_256.json').read_text())
    model = gi.build_model(gi.qwen3_1p7b_config())
    assert gi.state_hash(model) == g['state_sha256'], 'HF random init changed: golden tokens do not apply'
    model = model.cuda()
    _quantize(model, torch.bfloat16, 'cpu')
    prompt = torch.tensor([g['prompt']], device=cuda)
    eng = Qwen3Engine(model, 32 + 256, keep_logits=True)
    pairs = [[g['tokens'][i], g['runner_up'][i]] for i in range(256)]
    got, at = _teacher_forced(eng, prompt, g['tokens'], logits_at=pairs)
    want = np.array([[g['tops'][i], g['tops'][i] - g['margins'][i]] for i in range(256)])
    have = np.array(at)
    err = np.abs(have - want)
    ulps = err / 2.0 ** (np.floor(np.log2(np.abs(want))) - 7)
    within = float(np.mean(err <= 1e-2 + 1e-2 * np.abs(want)))
    diff = [i for i in range(256) if got[i] != g['tokens'][i]]
    swap_ok = [g['margins'][i] <= 2 * (1e-2 + 1e-2 * abs(g['tops'][i])) for i in range(256)]
    bad = [(i, g['margins'][i]) for i in diff if not (swap_ok[i] or got[i] == g['runner_up'][i])]
    ties = sum(1 for i in diff if g['margins'][i] == 0.0)
    dg = g['exact_sum_diagnostic']
    warnings.warn(f'config 2 x 256 teacher-forced ({eng.step_kind} step): {256 - len(diff)}/256 steps pick the '
                  f"reference's token; {len(diff)} differ ({ties} at exact ties of the reference's bf16 logits); "
                  f'decisive logits: max {ulps.max():.0f} ulps ({err.max():.4g}), {within:.2%} within 1e-2 abs+rel; '
                  f'reference forward with only the exact-sum GEMV: {dg["identical"]}/256, '
                  f'{dg["decisive_logits_within_1e-2_abs_rel"]:.2%} within')
    assert ulps.max() <= 8, f'decisive logits: max {ulps.max()} bf16 ulps'
    assert len(diff) <= 32, diff
    assert not bad, f'steps differing where the decisive logits cannot swap within tolerance: {bad}'
    dec = GraphGreedyDecoder(model, max_cache_len=32 + 256)
    free, _ = dec.generate(prompt, 256)
    first = next((i for i in range(256) if free[i] != g['tokens'][i]), None)
    warnings.warn(f'config 2 x 256 free-running: first divergence at step {first}')
    assert first is None or swap_ok[first] or free[first] == g['runner_up'][first], (first, g['margins'][first])
