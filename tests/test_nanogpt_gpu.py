"""GPU parity of the nanoGPT int8 decode (efficientgpt_b200/nanogpt.py) against the reference's
greedy tokens and logits (tests/golden/nanogpt_tiny.npz, made by tests/golden/make_golden_nanogpt.py from the
reference's research/phase4 decoder) and against the oracle (oracle/nanogpt_ref.py) at config-1 size.
Mirrors research/phase4/test_decoder.py."""
import json

import numpy as np
import pytest
import torch

from oracle.bf16 import from_torch
from oracle.nanogpt_ref import NanoGPTRef

pytestmark = pytest.mark.gpu


def _golden():
    from conftest import ROOT
    z = np.load(ROOT / 'tests' / 'golden' / 'nanogpt_tiny.npz')
    meta = json.loads((ROOT / 'tests' / 'golden' / 'nanogpt.json').read_text())
    return {k[len('param.'):]: z[k] for k in z.files if k.startswith('param.')}, meta, z


def _quantize_cpu_semantics(model, params):
    """quantize_model, then the golden's quantiser arithmetic (the reference ran on the CPU, where max|w| / 127.0
    is a true division; on the GPU PyTorch multiplies by fl32(1/127))."""
    from efficientgpt_b200.int8_linear import Int8Linear, quantize_model
    orig = {n: m.weight.detach().float().clone() for n, m in model.named_modules() if isinstance(m, torch.nn.Linear)}
    quantize_model(model)
    for n, m in model.named_modules():
        if isinstance(m, Int8Linear):
            w = orig[n]
            amax = w.abs().amax(1)
            s = (amax / torch.full_like(amax, 127.0)).clamp_min(1e-12)
            m.qweight.copy_(torch.round(w / s[:, None]).clamp(-127, 127).to(torch.int8))
            m.scale.copy_(s)
    return model


def _tiny_model():
    from efficientgpt_b200.nanogpt import GPT, GPTConfig
    params, meta, z = _golden()
    c = meta['config']
    model = GPT(GPTConfig(block_size=c['block_size'], vocab_size=c['vocab_size'], n_layer=c['n_layer'],
                          n_head=c['n_head'], n_embd=c['n_embd'], bias=c['bias'])).load_params(params).cuda().eval()
    return _quantize_cpu_semantics(model, params), params, meta, z


def _near_tie_ok(want, margins, got):
    for i, (a, b) in enumerate(zip(want, got)):
        if a != b:
            return margins[i] <= 1e-4, i
    return True, None


def test_tiny_tokens_and_logits_match_reference_golden(cuda):
    from efficientgpt_b200.nanogpt import GraphDecoder, StaticKVDecoder
    model, params, meta, z = _tiny_model()
    exact = 0
    for run in meta['runs']:
        prompt = torch.tensor([run['prompt']], dtype=torch.long, device='cuda')
        n = len(run['tokens'])
        dec = StaticKVDecoder(model, keep_logits=True)
        logits = dec.reset(prompt)
        np.testing.assert_allclose(from_torch(logits), z[f"logits_first_{len(run['prompt'])}"], atol=2e-5, rtol=1e-4)
        got = dec.generate_eager(prompt, n)[0, len(run['prompt']):].tolist()
        ok, first = _near_tie_ok(run['tokens'], run['margins'], got)
        assert ok, (run['prompt'], first, got, run['tokens'])
        exact += first is None
        graph = GraphDecoder(model, prompt).generate(prompt, n)[0, len(run['prompt']):].tolist()
        assert graph == got
    assert exact >= 3


def test_config1_decode_matches_oracle_teacher_forced(cuda):
    """BASELINE config 1 size (6 layers, 6 heads, 384 dims, block 256, vocab 50304), N(0, 0.02) init: 64-token
    prompt, 64 teacher-forced steps; fp32 logits within 1e-4 relative of the oracle, tokens equal but at near-ties."""
    from efficientgpt_b200.int8_linear import quantize_model
    from efficientgpt_b200.nanogpt import GPT, GPTConfig, NanoGPTEngine
    cfg = GPTConfig(block_size=256, vocab_size=50304, n_layer=6, n_head=6, n_embd=384, bias=True)
    model = GPT(cfg, seed=0).cuda().eval()
    params = {n: p.detach().cpu().numpy().copy() for n, p in model.named_parameters()}
    params['lm_head.weight'] = params['transformer.wte.weight']
    quantize_model(model)
    eng = NanoGPTEngine(model, keep_logits=True)
    ref = NanoGPTRef(params, {'block_size': 256, 'n_layer': 6, 'n_head': 6, 'n_embd': 384}, semantics='cuda')
    prompt = torch.randint(0, 50304, (64,), generator=torch.Generator().manual_seed(0))
    eng.prefill(prompt.cuda())
    lg = ref.forward(prompt.tolist(), 0)
    np.testing.assert_allclose(from_torch(eng.logits), lg, atol=1e-4, rtol=1e-4)
    pos, same = 64, 0
    for i in range(64):
        tok = int(np.argmax(lg))
        eng.token.fill_(tok)
        eng.step()
        lg = ref.forward([tok], pos)
        pos += 1
        assert int(eng.position) == pos
        np.testing.assert_allclose(from_torch(eng.logits), lg, atol=1e-4, rtol=1e-4, err_msg=f'step {i}')
        if int(eng.token) == int(np.argmax(lg)):
            same += 1
        else:
            top = np.sort(lg)[-2:]
            assert top[1] - top[0] <= 1e-4, i
    assert same >= 62


def test_guards(cuda):
    """research/phase4/test_decoder.py:35-46: batch mismatch and context overflow are refused."""
    from efficientgpt_b200.nanogpt import StaticKVDecoder
    model, _, _, _ = _tiny_model()
    dec = StaticKVDecoder(model)
    with pytest.raises(ValueError):
        dec.generate_eager(torch.randint(0, 128, (2, 5), device='cuda'), 3)
    with pytest.raises(ValueError):
        dec.generate_eager(torch.randint(0, 128, (1, 31), device='cuda'), 2)
    with pytest.raises(ValueError):
        StaticKVDecoder(model, batch=2)
    out = dec.generate_eager(torch.randint(0, 128, (1, 29), device='cuda'), 3)
    assert out.shape == (1, 32)
