"""On-device sampling (efficientgpt_b200.sampling, csrc/sampling.cu) against the reference's sampler.

CPU: the oracle restatement (oracle/sampling_ref.py) reproduces the reference's own draws (tests/golden/
sampling_cases.json, made by importing research/phase5/sampling.py) and its known-answer tables; the config errors.
GPU: egpt_sample against the same golden draws and the oracle on fresh rows (tokens identical except draws the
oracle's fp64 check accepts as within rounding of a CDF step or of the top-p cut), the reference's known-answer tables, a chi-square test of
the drawn distribution (research/phase5/test_sampling.py:97-137), determinism, the zeroed workspace contract, and
the sampled graph decoder on a tiny Qwen3.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import sampling_ref as sr

G = json.loads((Path(gi.__file__).with_name('sampling_cases.json')).read_text())


# tokens of the known-answer row log([0.15, 0.5, 0.05, 0.3]) whose exact exclusive prefix mass equals top_p
_ON_CUT = {'0.5': {3}, '0.6': set(), '0.95': {2}, '0.99': set(), '1e-09': set()}


def _row(c):
    x = gi.sampling_logits(c['V'], c['seed'], c['scale'], torch.bfloat16 if c['dtype'] == 'bf16' else torch.float32)
    u = gi.sampling_uniforms(G['n_uniforms'], c['seed'])
    assert gi.sha(x) == c['sha_logits'] and gi.sha(u) == c['sha_u'], 'torch CPU generator changed'
    return x, u


def _cfg(c):
    k = c['cfg']
    return k.get('temperature', 1.0), k.get('top_k'), k.get('top_p')


def test_oracle_matches_reference_draws():
    """The restatement reproduces the reference's draws: identical tokens except where the reference's own fp32
    sums decide (draws within the tolerance of token_ok of a CDF step or of the top-p cut), and the reference's
    tokens are themselves correct draws by token_ok."""
    same, total = 0, 0
    for c in G['cases']:
        x, u = _row(c)
        t, k, p = _cfg(c)
        xf = x.float().numpy()
        for i in range(len(u)):
            want = c['tokens'][i]
            assert sr.token_ok(xf, float(u[i]), want, t, k, p), (c['V'], c['seed'], c['cfg'], i)
            got = sr.sample(xf, float(u[i]), t, k, p)
            total += 1
            same += got == want
            if got != want:
                assert sr.token_ok(xf, float(u[i]), got, t, k, p), (c['V'], c['seed'], c['cfg'], i, got, want)
    assert same >= 0.97 * total, (same, total)


def test_oracle_known_answer_tables():
    """research/phase5/test_sampling.py:25-30, 49-53 as the reference evaluated them. Two rows sit exactly on the
    cut (the exclusive mass of token 3 is 0.5 = top_p, of token 2 is 0.95 = top_p), where fp32 rounding of the
    softmax decides; the kept sets must agree elsewhere and may differ there only by that token."""
    lg = np.log(np.array([0.15, 0.5, 0.05, 0.3], dtype=np.float32))
    for p, kept in G['top_p_keep'].items():
        probs, _ = sr.filtered_probs(lg, 1.0, None, float(p))
        got = set(np.nonzero(probs)[0].tolist())
        assert got ^ set(kept) <= _ON_CUT[p], (p, got, kept)
    ic = G['inverse_cdf']
    probs = np.array(ic['probs'], dtype=np.float32)
    assert [sr.sample_from(probs, u) for u in ic['u']] == ic['tokens'] == [0, 0, 2, 2, 2]


def test_config_errors():
    from efficientgpt_b200.sampling import SamplingConfig
    for kw in [dict(temperature=0), dict(top_k=0), dict(top_p=0), dict(top_p=1.5)]:
        with pytest.raises(ValueError):
            SamplingConfig(**kw)


def test_sampling_exports_and_workspace_size():
    from efficientgpt_b200 import _lib
    lib = _lib.load()
    one, two, three = (lib.egpt_sample_ws_bytes(r) for r in (1, 2, 3))
    assert one > 0 and three - two == two - one > 0 and one % 16 == 0 and lib.egpt_sample_ws_bytes(0) == 0


# ------------------------------------------------------------------------------------------------ GPU
def _gpu_sample(x, u, t, k, p, ws=None):
    from efficientgpt_b200.sampling import SamplingConfig, sample
    cfg = SamplingConfig(t, k, p)
    return sample(x.cuda().reshape(1, -1), cfg, torch.tensor([float(u)], device='cuda'), ws=ws)


@pytest.mark.gpu
def test_gpu_matches_reference_draws(cuda):
    from efficientgpt_b200 import _lib
    from efficientgpt_b200.sampling import SamplingConfig, sample, sample_ws
    bad, near, total = [], 0, 0
    for c in G['cases']:
        x, u = _row(c)
        t, k, p = _cfg(c)
        cfg = SamplingConfig(t, k, p)
        xs = x.cuda().reshape(1, -1).expand(len(u), -1).contiguous()  # one row per uniform
        got = sample(xs, cfg, u.cuda()).flatten().tolist()
        xf = x.float().numpy()
        for i, (g, want) in enumerate(zip(got, c['tokens'])):
            total += 1
            if g == want:
                near += 1
            elif not sr.token_ok(xf, float(u[i]), g, t, k, p):
                bad.append((c['V'], c['seed'], c['cfg'], i, g, want))
    assert _lib.device_error() == 0
    assert not bad, bad[:5]
    assert near >= 0.97 * total, (near, total)  # identical draws


@pytest.mark.gpu
def test_gpu_known_answer_tables(cuda):
    from efficientgpt_b200.sampling import SamplingConfig, sample
    lg = torch.log(torch.tensor([0.15, 0.5, 0.05, 0.3]))
    us = torch.linspace(0, 1 - 2 ** -24, 257)
    for p, kept in G['top_p_keep'].items():
        toks = sample(lg.cuda().reshape(1, -1).expand(len(us), -1).contiguous(), SamplingConfig(1.0, top_p=float(p)),
                      us.cuda()).flatten().tolist()
        got = set(toks)  # 257 evenly spaced draws reach every kept token (the smallest holds 5% of the mass)
        assert got ^ set(kept) <= _ON_CUT[p], (p, sorted(got), kept)
    # zero-probability tokens are never drawn, and the mapping of the reference's table
    ic = G['inverse_cdf']
    lg = torch.log(torch.tensor(ic['probs']))
    toks = sample(lg.cuda().reshape(1, -1).expand(5, -1).contiguous(), SamplingConfig(1.0),
                  torch.tensor(ic['u'], device='cuda')).flatten().tolist()
    for t, u, want in zip(toks, ic['u'], ic['tokens']):
        assert t in (0, 2)
        if abs(u - 0.25) > 1e-6:  # u = 0.25 sits on the CDF step (exact there only with exact probabilities)
            assert t == want, (u, t, want)


@pytest.mark.gpu
def test_gpu_fresh_rows_against_oracle(cuda):
    from efficientgpt_b200.sampling import SamplingConfig, sample
    rng = np.random.default_rng(7)
    bad, near = [], 0
    for trial in range(12):
        v = int(rng.choice([7, 300, 4096, 151936]))
        x = torch.tensor(rng.standard_normal(v) * rng.choice([0.3, 1.0, 4.0]), dtype=torch.float32).to(torch.bfloat16)
        x[rng.integers(0, v, size=min(v, 20))] = x.max()  # ties at the top
        t = float(rng.choice([0.5, 1.0, 1.7]))
        k = [None, 1, 5, 40, v + 3][trial % 5]
        p = [None, 0.3, 0.9, 0.999][trial % 4]
        u = torch.rand(32, generator=torch.Generator().manual_seed(trial))
        got = sample(x.cuda().reshape(1, -1).expand(32, -1).contiguous(), SamplingConfig(t, k, p), u.cuda())
        xf = x.float().numpy()
        for i, g in enumerate(got.flatten().tolist()):
            want = sr.sample(xf, float(u[i]), t, k, p)
            near += g == want
            if g != want and not sr.token_ok(xf, float(u[i]), g, t, k, p):
                bad.append((v, t, k, p, i, g, want))
    assert not bad, bad[:5]
    assert near >= 0.95 * 12 * 32, near  # identical draws


@pytest.mark.gpu
def test_gpu_distribution_chi_square(cuda):
    """All draws of one row of V = 8 logits (exact probabilities from the oracle in fp64) against 100k draws."""
    from efficientgpt_b200.sampling import SamplingConfig, sample
    from scipy.stats import chisquare
    x = torch.tensor([1.2, -0.3, 0.8, 2.0, 0.0, -1.5, 1.9, 0.4])
    configs = [SamplingConfig(1.0), SamplingConfig(0.7, top_k=3), SamplingConfig(1.3, top_p=0.8),
               SamplingConfig(0.9, top_k=5, top_p=0.9)]
    n = 100_000
    for i, cfg in enumerate(configs):
        u = torch.rand(n, generator=torch.Generator().manual_seed(100 + i)).cuda()
        toks = torch.cat([sample(x.cuda().reshape(1, -1).expand(m.numel(), -1).contiguous(), cfg, m)
                          for m in u.split(50_000)]).flatten().cpu()
        counts = torch.bincount(toks, minlength=8).double().numpy()
        p, _ = sr.filtered_probs(x.numpy(), cfg.temperature, cfg.top_k, cfg.top_p)
        p = p.astype(np.float64) / p.sum()
        assert counts[p == 0].sum() == 0, cfg
        keep = p > 0
        stat = chisquare(counts[keep], p[keep] / p[keep].sum() * counts[keep].sum())
        assert stat.pvalue > 1e-3, (cfg, stat)


@pytest.mark.gpu
def test_gpu_deterministic_and_workspace_left_zero(cuda):
    from efficientgpt_b200.sampling import SamplingConfig, sample, sample_ws
    x = gi.sampling_logits(151936, 3, 2.0).cuda().reshape(1, -1).expand(4, -1).contiguous()
    u = torch.rand(4, generator=torch.Generator().manual_seed(1)).cuda()
    ws = sample_ws(4, 'cuda')
    cfg = SamplingConfig(0.8, top_k=50, top_p=0.9)
    a = sample(x, cfg, u, ws=ws)
    assert int(ws.count_nonzero()) == 0
    b = sample(x, cfg, u, ws=ws)
    assert torch.equal(a, b)


@pytest.mark.gpu
def test_gpu_u_index_advances(cuda):
    from efficientgpt_b200.sampling import SamplingConfig, sample
    x = gi.sampling_logits(1000, 2, 3.0).cuda().reshape(1, -1)
    u = torch.rand(1, 6, generator=torch.Generator().manual_seed(3)).cuda()
    idx = torch.zeros((), dtype=torch.int64, device='cuda')
    cfg = SamplingConfig(1.0, top_p=0.9)
    got = [int(sample(x, cfg, u, u_index=idx)) for _ in range(6)]
    assert int(idx) == 6
    want = [int(sample(x, cfg, u[:, i].contiguous())) for i in range(6)]
    assert got == want


@pytest.mark.gpu
def test_gpu_errors(cuda):
    from efficientgpt_b200 import _lib
    from efficientgpt_b200.sampling import SamplingConfig, sample
    x = torch.zeros(1, 10, dtype=torch.bfloat16, device='cuda')
    with pytest.raises(ValueError):
        sample(x, SamplingConfig(1.0), torch.zeros(1, dtype=torch.float64, device='cuda'))
    with pytest.raises(ValueError):
        sample(x.cpu(), SamplingConfig(1.0), torch.zeros(1))
    lib = _lib.load()
    rc = lib.egpt_sample(x.data_ptr(), _lib.EGPT_BF16, 1, 10, 10, 0.0, 0, 1.0, x.data_ptr(), 1, None, x.data_ptr(), 1,
                         x.data_ptr(), 1 << 20, None)
    assert rc == _lib.EGPT_ERR_ARG and 'temperature' in _lib.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize('step', ['dataflow', 'sequence'])
def test_sampled_graph_decoder(cuda, step):
    """SampledGraphDecoder on the tiny Qwen3: every emitted token is the draw egpt_sample makes from the engine's
    own logits at that step with that step's uniform (a teacher-forced engine replays the emitted tokens), the
    stream is deterministic given the uniforms, and top_k = 1 reproduces greedy decoding."""
    from efficientgpt_b200.engine import Qwen3Engine
    from efficientgpt_b200.fast_decode import GraphGreedyDecoder, SampledGraphDecoder
    from efficientgpt_b200.int8_linear import quantize_model
    from efficientgpt_b200.sampling import SamplingConfig, draw_uniforms, sample
    model = gi.build_model(gi.tiny_config(), seed=3).cuda()
    quantize_model(model, scale_dtype=torch.bfloat16)
    prompt = gi.tiny_prompts()[5].cuda().reshape(1, -1)
    n = 40
    cfg = SamplingConfig(0.9, top_k=20, top_p=0.9)
    dec = SampledGraphDecoder(model, prompt.shape[1] + n, cfg, step=step)
    u = draw_uniforms(1, n, torch.Generator(device='cuda').manual_seed(11))
    toks, st = dec.generate(prompt, n, u)
    assert st['tokens'] == n and len(toks) == n
    again, _ = dec.generate(prompt, n, u)
    assert again == toks
    ref = Qwen3Engine(model, prompt.shape[1] + n, keep_logits=True, step=step)
    ref.prefill(prompt)
    for i in range(n):
        want = int(sample(ref.logits.view(1, -1), cfg, u[:, i].contiguous()))
        assert toks[i] == want, i
        ref.token.fill_(toks[i])
        ref.step()
    greedy, _ = GraphGreedyDecoder(model, prompt.shape[1] + n, step=step).generate(prompt, n)
    one, _ = SampledGraphDecoder(model, prompt.shape[1] + n, SamplingConfig(1.0, top_k=1), step=step).generate(
        prompt, n, u)
    assert one == greedy
