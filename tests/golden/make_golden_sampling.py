"""Generate tests/golden/sampling_cases.json: tokens drawn by the REFERENCE's own sampler.

    python tests/golden/make_golden_sampling.py --reference /path/to/efficientgpt

Runs once in the development container (CPU) and its output is committed; nothing on the test or GPU side imports
the reference. For each case the logits row is rebuilt from (V, seed, scale, dtype) by golden_inputs.sampling_logits
and the uniforms by golden_inputs.sampling_uniforms; the tokens are
research/phase5/sampling.py sample_from(filtered_probs(logits[None], SamplingConfig(...)), u) for each uniform.
Also recorded: the reference's own known-answer tables of research/phase5/test_sampling.py (top-p keep sets on
log([0.15, 0.5, 0.05, 0.3]); the inverse-CDF mapping on [0.25, 0, 0.75, 0]) evaluated by the reference.
"""
import argparse
import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import golden_inputs as gi  # noqa: E402

CONFIGS = [dict(temperature=1.0), dict(temperature=0.7, top_k=3), dict(temperature=1.3, top_p=0.8),
           dict(temperature=0.9, top_k=5, top_p=0.9), dict(temperature=0.8, top_k=50, top_p=0.9),
           dict(temperature=1.0, top_p=0.95), dict(temperature=1.2, top_k=1000), dict(temperature=1.0, top_k=1),
           dict(temperature=0.6, top_p=0.5)]
ROWS = [(64, 1, 1.0, 'bf16'), (1000, 2, 3.0, 'bf16'), (151936, 3, 2.0, 'bf16'), (151936, 4, 6.0, 'bf16'),
        (50304, 5, 2.0, 'f32'), (1000, 6, 0.5, 'f32')]
N_U = 24


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    from research.phase5.sampling import SamplingConfig, filtered_probs, sample_from
    cases = []
    for v, seed, scale, dt in ROWS:
        x = gi.sampling_logits(v, seed, scale, torch.bfloat16 if dt == 'bf16' else torch.float32)
        u = gi.sampling_uniforms(N_U, seed)
        for ci, cfg in enumerate(CONFIGS):
            p = filtered_probs(x[None], SamplingConfig(**cfg))
            toks = [int(sample_from(p, u[i:i + 1])[0, 0]) for i in range(N_U)]
            cases.append({'V': v, 'seed': seed, 'scale': scale, 'dtype': dt, 'cfg': cfg, 'tokens': toks,
                          'sha_logits': gi.sha(x), 'sha_u': gi.sha(u)})
    # the reference's known-answer tables (research/phase5/test_sampling.py:25-30, 49-53)
    lg = torch.log(torch.tensor([[0.15, 0.5, 0.05, 0.3]]))
    keep = {}
    for p in (0.5, 0.6, 0.95, 0.99, 1e-9):
        pr = filtered_probs(lg, SamplingConfig(1.0, top_p=p))
        keep[repr(p)] = sorted(torch.nonzero(pr[0]).flatten().tolist())
    probs = torch.tensor([[0.25, 0.0, 0.75, 0.0]]).repeat(5, 1)
    u = torch.tensor([0.0, 0.2499, 0.25, 0.9999, 1 - 2 ** -24])
    mapping = sample_from(probs, u).flatten().tolist()
    out = {'reference': 'research/phase5/sampling.py filtered_probs + sample_from (CPU)', 'torch': torch.__version__,
           'n_uniforms': N_U, 'cases': cases, 'top_p_keep': keep, 'inverse_cdf': {'probs': [0.25, 0.0, 0.75, 0.0],
           'u': u.tolist(), 'tokens': mapping}}
    (HERE / 'sampling_cases.json').write_text(json.dumps(out, indent=1))
    print('wrote sampling_cases.json', len(cases), 'cases')


if __name__ == '__main__':
    main()
