"""Token-parity rule for greedy decoding with bf16 logits (test infrastructure; see oracle/__init__.py).

The reference accepts a divergence between two greedy decoders only at a near-tie of the reference logits
(BagelsFun/efficientgpt research/phase5/benchmark_review.py:54-67: first divergence, top-1/top-2 margin < 1e-2).
That rule was written for fp32 logits. The int8 path's logits are bf16 (modeling_qwen3.py:503-505 has no
upcast), whose spacing near |logit| = 4 is 0.03125, so exact ties (margin 0) and one-ulp margins are common
and any change of fp32 summation order can flip them. The rule used here: identical tokens up to the first
divergence, and that divergence must sit where the reference's margin is within two bf16 ulps of its top-1
logit (or below 1e-2). Steps after a legitimate divergence are not compared (the contexts differ).
"""
import math


def bf16_ulp(v):
    """Spacing of bf16 values at |v| (normal range)."""
    a = abs(float(v))
    if a == 0.0 or not math.isfinite(a):
        return 0.0
    return 2.0 ** (math.floor(math.log2(a)) - 7)


def near_tie_threshold(top):
    return max(1e-2, 2.0 * bf16_ulp(top))


def near_tie_match(ref_tokens, ref_margins, ref_tops, got_tokens):
    """Returns (ok, first_divergence_index_or_None, detail)."""
    n = min(len(ref_tokens), len(got_tokens))
    if len(got_tokens) != len(ref_tokens):
        return False, None, f'length {len(got_tokens)} != {len(ref_tokens)}'
    for i in range(n):
        if ref_tokens[i] != got_tokens[i]:
            thr = near_tie_threshold(ref_tops[i])
            ok = ref_margins[i] <= thr
            return ok, i, f'step {i}: ref margin {ref_margins[i]:.5g}, near-tie threshold {thr:.5g}'
    return True, None, 'identical'


def logits_close(got, want, atol=1e-2, rtol=1e-2, frac=0.99, hard=4e-2):
    """Logit rule for long sequences. fp32 transcendental functions of CUDA (expf in softmax and SiLU, rsqrtf in
    RMSNorm) and of numpy can differ by one fp32 ulp; now and then that moves a value across a bf16 rounding
    boundary, and a high-gain model carries the flip into a few bf16 ulps of the logits. The rule: at least
    `frac` of the logits within atol + rtol |want|, and every logit within `hard` + rtol |want|.
    Returns (ok, detail)."""
    import numpy as np
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    d = np.abs(got - want)
    soft = d <= atol + rtol * np.abs(want)
    firm = d <= hard + rtol * np.abs(want)
    ok = bool(soft.mean() >= frac and firm.all())
    return ok, f'within 1e-2: {soft.mean():.4f}, max |diff| {d.max():.4g}'
