"""CPU restatement of the reference's stochastic decoding transforms (test infrastructure only: the checker of
efficientgpt_b200.sampling, never on the product path).

Follows BagelsFun/efficientgpt research/phase5/sampling.py:
  filtered_probs  (39-59)  x = logits.float() / T; top-k masks x below the k-th largest (duplicates counted, ties
                           kept); softmax; top-p drops, in the stable descending order of p, every token whose
                           exclusive prefix mass is >= top_p, then renormalises
  sample_from     (62-73)  cdf = cumsum(p); token = searchsorted(cdf, u * cdf[-1], right=True), clamped to the last
                           index with p > 0
in numpy float32 with sequential prefix sums (the reference's CPU cumsum order). Pinned against the reference's own
outputs by tests/golden/sampling_cases.json (tests/golden/make_golden_sampling.py imports the reference).

`boundary(...)` reports how close a draw is to a decision boundary of the arithmetic (the CDF step it falls in, the
top-p cut), which is where two correct implementations with different fp32 summation orders may disagree.
"""
import numpy as np


def filtered_probs(logits, temperature=1.0, top_k=None, top_p=None):
    """logits [V] (any float dtype) -> float32 probabilities [V] and, with top_p, the exclusive prefix masses of the
    stable descending order (for boundary checks; None otherwise)."""
    x = np.asarray(logits, dtype=np.float32) / np.float32(temperature)
    v = x.shape[-1]
    if top_k is not None and top_k < v:
        kth = np.sort(x)[::-1][top_k - 1]
        x = np.where(x < kth, np.float32(-np.inf), x)
    m = np.max(x)
    e = np.exp(x - m, dtype=np.float32)
    s = np.cumsum(e, dtype=np.float32)[-1]  # sequential fp32 sum
    p = (e / s).astype(np.float32)
    excl = None
    if top_p is not None and top_p < 1:
        order = np.argsort(-p, kind='stable')
        ordered = p[order]
        cs = np.cumsum(ordered, dtype=np.float32)
        excl = (cs - ordered).astype(np.float32)
        drop_sorted = excl >= np.float32(top_p)
        drop = np.zeros(v, dtype=bool)
        drop[order] = drop_sorted
        p = np.where(drop, np.float32(0), p)
        tot = np.cumsum(p, dtype=np.float32)[-1]
        p = (p / tot).astype(np.float32)
    return p, excl


def sample_from(p, u):
    """Inverse CDF on float32 probabilities [V] with one uniform u in [0, 1)."""
    cdf = np.cumsum(p, dtype=np.float32)
    target = np.float32(np.float32(u) * cdf[-1])
    tok = int(np.searchsorted(cdf, target, side='right'))
    nz = np.nonzero(p > 0)[0]
    last = int(nz[-1]) if nz.size else 0
    return min(tok, last)


def sample(logits, u, temperature=1.0, top_k=None, top_p=None):
    p, _ = filtered_probs(logits, temperature, top_k, top_p)
    return sample_from(p, u)


def _probs64(logits, temperature, top_k):
    x = np.asarray(logits, dtype=np.float32) / np.float32(temperature)  # the reference's fp32 x
    if top_k is not None and top_k < x.shape[-1]:
        kth = np.sort(x)[::-1][top_k - 1]
        x = np.where(x < kth, np.float32(-np.inf), x)
    x = x.astype(np.float64)
    e = np.exp(x - np.max(x))
    return e / e.sum()


def token_ok(logits, u, token, temperature=1.0, top_k=None, top_p=None, tol=1e-4):
    """Whether `token` is a correct draw for uniform u up to rounding: computed in fp64 from the reference's fp32 x,
    the token must be kept by top-p under some cut within `tol` of top_p (the exclusive prefix mass of the stable
    descending order) and u must fall within `tol` of the token's CDF step (renormalised over that kept set).
    `tol` covers the reference's own fp32 sums (a sequential fp32 cumsum over 151936 terms drifts by ~1e-5)."""
    p = _probs64(logits, temperature, top_k)
    sets = [p]
    if top_p is not None and top_p < 1:
        order = np.argsort(-p, kind='stable')
        excl = np.cumsum(p[order]) - p[order]
        lo, hi = max(1, int(np.sum(excl < top_p - tol))), max(1, int(np.sum(excl < top_p + tol)))
        sets = []
        for c in range(lo, hi + 1):
            m = np.zeros(len(p), dtype=bool)
            m[order[:c]] = True
            sets.append(np.where(m, p, 0.0))
    for q in sets:
        if q[token] <= 0:
            continue
        cdf = np.cumsum(q / q.sum())
        lo = cdf[token - 1] if token > 0 else 0.0
        if lo - tol <= u < cdf[token] + tol:
            return True
    return False


def boundary(logits, u, temperature=1.0, top_k=None, top_p=None):
    """Relative distance of this draw from the nearest decision boundary: the CDF steps around u * total, and the
    top-p cut (|exclusive prefix mass - top_p| nearest to top_p). Small values (< 1e-5) mark draws that fp32
    summation order alone may flip."""
    p, excl = filtered_probs(logits, temperature, top_k, top_p)
    cdf = np.cumsum(p.astype(np.float64))
    t = float(u) * cdf[-1]
    j = int(np.searchsorted(cdf, t, side='right'))
    lo = cdf[j - 1] if j > 0 else 0.0
    hi = cdf[j] if j < len(cdf) else cdf[-1]
    d = min(abs(t - lo), abs(hi - t)) / max(cdf[-1], 1e-30)
    if excl is not None:
        d = min(d, float(np.min(np.abs(excl.astype(np.float64) - float(top_p)))))
    return d
