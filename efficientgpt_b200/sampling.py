"""On-device stochastic decoding: temperature -> top-k -> top-p -> inverse CDF, on B200 CUDA kernels.

Drop-in for BagelsFun/efficientgpt research/phase5/sampling.py: the same SamplingConfig (and its errors), the same
contract for the draws (one U[0, 1) per row and generated token, pre-drawn by the caller: draw_uniforms), and
`sample(logits, cfg, u)`, which returns what `sample_from(filtered_probs(logits, cfg), u)` returns
(research/phase5/sampling.py:39-71) without leaving the GPU: egpt_sample in libegpt_b200.so (csrc/sampling.cu),
a chain of small kernels with integer histograms and fixed-order sums (deterministic; no sort).

The probabilities themselves are never materialised; filtered_probs / sample_from of the reference are restated
for the CPU in oracle/sampling_ref.py (test infrastructure). Given the same logits and uniforms the tokens are
the reference's except for draws within a few ulps of a CDF boundary or top_p within a few ulps of a prefix sum
(the reference's fp32 cumsum against exact fixed-point sums here).
"""
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib as L
from .ops import _cuda, _dt, _p, _stream


@dataclass(frozen=True)
class SamplingConfig:
    """research/phase5/sampling.py:24-37: temperature > 0, top_k >= 1 or None, top_p in (0, 1] or None."""
    temperature: float = 1.0
    top_k: Optional[int] = None
    top_p: Optional[float] = None

    def __post_init__(self):
        if not self.temperature > 0:
            raise ValueError('temperature must be > 0; use the greedy decoders for temperature 0')
        if self.top_k is not None and self.top_k < 1:
            raise ValueError('top_k must be >= 1')
        if self.top_p is not None and not 0 < self.top_p <= 1:
            raise ValueError('top_p must be in (0, 1]')


def draw_uniforms(batch, count, generator, device='cuda'):
    """One U[0, 1) per row and generated token (research/phase5/sampling.py:73-75)."""
    return torch.rand((batch, count), generator=generator, device=device, dtype=torch.float32)


def sample_ws(rows, device):
    """Workspace of egpt_sample for `rows` rows (zeroed; every call leaves it zeroed)."""
    return torch.zeros(int(L.load().egpt_sample_ws_bytes(rows)), dtype=torch.uint8, device=device)


def sample(logits, cfg, u, *, out=None, ws=None, u_index=None):
    """Tokens int64 [rows, 1] drawn from bf16/fp32 logits [rows, V] (contiguous rows) with uniforms u.

    u: float32 [rows] (one draw per row), or [rows, n] with `u_index` (int64 device scalar): column *u_index is used
    and *u_index advances by one on the device (graph-capturable). `out` (int64, [rows, 1] or a [rows] view) and
    `ws` may be given to avoid allocations (CUDA-graph capture)."""
    _cuda(logits, u)
    if logits.dim() != 2 or logits.stride(-1) != 1:
        raise ValueError('logits must be [rows, V] with contiguous rows')
    if u.dtype != torch.float32:
        raise ValueError('uniforms must be float32')
    rows, v = logits.shape
    u2 = u.reshape(rows, -1)
    if u_index is None and u2.shape[1] != 1:
        raise ValueError('u must hold one draw per row (or pass u_index)')
    if out is None:
        out = torch.empty((rows, 1), dtype=torch.int64, device=logits.device)
    if ws is None:
        ws = sample_ws(rows, logits.device)
    top_k = 0 if cfg.top_k is None or cfg.top_k >= v else int(cfg.top_k)
    top_p = 1.0 if cfg.top_p is None else float(cfg.top_p)
    L.check(L.load().egpt_sample(_p(logits), _dt(logits), rows, v, logits.stride(0), float(cfg.temperature), top_k,
                                 top_p, _p(u2), u2.stride(0), _p(u_index), _p(out), out.stride(0), _p(ws),
                                 ws.numel(), _stream()), 'sample')
    return out


__all__ = ['SamplingConfig', 'draw_uniforms', 'sample', 'sample_ws']
