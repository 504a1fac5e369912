"""Restatement of the reference's int8 weight-only linear in numpy (test infrastructure; see oracle/__init__.py).

Reference: BagelsFun/efficientgpt research/realmodel/int8_linear.py.
"""
import numpy as np

from .bf16 import round_bf16

MAX_DECODE_ROWS = 16  # int8_linear.py:18


def quantize_weight(w, semantics='cuda'):
    """int8_linear.py:106-117 quantize_weight: per-row s = max(max|w| / 127, 1e-12) in fp32,
    q = clamp(round_half_even(w / s), -127, 127) as int8. (The 8192-row chunking there is elementwise per row.)

    `max|w| / 127.0` divides a tensor by a Python scalar. On CUDA tensors (where the reference quantises: the
    model is moved to the GPU first, assistant/backends.py:198-202) PyTorch evaluates that as a multiplication
    by fl32(1/127); on CPU tensors as a true division. semantics='cuda' | 'cpu' selects which; `w / s` is a true
    division in both."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    amax = np.abs(w).max(axis=1)
    if semantics == 'cuda':
        s0 = amax * (np.float32(1.0) / np.float32(127.0))
    elif semantics == 'cpu':
        s0 = amax / np.float32(127.0)
    else:
        raise ValueError(semantics)
    s = np.maximum(s0.astype(np.float32), np.float32(1e-12)).astype(np.float32)
    with np.errstate(invalid='ignore'):
        q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s


def int8_matmul(x, q, s):
    """int8_linear.py:26-38,67-78 (_dot16 via int8_matmul, <= 16 rows): bf16(s * (x @ q.T)), fp32 accumulation.
    x float32 array holding bf16 values [M, K]; q int8 [N, K]; s float32 [N] (bf16 scales passed as their values)."""
    x = np.asarray(x, dtype=np.float32)
    if x.shape[0] > MAX_DECODE_ROWS:
        raise ValueError(f'int8_matmul handles at most {MAX_DECODE_ROWS} rows, got {x.shape[0]}')
    acc = x @ q.astype(np.float32).T
    return round_bf16(acc * np.asarray(s, dtype=np.float32)[None, :])


def int8_linear_prefill(x, q, s):
    """int8_linear.py:96-97 (> 16 rows): bf16(bf16(x @ bf16(q).T) * s)."""
    acc = np.asarray(x, dtype=np.float32) @ q.astype(np.float32).T
    return round_bf16(round_bf16(acc) * np.asarray(s, dtype=np.float32)[None, :])


def int8_linear(x, q, s):
    """int8_linear.py:88-98: the op, dispatching on the row count."""
    x2 = np.asarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
    y = int8_matmul(x2, q, s) if x2.shape[0] <= MAX_DECODE_ROWS else int8_linear_prefill(x2, q, s)
    return y.reshape(*x.shape[:-1], q.shape[0])


def int8_exact(x, q, s):
    """The exact-sum GEMV of the persistent decode step and EGPT_FLAG_EXACT: bf16(fp32(x . q) * s) with the dot
    product exact (fp64 holds these bf16 x int8 sums exactly) and rounded once to fp32 (the rounding points of
    int8_linear.py:37, `bf16(acc * s)`, with an exact acc)."""
    acc = (np.asarray(x, np.float64) @ q.astype(np.float64).T).astype(np.float32)
    return round_bf16(acc * np.asarray(s, np.float32)[None, :])


def fixed_point_stage(x):
    """The exact GEMV's input staging in numpy (the arithmetic of the product's stage_input, not a reference
    function): bound = max |x|, E = floor(log2 bound) - 29, X = rint(x 2^-E) with |X| < 2^30, and X's balanced
    base-256 digits d0..d3 in [-128, 127] (X = sum d_i 256^i). Returns (E, X int64, digits int64 [4, ...])."""
    x = np.asarray(x, np.float32)
    bound = float(np.max(np.abs(x))) if x.size else 0.0
    ex = int(np.floor(np.log2(bound))) if bound > 0 else 0
    e = ex - 29
    big = np.rint(x.astype(np.float64) * 2.0 ** -e).astype(np.int64)
    digits, rest = [], big.copy()
    for _ in range(3):
        d = ((rest + 128) & 0xFF) - 128  # balanced digit: the low byte read as int8
        digits.append(d)
        rest = (rest - d) >> 8
    digits.append(rest)
    return e, big, np.stack(digits)


def int8_fixed_point(x, q, s):
    """bf16(fp32(sum_k X_k q_nk 2^E) * s): the exact GEMV on the staged fixed-point input (int64 sums)."""
    e, big, _ = fixed_point_stage(np.asarray(x, np.float32)[0])
    acc = (big[None, :] @ q.astype(np.int64).T).astype(np.float64) * 2.0 ** e
    return round_bf16(acc.astype(np.float32) * np.asarray(s, np.float32)[None, :])


def int8_truth(x, q, s):
    """fp64 ground truth of x @ (q * s).T (research/kernelagent/tasks.py:150-158, chunking irrelevant in numpy)."""
    return np.asarray(x, np.float64) @ (q.astype(np.float64) * np.asarray(s, np.float64)[:, None]).T


def gemv_inputs(n, k, seed, m=1, edge=None):
    """Seeded GEMV sweep inputs (BASELINE config 3 and research/kernelagent/tasks.py:132-147):
    x ~ N(0,1) bf16 [m, k] (x30 for edge='large'), q uniform in [-127, 127] (+-127 for edge='extreme_w'),
    s ~ U(0.001, 0.02) rounded to bf16. Returns (x float32 holding bf16 values, q int8, s float32 holding bf16)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    if edge == 'large':
        x = x * np.float32(30.0)
    x = round_bf16(x)
    q = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    if edge == 'extreme_w':
        q = np.where(q >= 0, 127, -127).astype(np.int8)
    s = round_bf16(rng.uniform(0.001, 0.02, size=n).astype(np.float32))
    return x, q, s
