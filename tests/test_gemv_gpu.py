"""GPU parity of the int8 GEMV kernels (C-ABI egpt_gemv_i8 / egpt_lm_head_argmax / egpt_quantize_rows) against
the oracle and the reference's golden vectors. Mirrors research/realmodel/test_int8_linear.py and the
int8_gemv task of research/kernelagent/tasks.py."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
from oracle import int8_ref
from oracle.bf16 import from_bits, from_torch, round_bf16

pytestmark = pytest.mark.gpu

SWEEP = [(4096, 2048), (2048, 2048), (12288, 2048), (2048, 6144), (151936, 2048)]


def _lib():
    from efficientgpt_b200 import _lib as L, ops
    return L, ops


def _to_dev(x, q, s, cuda, s_dtype=torch.bfloat16):
    return (torch.from_numpy(x).to(cuda, torch.bfloat16), torch.from_numpy(q).to(cuda),
            torch.from_numpy(s).to(cuda, s_dtype))


def _bf16_ulps(a, b):
    """|a - b| in units of the bf16 spacing at max(|a|, |b|)."""
    m = np.maximum(np.abs(a), np.abs(b))
    ulp = np.where(m > 0, 2.0 ** (np.floor(np.log2(np.maximum(m, 1e-38))) - 7), 1.0)
    return np.abs(a - b) / ulp


def _sum_err_bound(x, q, s):
    """Bound on the difference two fp32 summation orders can make before the bf16 rounding:
    4 sqrt(K) 2^-24 sum_k |x_k q_k| s (probabilistic, generous), per output element."""
    x = np.asarray(x, np.float64).reshape(-1, np.shape(x)[-1])
    k = x.shape[1]
    return 4 * np.sqrt(k) * 2.0 ** -24 * (np.abs(x) @ np.abs(q.astype(np.float64)).T) * np.asarray(s, np.float64)


def _check_vs_oracle(y, ref, what, x=None, q=None, s=None):
    """The kernel and the oracle sum the same exact products in different fp32 orders: outputs agree to one
    bf16 ulp, plus the fp32 summation error where cancellation makes it larger than an ulp, and differ only
    on a small fraction of elements."""
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    m = np.maximum(np.abs(y), np.abs(ref))
    ulp = np.where(m > 0, 2.0 ** (np.floor(np.log2(np.maximum(m, 1e-38))) - 7), 0.0)
    tol = ulp + (_sum_err_bound(x, q, s).reshape(y.shape) if x is not None else 0.0)
    d = np.abs(y - ref)
    assert np.all(d <= tol), (what, float((d / np.maximum(tol, 1e-30)).max()))
    assert (d > 0).mean() < 0.01, (what, float((d > 0).mean()))


@pytest.mark.parametrize('n,k', SWEEP)
@pytest.mark.parametrize('seed,edge', [(0, None), (1, None), (0, 'large'), (0, 'extreme_w')])
def test_gemv_sweep_vs_oracle_and_fp64(cuda, n, k, seed, edge):
    L, ops = _lib()
    x, q, s = int8_ref.gemv_inputs(n, k, seed, edge=edge)
    xd, qd, sd = _to_dev(x, q, s, cuda)
    y = from_torch(ops.gemv_i8(xd, qd, sd))
    ref = int8_ref.int8_matmul(x, q, s)
    _check_vs_oracle(y, ref, (n, k, seed, edge), x, q, s)
    truth = int8_ref.int8_truth(x, q, s)
    naive = from_torch((xd @ (qd.to(torch.bfloat16) * sd[:, None]).t()))  # bf16 dequant + cuBLAS
    err = np.abs(y - truth).max()
    assert err <= max(2 * np.abs(naive - truth).max(), 1e-3), (n, k, err)


@pytest.mark.parametrize('n,k', SWEEP + [(2048, 12288), (48, 32)])
@pytest.mark.parametrize('seed,edge', [(0, None), (1, None), (0, 'large'), (0, 'extreme_w')])
def test_exact_gemv_sweep_is_the_exact_sum_rounded_once(cuda, n, k, seed, edge):
    """EGPT_FLAG_EXACT: the tensor-core kernel's output is bf16(fp32(exact x . q) * s) (oracle int8_exact) bit for
    bit, except where an x value falls below the fixed-point grid (2^-29 of the largest |x|): allowed on 0.1%
    of the outputs, one bf16 ulp at most. Covers the split-chunk mode (few tiles per CTA), the whole-tile mode
    (lm_head) and the two-pass staging of inputs wider than 6144."""
    L, ops = _lib()
    x, q, s = int8_ref.gemv_inputs(n, k, seed, edge=edge)
    xd, qd, sd = _to_dev(x, q, s, cuda)
    y = from_torch(ops.gemv_i8(xd, qd, sd, exact=True))
    ref = int8_ref.int8_exact(x, q, s)
    same = np.mean(y == ref)
    assert same >= 0.999, (n, k, same)
    assert _bf16_ulps(y, ref).max() <= 1.0


def test_exact_gemv_epilogues(cuda):
    """Residual (in place), SiLU*up over cat(gate, up) and the fused RMSNorm prologue of the exact kernel against the
    same rounding points on the oracle's exact sums."""
    L, ops = _lib()
    k, n = 2048, 1024
    x, q, s = int8_ref.gemv_inputs(n, k, 3)
    xd, qd, sd = _to_dev(x, q, s, cuda)
    base = int8_ref.int8_exact(x, q, s)
    rng = np.random.default_rng(5)
    r0 = round_bf16(rng.standard_normal((1, n)).astype(np.float32))
    r = torch.from_numpy(r0).to(cuda, torch.bfloat16)
    ops.gemv_i8(xd, qd, sd, epilogue=L.EPI_RESIDUAL, residual=r, exact=True)
    assert np.mean(from_torch(r) == round_bf16(r0 + base)) >= 0.999
    y = from_torch(ops.gemv_i8(xd, qd, sd, epilogue=L.EPI_SILU_MUL, exact=True))
    g, u = base[:, :n // 2], base[:, n // 2:]
    want = round_bf16(round_bf16(g / (np.float32(1) + np.exp(-g))) * u)
    assert y.shape == (1, n // 2) and _bf16_ulps(y, want).max() <= 1.0 and np.mean(y == want) >= 0.99
    w = torch.from_numpy(round_bf16(rng.standard_normal(k).astype(np.float32))).to(cuda, torch.bfloat16)
    fused = from_torch(ops.gemv_i8(xd, qd, sd, norm_w=w, eps=1e-6, exact=True))
    sep = from_torch(ops.gemv_i8(ops.rmsnorm(xd, w, 1e-6), qd, sd, exact=True))
    assert np.mean(fused == sep) >= 0.99 and _bf16_ulps(fused, sep).max() <= 2.0
    with pytest.raises(ValueError):
        ops.gemv_i8(xd.repeat(2, 1), qd, sd, exact=True)  # one row only
    with pytest.raises(ValueError):
        ops.gemv_i8(xd.float(), qd, sd, exact=True)  # bf16 only


@pytest.mark.parametrize('m,k,n', [(1, 2048, 6144), (4, 6144, 2048), (16, 2048, 1024), (3, 100, 70), (17, 2048, 512),
                                   (64, 512, 256), (2, 2048, 1024), (1, 6144, 2048)])
def test_op_matches_oracle_and_fp64(cuda, m, k, n):
    """research/realmodel/test_int8_linear.py:14-35 shapes and bound (err <= max(2 naive_err, 1e-3))."""
    from efficientgpt_b200.int8_linear import int8_linear
    g = torch.Generator(device='cuda').manual_seed(0)
    q = torch.randint(-127, 128, (n, k), device=cuda, dtype=torch.int8, generator=g)
    s = torch.rand(n, device=cuda, generator=g) * 0.01 + 1e-4
    x = torch.randn(m, k, device=cuda, generator=g).to(torch.bfloat16)
    y = int8_linear(x, q, s)
    assert (y.shape, y.dtype) == ((m, n), torch.bfloat16)
    ref = x.double() @ (q.double() * s.double()[:, None]).t()
    naive = (x @ (q.to(torch.bfloat16) * s.to(torch.bfloat16)[:, None]).t()).double()
    err, naive_err = float((y.double() - ref).abs().max()), float((naive - ref).abs().max())
    assert err <= max(2 * naive_err, 1e-3), (m, k, n)
    orc = int8_ref.int8_linear(from_torch(x), from_torch(q).astype(np.int8), from_torch(s))
    _check_vs_oracle(from_torch(y), orc, (m, k, n), from_torch(x), from_torch(q).astype(np.int8), from_torch(s))


def test_prefill_branch_matches_reference_golden(cuda):
    from conftest import ROOT
    from efficientgpt_b200.int8_linear import int8_linear
    z = np.load(ROOT / 'tests' / 'golden' / 'prefill_linear.npz')
    for i, shp in enumerate(gi.PREFILL_SHAPES):
        x, q, s = gi.prefill_case(i)
        y = from_torch(int8_linear(x.to(cuda), q.to(cuda), s.to(cuda)))
        _check_vs_oracle(y, from_bits(z[f"y{i}"]), shp, from_torch(x), q.numpy(), s.numpy())


def test_more_than_16_rows_refused_by_kernel(cuda):
    from efficientgpt_b200.int8_linear import int8_matmul
    q = torch.zeros(64, 32, device=cuda, dtype=torch.int8)
    with pytest.raises(ValueError):
        int8_matmul(torch.zeros(17, 32, device=cuda, dtype=torch.bfloat16), q, torch.ones(64, device=cuda))


def test_quantizer_bit_identical_to_reference_golden(cuda, golden):
    from conftest import ROOT
    from efficientgpt_b200.int8_linear import quantize_weight
    z = np.load(ROOT / 'tests' / 'golden' / 'quantize.npz')
    w = gi.quantize_input()
    assert gi.sha(w) == golden['quantize']['w_sha256']
    q, s = quantize_weight(w.to(cuda))
    # the golden ran the reference on CPU (true division by 127); the product reproduces the reference on
    # the GPU (PyTorch multiplies by fl32(1/127)): identical wherever the two scalar divisions agree ...
    qo, so = int8_ref.quantize_weight(from_torch(w), 'cuda')
    np.testing.assert_array_equal(q.cpu().numpy(), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    same = so == z['s']
    assert same.mean() > 0.5
    np.testing.assert_array_equal(q.cpu().numpy()[same], z['q'][same])
    # ... and bit-identical to the reference's own formula evaluated by PyTorch on the GPU
    wc = w.to(cuda).float()
    s_t = (wc.abs().amax(1) / 127.0).clamp_min(1e-12)
    assert torch.equal(s, s_t)
    assert torch.equal(q, torch.round(wc / s_t[:, None]).clamp(-127, 127).to(torch.int8))
    edge = gi.quantize_edge_rows()
    qe, se = quantize_weight(edge.to(cuda))
    qeo, seo = int8_ref.quantize_weight(edge.numpy(), 'cuda')
    np.testing.assert_array_equal(qe.cpu().numpy(), qeo)
    np.testing.assert_array_equal(se.cpu().numpy(), seo)
    big = torch.randn(20000, 64, device=cuda)  # reference test: > one 8192-row chunk, whole-matrix formula
    qb, sb = quantize_weight(big)
    s_ref = (big.abs().amax(1) / 127.0).clamp_min(1e-12)
    assert torch.equal(sb, s_ref)
    assert torch.equal(qb, torch.round(big / s_ref[:, None]).clamp(-127, 127).to(torch.int8))
    _, sbf = quantize_weight(big, torch.bfloat16)
    assert torch.equal(sbf, s_ref.to(torch.bfloat16))


def test_quantize_model_surgery(cuda):
    """research/realmodel/test_int8_linear.py:43-60 (model part)."""
    from efficientgpt_b200.int8_linear import Int8Linear, quantize_model
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(128, 64, bias=True), torch.nn.GELU(), torch.nn.Linear(64, 32)).cuda()
    net = net.to(torch.bfloat16)
    x = torch.randn(5, 128, device=cuda, dtype=torch.bfloat16)
    ref = net(x).float()
    assert quantize_model(net, include_lm_head=False) == 2
    assert isinstance(net[0], Int8Linear)
    assert float((net(x).float() - ref).abs().max()) < 0.05 * float(ref.abs().max()) + 1e-2


def test_compile_and_cuda_graph_bit_identical(cuda):
    """research/realmodel/test_int8_linear.py:62-79."""
    from efficientgpt_b200.int8_linear import int8_linear
    q = torch.randint(-127, 128, (512, 256), device=cuda, dtype=torch.int8)
    s = torch.rand(512, device=cuda) * 0.01
    x = torch.randn(2, 256, device=cuda, dtype=torch.bfloat16)
    eager = int8_linear(x, q, s)
    assert torch.equal(torch.compile(lambda t: int8_linear(t, q, s), fullgraph=True)(x), eager)
    static_x = x.clone()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        int8_linear(static_x, q, s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = int8_linear(static_x, q, s)
    static_x.copy_(x * 2)
    g.replay()
    assert torch.equal(out, int8_linear(x * 2, q, s))


def test_epilogues_vs_torch(cuda):
    L, ops = _lib()
    g = torch.Generator(device='cuda').manual_seed(7)
    k, n = 2048, 1024
    q = torch.randint(-127, 128, (n, k), device=cuda, dtype=torch.int8, generator=g)
    s = (torch.rand(n, device=cuda, generator=g) * 0.02 + 1e-3).to(torch.bfloat16)
    x = torch.randn(1, k, device=cuda, generator=g).to(torch.bfloat16)
    base = ((x.float() @ q.float().t()) * s.float()).to(torch.bfloat16)
    # residual (in place)
    r = torch.randn(1, n, device=cuda, generator=g).to(torch.bfloat16)
    r0 = r.clone()
    ops.gemv_i8(x, q, s, epilogue=L.EPI_RESIDUAL, residual=r)
    assert (r.float() - (r0 + base).float()).abs().max() <= 2 * 2 ** -7 * (r0 + base).float().abs().max()
    # SiLU * up over cat(gate, up)
    y = ops.gemv_i8(x, q, s, epilogue=L.EPI_SILU_MUL)
    gate, up = base[:, :n // 2], base[:, n // 2:]
    ref = (torch.nn.functional.silu(gate) * up)
    assert y.shape == (1, n // 2)
    torch.testing.assert_close(y.float(), ref.float(), atol=2e-2, rtol=2e-2)
    # fused RMSNorm prologue == rmsnorm then gemv (same bits)
    w = torch.randn(k, device=cuda, generator=g).to(torch.bfloat16)
    fused = ops.gemv_i8(x, q, s, norm_w=w, eps=1e-6)
    sep = ops.gemv_i8(ops.rmsnorm(x, w, 1e-6), q, s)
    assert torch.equal(fused, sep)
    # fp32 path with bias and GELU (nanoGPT)
    xf = torch.randn(3, k, device=cuda, generator=g)
    bias = torch.randn(n, device=cuda, generator=g)
    sf = s.float()
    yf = ops.gemv_i8(xf, q, sf, bias=bias, epilogue=L.EPI_GELU)
    reff = torch.nn.functional.gelu(xf @ (q.float() * sf[:, None]).t() + bias)
    torch.testing.assert_close(yf, reff, atol=1e-4, rtol=1e-4)
    # plain-load fallback agrees with the bulk-copy kernel
    assert torch.equal(ops.gemv_i8(x, q, s, no_tma=True), ops.gemv_i8(x, q, s))


@pytest.mark.parametrize('n,k', [(151936, 2048), (50304, 384), (512, 128)])
def test_exact_lm_head_argmax(cuda, n, k):
    """EGPT_FLAG_EXACT on the lm_head: logits bf16(fp32(exact sum) * s) (oracle int8_exact), token = first index
    of the maximum, position advanced; whole-tile mode (151936, 50304) and split mode (512), two calls in a row
    (the workspace counter is left at zero)."""
    L, ops = _lib()
    x, q, s = int8_ref.gemv_inputs(n, k, 2)
    xd, qd, sd = _to_dev(x, q, s, cuda)
    ws = ops.lm_head_ws(n, cuda)
    want = int8_ref.int8_exact(x, q, s)[0]
    pos = torch.zeros(1, dtype=torch.int64, device=cuda)
    for it in range(2):
        logits = torch.empty(n, dtype=torch.bfloat16, device=cuda)
        tok = ops.lm_head_argmax(xd[0], qd, sd, ws, logits=logits, position=pos, advance=True, exact=True)
        got = from_torch(logits)
        assert np.mean(got == want) >= 0.999 and _bf16_ulps(got, want).max() <= 1.0
        assert int(tok) == int(np.argmax(got))  # first index of the maximum of its own logits
        assert int(pos) == it + 1


@pytest.mark.parametrize('n,k', [(151936, 2048), (50304, 384), (512, 128)])
def test_lm_head_argmax_vs_oracle(cuda, n, k):
    L, ops = _lib()
    x, q, s = int8_ref.gemv_inputs(n, k, seed=3)
    xd, qd, sd = _to_dev(x, q, s, cuda)
    ws = ops.lm_head_ws(n, cuda)
    logits = torch.empty(n, device=cuda, dtype=torch.bfloat16)
    for _ in range(2):  # the workspace counter must be left at zero
        tok = ops.lm_head_argmax(xd[0], qd, sd, ws, logits=logits)
        y = from_torch(logits)
        assert int(tok) == int(np.argmax(y))
    _check_vs_oracle(y, int8_ref.int8_matmul(x, q, s)[0], (n, k), x, q, s)
    # ties: two equal maxima -> the lower index wins
    qd2 = qd.clone()
    qd2[n // 3] = 127
    qd2[n // 2] = 127
    sd2 = sd.clone()
    sd2[n // 3] = sd2[n // 2] = 1.0
    xd2 = xd.abs()
    tok = ops.lm_head_argmax(xd2[0], qd2, sd2, ws, logits=logits)
    assert int(tok) == n // 3
