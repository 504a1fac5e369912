"""tcgen05 int8-weight GEMM (egpt_gemm_i8_tc, csrc/gemm_tc.cu) against the reference's >16-row arithmetic
bf16(bf16(x @ bf16(q).T) * s) (research/realmodel/int8_linear.py:96-97), with the sum in fp64 as the truth: every
output within 2 bf16 ulps of bf16(bf16(truth) * s) (the two roundings of an fp32-accumulated sum can each move one
ulp) plus the fp32 summation bound K 2^-24 sum|x q| scaled by s (cancellation can leave a result far below its
terms), at least 99% identical, and no worse than PyTorch's own fp32-accumulated bf16 matmul of the same operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ulp(v):
    a = v.abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


def _case(m, n, k, scale_dtype, seed, double_round=True, x_scale=1.0):
    from efficientgpt_b200 import ops
    g = torch.Generator(device='cuda').manual_seed(seed)
    x = (torch.randn(m, k, generator=g, device='cuda') * x_scale).to(torch.bfloat16)
    q = torch.randint(-127, 128, (n, k), generator=g, device='cuda', dtype=torch.int8)
    s = (torch.rand(n, generator=g, device='cuda') * 0.02 + 0.001).to(scale_dtype)
    y = ops.gemm_i8_tc(x, q, s, double_round=double_round)
    t = x.double() @ q.double().t()
    acc = t.float().to(torch.bfloat16).float() if double_round else t.float()
    want = (acc * s.float()).to(torch.bfloat16)
    mine = torch.matmul(x, q.to(torch.bfloat16).t())  # PyTorch's bf16 GEMM (fp32 accumulation)
    torch_y = ((mine.float() if double_round else (x.float() @ q.float().t())) * s.float()).to(torch.bfloat16)
    absum = x.abs().double() @ q.abs().double().t()
    bound = (k * 2.0 ** -24 * absum * s.double()).float()
    return y.float(), want.float(), torch_y.float(), bound


@pytest.mark.parametrize('m,n,k', [(1, 256, 64), (128, 256, 2048), (300, 4096, 2048), (77, 96, 128),
                                   (1000, 2048, 6144), (4096, 768, 4096), (129, 12288, 2048)])
@pytest.mark.parametrize('scale_dtype', [torch.bfloat16, torch.float32])
def test_gemm_i8_tc_matches_reference_rounding(cuda, m, n, k, scale_dtype):
    y, want, torch_y, bound = _case(m, n, k, scale_dtype, seed=m + n + k)
    assert y.shape == (m, n)
    err = (y - want).abs()
    tol = 2 * _ulp(want) + bound
    assert bool((err <= tol).all()), float((err - tol).max())
    same = float((y == want).float().mean())
    same_torch = float((torch_y == want).float().mean())
    assert same >= 0.99 and same >= same_torch - 0.01, (same, same_torch)


def test_gemm_i8_tc_single_rounding_and_large_inputs(cuda):
    y, want, _, bound = _case(512, 1024, 4096, torch.float32, seed=9, double_round=False, x_scale=30.0)
    assert bool(((y - want).abs() <= 2 * _ulp(want) + bound).all())
    assert float((y == want).float().mean()) >= 0.99


def test_gemm_i8_tc_guards(cuda):
    from efficientgpt_b200 import ops
    x = torch.zeros(4, 100, dtype=torch.bfloat16, device='cuda')
    q = torch.zeros(256, 100, dtype=torch.int8, device='cuda')
    s = torch.ones(256, dtype=torch.bfloat16, device='cuda')
    with pytest.raises(ValueError):  # K not a multiple of 64
        ops.gemm_i8_tc(x, q, s)
    with pytest.raises(ValueError):
        ops.gemm_i8_tc(x.float(), q, s)


@pytest.mark.parametrize('m,n,k', [(300, 2048, 2048), (5, 4096, 6144), (4096, 768, 4096)])
def test_gemm_i8_tc_residual_add_in_epilogue(cuda, m, n, k):
    """EGPT_FLAG_ADD_OUT: out = bf16(residual + bf16(result)), the HF residual add of o_proj/down_proj over the
    prompt rows, equal bit for bit to the GEMM followed by PyTorch's bf16 add (split-K rows included)."""
    from efficientgpt_b200 import ops
    g = torch.Generator(device='cuda').manual_seed(m + n)
    x = torch.randn(m, k, generator=g, device='cuda').to(torch.bfloat16)
    q = torch.randint(-127, 128, (n, k), generator=g, device='cuda', dtype=torch.int8)
    s = (torch.rand(n, generator=g, device='cuda') * 0.02 + 0.001).to(torch.bfloat16)
    h = torch.randn(m, n, generator=g, device='cuda').to(torch.bfloat16)
    want = h + ops.gemm_i8_tc(x, q, s)
    got = h.clone()
    out = ops.gemm_i8_tc(x, q, s, out=got, add_out=True)
    assert out.data_ptr() == got.data_ptr()
    assert torch.equal(got, want)


@pytest.mark.parametrize('m,inter', [(1, 6144), (300, 6144), (33, 12288), (7, 2)])
def test_silu_mul_matches_eager_bf16(cuda, m, inter):
    """egpt_silu_mul: bf16(bf16(silu(gate)) * up) as the HF MLP evaluates it in eager bf16 (modeling_qwen3.py:81-82);
    within one bf16 ulp of PyTorch's F.silu(gate) * up (CUDA's expf and PyTorch's may differ in the last fp32 bit,
    which can move a bf16 rounding), and identical for at least 99.9% of the values."""
    import torch.nn.functional as F
    from efficientgpt_b200 import ops
    g = torch.Generator(device='cuda').manual_seed(m + inter)
    gu = (torch.randn(m, 2 * inter, generator=g, device='cuda') * 3).to(torch.bfloat16)
    got = ops.silu_mul(gu, inter)
    want = F.silu(gu[:, :inter]) * gu[:, inter:]
    assert got.shape == want.shape
    diff = (got.float() - want.float()).abs()
    assert bool((diff <= _ulp(want.float())).all())
    assert float((got == want).float().mean()) >= 0.999
