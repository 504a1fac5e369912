"""Weight-only int8 linear layers for Hugging Face decoder models, on B200 CUDA kernels.

Drop-in for BagelsFun/efficientgpt research/realmodel/int8_linear.py: same names, arguments, buffers
(`qweight` int8 [N, K], `scale` [N]), errors and custom op `efficientgpt::int8_linear`. What changed is below
the op: the arithmetic runs in libegpt_b200.so (hand-written sm_100a CUDA, see csrc/gemv_i8.cu) instead of
Triton (decode) and cuBLAS (prefill).

  quantize_weight   int8_linear.py:106-117  per-row s = max|w|/127 (>= 1e-12), q = round(w/s) in [-127, 127];
                    bit-identical, computed by egpt_quantize_rows on the GPU. scale_dtype=torch.bfloat16 stores
                    bf16(s) (BASELINE configs 2 and 5), q is computed from the fp32 s as in the reference.
  int8_matmul       int8_linear.py:67-85    <= 16 rows: bf16(s * (x @ q.T)), fp32 accumulation
  int8_linear (op)  int8_linear.py:88-103   bf16 only; > 16 rows reproduces the reference's prefill rounding,
                    bf16(bf16(x @ q.T) * s), on the tcgen05 GEMM (csrc/gemm_tc.cu; K a multiple of 64) or the
                    GEMV kernel over 16-row blocks (other K); no cuBLAS
  Int8Linear        int8_linear.py:120-134
  quantize_model    int8_linear.py:137-157  every nn.Linear incl. lm_head; a tied lm_head becomes an int8 copy

There is no CPU path: CPU tensors raise ValueError.
"""
import torch
from torch import nn

from . import _lib as L
from . import ops

MAX_DECODE_ROWS = 16


def int8_matmul(x2, w, s):
    """x2 bf16 [M <= 16, K] contiguous rows; w int8 [N, K]; s fp32/bf16 [N] -> bf16 [M, N]."""
    m, k = x2.shape
    if m > MAX_DECODE_ROWS:  # the kernel holds at most 16 rows of x
        raise ValueError(f'int8_matmul handles at most {MAX_DECODE_ROWS} rows, got {m}')
    return ops.gemv_i8(x2, w, s)


@torch.library.custom_op('efficientgpt::int8_linear', mutates_args=())
def int8_linear(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.dtype != torch.bfloat16:
        raise ValueError('int8_linear expects bf16 activations')
    if x2.shape[0] == 0:
        return x.new_empty(*x.shape[:-1], w.shape[0])
    if x2.shape[0] <= MAX_DECODE_ROWS:
        y = int8_matmul(x2.contiguous(), w, s)
    elif k % 64 == 0 and w.is_contiguous():  # the reference's prefill branch: bf16 GEMM output, then the scale
        y = ops.gemm_i8_tc(x2.contiguous(), w, s, double_round=True)
    else:
        y = ops.gemv_i8_rows(x2.contiguous(), w, s, double_round=True)
    return y.reshape(*x.shape[:-1], w.shape[0])


@int8_linear.register_fake
def _(x, w, s):
    return x.new_empty(*x.shape[:-1], w.shape[0])


def quantize_weight(weight, scale_dtype=torch.float32):
    """Per-output-channel symmetric int8: returns (q int8 [N, K], s [N]) with weight ~= q * s[:, None]."""
    if scale_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError('scale_dtype must be torch.float32 or torch.bfloat16')
    w = weight.detach()
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    return ops.quantize_rows(w, scale_dtype)


class Int8Linear(nn.Module):
    """A frozen linear layer stored as int8 rows: buffers `qweight` int8 [out, in] and `scale` [out] (fp32, or bf16
    with scale_dtype=torch.bfloat16), plus the source layer's bias (frozen) when it has one. The forward is the
    custom op, then the bias add in the activation dtype (the reference's rounding order)."""

    def __init__(self, linear, scale_dtype=torch.float32):
        super().__init__()
        weight, bias = linear.weight, linear.bias
        self.out_features, self.in_features = weight.shape
        qweight, scale = quantize_weight(weight, scale_dtype)
        self.register_buffer('qweight', qweight)
        self.register_buffer('scale', scale)
        self.bias = None if bias is None else nn.Parameter(bias.detach().clone(), requires_grad=False)

    def forward(self, x):
        y = int8_linear(x, self.qweight, self.scale)
        if self.bias is not None:
            y = y + self.bias
        return y

    def extra_repr(self):
        return f'{self.in_features} -> {self.out_features}, int8 rows, {str(self.scale.dtype)[6:]} scales'


def _convert_children(module, prefix, skip, scale_dtype):
    """Depth-first over the module tree: every nn.Linear child (but `skip`) is replaced by its Int8Linear in the
    parent's slot as soon as it is met, so its bf16 weight is released before the next one is quantised."""
    count = 0
    for name in list(module._modules):
        child = module._modules[name]
        path = f'{prefix}.{name}' if prefix else name
        if isinstance(child, nn.Linear):
            if path != skip:
                module._modules[name] = Int8Linear(child, scale_dtype)
                count += 1
        elif child is not None:
            count += _convert_children(child, path, skip, scale_dtype)
        del child
    return count


@torch.no_grad()
def quantize_model(model, include_lm_head=True, scale_dtype=torch.float32):
    """Replace every nn.Linear of `model` (the lm_head too unless include_lm_head=False) by Int8Linear, in place;
    returns how many. Embeddings and norms keep their dtype. A tied lm_head becomes its own int8 copy and the config
    is marked untied (the input embedding keeps its weight)."""
    count = _convert_children(model, '', None if include_lm_head else 'lm_head', scale_dtype)
    if include_lm_head and getattr(model, 'config', None) is not None:
        model.config.tie_word_embeddings = False
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return count


__all__ = ['MAX_DECODE_ROWS', 'int8_matmul', 'int8_linear', 'quantize_weight', 'Int8Linear', 'quantize_model', 'L']
