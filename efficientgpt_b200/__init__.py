"""efficientgpt_b200: batch-1 int8 decode engine for NVIDIA B200 (sm_100a).

Drop-in for the research/realmodel path of BagelsFun/efficientgpt: `int8_linear` (op, Int8Linear, quantize_model),
`fast_decode.GraphGreedyDecoder` (and `SampledGraphDecoder` with `sampling`: temperature, top-k, top-p, inverse
CDF on the device), `backend.BucketedGraphDecoder` (the request-sized decoder pool of HFBackend), plus
`ragged.RaggedGraphDecoder` (up to 16 sequences of different lengths), `tp.TPQwen3Engine` (tensor parallelism)
and `nanogpt` (config 1), with the
arithmetic in hand-written CUDA (libegpt_b200.so, C-ABI in
include/egpt_b200.h). Submodules import lazily so the package imports without a GPU.
"""
from . import _lib  # noqa: F401

__version__ = '0.1.0'


def __getattr__(name):
    if name in ('quantize_weight', 'Int8Linear', 'quantize_model', 'int8_linear', 'int8_matmul'):
        from . import int8_linear as m
        return getattr(m, name)
    if name in ('GraphGreedyDecoder', 'SampledGraphDecoder'):
        from . import fast_decode as m
        return getattr(m, name)
    if name in ('RaggedEngine', 'RaggedGraphDecoder'):  # ragged small-batch decode
        from . import ragged as m
        return getattr(m, name)
    if name in ('SamplingConfig', 'draw_uniforms', 'sample'):
        from . import sampling as m
        return getattr(m, name)
    if name in ('BucketedGraphDecoder', 'pick_bucket', 'GRAPH_BUCKETS', 'MAX_GRAPH_DECODERS'):  # serving decode layer
        from . import backend as m
        return getattr(m, name)
    if name == 'Qwen3Engine':
        from .engine import Qwen3Engine
        return Qwen3Engine
    if name == 'TPQwen3Engine':  # tensor parallelism over 2/4/8 GPUs of one box
        from .tp import TPQwen3Engine
        return TPQwen3Engine
    if name in ('GPT', 'GPTConfig', 'NanoGPTEngine'):  # nanoGPT
        from . import nanogpt as m
        return getattr(m, name)
    raise AttributeError(name)
