"""egpt_attn_decode_noalloc: the decode attention entry point for callers that must not allocate device memory
(an operator inside another framework whose device memory belongs to that framework's allocator, or a serving
path that plans all memory up front). Its scratch is a built-in device array; these tests call it through the
C-ABI and compare it with egpt_attn_decode given a caller workspace. The file is named so that pytest collects
it last; it passes alone in a fresh process and after the other tests."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

NQ, NKV, D = 16, 8, 128


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _call(lib, fn, out, q, k, v, pos, m, max_split, flags, ws=None):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = (_p(out), out.stride(0), _p(q), q.stride(0), _p(k), _p(v), k.shape[1], _p(pos), m, NQ, NKV, D, None, None,
              1e-6, None, None, D ** -0.5, max_split)
    if fn == 'noalloc':
        return lib.egpt_attn_decode_noalloc(*common, 1, flags, stream)
    return lib.egpt_attn_decode(*common, _p(ws), ws.numel(), 1, flags, stream)


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row(cuda):
    from efficientgpt_b200 import _lib as L
    lib = L.load()
    g = torch.Generator(device='cuda').manual_seed(5)
    cap = 4096
    k = torch.randn(NKV, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    v = torch.randn(NKV, cap, D, device=cuda, generator=g).to(torch.bfloat16)
    # two calls in a row with different contexts and split counts: the shared counters must be reusable
    for length, max_split, flags in ((3000, 18, L.FLAG_REF_SOFTMAX), (777, 7, 0)):
        q = torch.randn(1, NQ * D, device=cuda, generator=g).to(torch.bfloat16)
        pos = torch.tensor([length - 1], device=cuda)
        ws = torch.zeros(int(lib.egpt_attn_ws_bytes(1, NQ, NKV, D, max_split)), dtype=torch.uint8, device=cuda)
        want = torch.empty(1, NQ * D, dtype=torch.bfloat16, device=cuda)
        got = torch.full((1, NQ * D), float('nan'), dtype=torch.bfloat16, device=cuda)
        assert _call(lib, fn='ws', out=want, q=q, k=k, v=v, pos=pos, m=1, max_split=max_split, flags=flags, ws=ws) == 0
        assert _call(lib, fn='noalloc', out=got, q=q, k=k, v=v, pos=pos, m=1, max_split=max_split, flags=flags) == 0, \
            L.last_error()
        torch.cuda.synchronize()
        # the same kernel on the same inputs: identical bits (the attention tests' tolerance is looser than this)
        assert torch.equal(got, want), (length, max_split)
    assert L.device_error() == 0


def test_noalloc_rejects_scratch_beyond_its_size(cuda):
    from efficientgpt_b200 import _lib as L
    lib = L.load()
    m, max_split = 64, 64
    assert lib.egpt_attn_ws_bytes(m, NQ, NKV, D, max_split) > 524288
    k = torch.zeros(NKV, 256, D, dtype=torch.bfloat16, device=cuda)
    q = torch.zeros(m, NQ * D, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros(m, NQ * D, dtype=torch.bfloat16, device=cuda)
    pos = torch.zeros(1, dtype=torch.int64, device=cuda)
    rc = _call(lib, fn='noalloc', out=out, q=q, k=k, v=k, pos=pos, m=m, max_split=max_split, flags=0)
    assert rc == L.EGPT_ERR_WORKSPACE
    assert 'built-in' in L.last_error()
