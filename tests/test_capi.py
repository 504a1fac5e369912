"""CPU tests of the C-ABI boundary: the library loads, exports every function the header declares, and
rejects bad arguments with the documented status before touching a GPU. No kernel is launched here."""
import ctypes

import pytest
import torch

from efficientgpt_b200 import _lib as L


def test_library_exports_every_header_function():
    lib = L.load()
    names = L.header_functions()
    assert len(names) >= 16
    for n in names:
        assert hasattr(lib, n), n
        assert n in L.SIGNATURES, f'{n} has no ctypes signature'
    assert set(L.SIGNATURES) == set(names)


def test_version_and_error_strings():
    lib = L.load()
    assert b'sm_100a' in lib.egpt_version()
    assert lib.egpt_last_error() is not None


def test_workspace_size_queries():
    lib = L.load()
    assert lib.egpt_lm_head_ws_bytes(151936) >= 1024 * 8
    a = lib.egpt_attn_ws_bytes(1, 16, 8, 128, 19)
    assert a >= 16 * 19 * 130 * 4 + 8 * 4
    assert lib.egpt_attn_ws_bytes(4, 16, 8, 128, 19) > a


def test_argument_validation_without_launch():
    lib = L.load()
    null = None
    rc = lib.egpt_gemv_i8(null, null, L.EGPT_BF16, 1, 16, 16, null, null, L.EGPT_F32, 16, 16, null, null, 0, null,
                          0.0, null, 0, null)
    assert rc == L.EGPT_ERR_ARG
    assert 'null' in L.last_error()
    dummy = ctypes.c_void_p(16)
    rc = lib.egpt_gemv_i8(dummy, dummy, L.EGPT_BF16, 17, 16, 16, dummy, dummy, L.EGPT_F32, 16, 16, null, null, 0, null,
                          0.0, null, 0, null)
    assert rc == L.EGPT_ERR_SHAPE
    rc = lib.egpt_gemv_i8(dummy, dummy, 7, 1, 16, 16, dummy, dummy, L.EGPT_F32, 16, 16, null, null, 0, null, 0.0, null,
                          0, null)
    assert rc == L.EGPT_ERR_DTYPE
    rc = lib.egpt_attn_decode(dummy, 64, dummy, 64, dummy, dummy, 8, dummy, 1, 6, 4, 32, null, null, 0.0, null, null,
                              1.0, 4, null, 0, L.EGPT_BF16, 0, null)
    assert rc == L.EGPT_ERR_SHAPE  # 6 q heads over 4 kv heads
    rc = lib.egpt_lm_head_argmax(dummy, null, null, dummy, dummy, dummy, L.EGPT_F32, 100, 64, null, 0.0, dummy, 8, 0,
                                 null)
    assert rc == L.EGPT_ERR_WORKSPACE
    with pytest.raises(ValueError, match='workspace'):
        L.check(rc, 'lm_head_argmax')
    # prefill attention and SwiGLU: shape checks before any tensor map or launch
    rc = lib.egpt_attn_prefill(dummy, 2048, dummy, 2048, dummy, dummy, 64, 0, 16, 16, 8, 64, 0.1, null)
    assert rc == L.EGPT_ERR_SHAPE and 'head_dim' in L.last_error()
    rc = lib.egpt_attn_prefill(dummy, 2048, dummy, 2048, dummy, dummy, 64, 60, 16, 16, 8, 128, 0.1, null)
    assert rc == L.EGPT_ERR_SHAPE  # pos0 + m > cap
    rc = lib.egpt_attn_prefill(null, 2048, dummy, 2048, dummy, dummy, 64, 0, 16, 16, 8, 128, 0.1, null)
    assert rc == L.EGPT_ERR_ARG
    rc = lib.egpt_silu_mul(dummy, 8, dummy, 16, 4, 7, null)
    assert rc == L.EGPT_ERR_SHAPE  # odd width


def test_ops_reject_cpu_tensors():
    from efficientgpt_b200 import ops
    from efficientgpt_b200.int8_linear import int8_linear, quantize_weight
    with pytest.raises(ValueError, match='CUDA'):
        ops.gemv_i8(torch.zeros(1, 32, dtype=torch.bfloat16), torch.zeros(8, 32, dtype=torch.int8), torch.ones(8))
    with pytest.raises(ValueError, match='CUDA'):
        quantize_weight(torch.randn(4, 4))
    with pytest.raises(ValueError, match='bf16'):
        int8_linear(torch.zeros(2, 32), torch.zeros(8, 32, dtype=torch.int8), torch.ones(8))
    with pytest.raises(ValueError, match='CUDA'):
        ops.silu_mul(torch.zeros(2, 16, dtype=torch.bfloat16), 8)
    with pytest.raises(ValueError, match='CUDA'):
        ops.attn_prefill(torch.zeros(4, 256, dtype=torch.bfloat16), torch.zeros(1, 8, 128, dtype=torch.bfloat16),
                         torch.zeros(1, 8, 128, dtype=torch.bfloat16), 0, 2, 1, 128, scale=0.1)


def test_plan_struct_layout_matches_the_header(tmp_path):
    """The ctypes mirror of egpt_qwen3_plan / egpt_qwen3_layer has the C compiler's size and field offsets."""
    import shutil
    import subprocess
    cc = shutil.which('gcc') or shutil.which('cc')
    if cc is None:
        pytest.skip('no C compiler')
    plan_fields = [f[0] for f in L.Qwen3Plan._fields_]
    layer_fields = [f[0] for f in L.Qwen3Layer._fields_]
    src = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{L.HEADER_PATH}"', 'int main(void) {',
           'printf("%zu %zu\\n", sizeof(egpt_qwen3_plan), sizeof(egpt_qwen3_layer));']
    src += [f'printf("%zu\\n", offsetof(egpt_qwen3_plan, {f}));' for f in plan_fields]
    src += [f'printf("%zu\\n", offsetof(egpt_qwen3_layer, {f}));' for f in layer_fields]
    src += ['return 0; }']
    (tmp_path / 'layout.c').write_text('\n'.join(src))
    subprocess.run([cc, '-o', str(tmp_path / 'layout'), str(tmp_path / 'layout.c')], check=True)
    out = subprocess.run([str(tmp_path / 'layout')], check=True, capture_output=True, text=True).stdout.split()
    vals = [int(v) for v in out]
    assert vals[0] == ctypes.sizeof(L.Qwen3Plan) and vals[1] == ctypes.sizeof(L.Qwen3Layer)
    got = vals[2:]
    want = [getattr(L.Qwen3Plan, f).offset for f in plan_fields] + [getattr(L.Qwen3Layer, f).offset for f in layer_fields]
    assert got == want


def test_tp_exchange_size_and_guards():
    lib = L.load()
    assert lib.egpt_tp_xchg_bytes(4096) == 4096 + 2 * 8 * 4096 * 16
    assert lib.egpt_tp_xchg_bytes(0) == 0
    assert lib.egpt_tp_xchg_alloc(None, 64) == L.EGPT_ERR_ARG
    assert lib.egpt_ipc_handle(None, None) == L.EGPT_ERR_ARG
    assert lib.egpt_ipc_open(None, None) == L.EGPT_ERR_ARG
    assert lib.egpt_ipc_close(None) == L.EGPT_OK


def test_dataflow_workspace_and_guards():
    """egpt_dataflow_ws_bytes: 256 B of step state + the LL words of every layer (h, q|k|v, attention, mid
    residual, act: two bf16 per 8-byte word) and the final h."""
    lib = L.load()
    p = L.Qwen3Plan()
    p.n_layers, p.hidden, p.n_q_heads, p.n_kv_heads, p.head_dim, p.intermediate = 28, 2048, 16, 8, 128, 6144
    words = 28 * (1024 + 2048 + 1024 + 1024 + 3072) + 1024
    assert lib.egpt_dataflow_ws_bytes(ctypes.byref(p)) == 256 + 8 * words
    assert lib.egpt_dataflow_ws_bytes(None) == 0
    assert lib.egpt_decode_step_dataflow_check(ctypes.byref(p)) == L.EGPT_ERR_ARG  # null pointers in the plan
    assert lib.egpt_decode_step_dataflow(None, None) == L.EGPT_ERR_ARG
    assert lib.egpt_dataflow_prepare(None) == L.EGPT_ERR_ARG
