"""ctypes binding of libegpt_b200.so (the C-ABI declared in include/egpt_b200.h).

There is no fallback: if the library is missing or no CUDA device is present, every op raises. Status codes
from the library become ValueError (bad shapes, dtypes, alignment, arguments, workspace) or RuntimeError
(launch failures, device-side timeouts), with the library's own message.
"""
import ctypes
import re
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / '_lib' / 'libegpt_b200.so'
HEADER_PATH = _PKG.parent / 'include' / 'egpt_b200.h'

EGPT_OK, EGPT_ERR_SHAPE, EGPT_ERR_DTYPE, EGPT_ERR_ALIGN, EGPT_ERR_LAUNCH, EGPT_ERR_TIMEOUT, EGPT_ERR_ARG, \
    EGPT_ERR_WORKSPACE = range(8)
EGPT_F32, EGPT_BF16 = 0, 1
EPI_NONE, EPI_RESIDUAL, EPI_SILU_MUL, EPI_GELU = 0, 1, 2, 3
FLAG_DOUBLE_ROUND, FLAG_RMSNORM, FLAG_PDL, FLAG_EMBED, FLAG_ADVANCE, FLAG_APPEND, FLAG_NO_TMA = 1, 2, 4, 8, 16, 32, 64
FLAG_REF_SOFTMAX = 128
FLAG_X_F32 = 256
FLAG_EXACT = 512
FLAG_RAGGED = 1024
FLAG_ADD_OUT = 2048

_VALUE_ERRORS = {EGPT_ERR_SHAPE, EGPT_ERR_DTYPE, EGPT_ERR_ALIGN, EGPT_ERR_ARG, EGPT_ERR_WORKSPACE}

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
U32 = ctypes.c_uint
F32 = ctypes.c_float
SZ = ctypes.c_size_t


class Qwen3Layer(ctypes.Structure):
    _fields_ = [('w_qkv', P), ('s_qkv', P), ('w_o', P), ('s_o', P), ('w_gu', P), ('s_gu', P), ('w_down', P),
                ('s_down', P), ('ln_in', P), ('ln_post', P), ('q_norm', P), ('k_norm', P), ('k_cache', P),
                ('v_cache', P)]


class Qwen3Plan(ctypes.Structure):
    _fields_ = [('n_layers', ctypes.c_int32), ('hidden', ctypes.c_int32), ('n_q_heads', ctypes.c_int32),
                ('n_kv_heads', ctypes.c_int32), ('head_dim', ctypes.c_int32), ('intermediate', ctypes.c_int32),
                ('vocab', I64), ('cap', I64), ('eps', F32), ('attn_scale', F32), ('scale_dtype', ctypes.c_int32),
                ('flags', ctypes.c_uint32), ('attn_max_split', ctypes.c_int32), ('layers', ctypes.POINTER(Qwen3Layer)),
                ('embed', P), ('final_norm', P), ('w_lm', P), ('s_lm', P), ('rope_cos', P), ('rope_sin', P),
                ('token', P), ('position', P), ('h', P), ('qkv', P), ('attn', P), ('act', P), ('logits', P),
                ('attn_ws', P), ('attn_ws_bytes', SZ), ('lm_ws', P), ('lm_ws_bytes', SZ),
                ('layers_dev', P), ('sync_ws', P), ('trace', P),
                ('tp_rank', ctypes.c_int32), ('tp_world', ctypes.c_int32), ('tp_xchg', P * 8), ('h2', P),
                ('df_ws', P), ('df_ws_bytes', SZ)]


# name -> (restype, argtypes)
SIGNATURES = {
    'egpt_version': (ctypes.c_char_p, []),
    'egpt_last_error': (ctypes.c_char_p, []),
    'egpt_device_error': (I32, [I32]),
    'egpt_num_sms': (I32, []),
    'egpt_quantize_rows': (I32, [P, P, I32, P, I32, I64, I64, P]),
    'egpt_gemv_i8': (I32, [P, P, I32, I64, I64, I64, P, P, I32, I64, I64, P, P, I32, P, F32, P, U32, P]),
    'egpt_lm_head_ws_bytes': (SZ, [I64]),
    'egpt_lm_head_argmax': (I32, [P, P, P, P, P, P, I32, I64, I64, P, F32, P, SZ, U32, P]),
    'egpt_rmsnorm': (I32, [P, P, P, I64, I64, F32, P]),
    'egpt_layernorm_f32': (I32, [P, P, P, P, I64, I64, F32, P]),
    'egpt_embed': (I32, [P, P, I64, P, P, I64, P, I64, I64, I32, P]),
    'egpt_qk_norm_rope_kv_append': (I32, [P, P, I64, P, P, I64, P, I64, I32, I32, I32, P, P, F32, P, P, I32, P]),
    'egpt_attn_ws_bytes': (SZ, [I64, I32, I32, I32, I32]),
    'egpt_attn_decode': (I32, [P, I64, P, I64, P, P, I64, P, I64, I32, I32, I32, P, P, F32, P, P, F32, I32, P, SZ, I32,
                               U32, P]),
    'egpt_attn_decode_noalloc': (I32, [P, I64, P, I64, P, P, I64, P, I64, I32, I32, I32, P, P, F32, P, P, F32, I32,
                                       I32, U32, P]),
    'egpt_argmax_rows': (I32, [P, P, I64, I64, I64, I32, P]),
    'egpt_sample_ws_bytes': (SZ, [I64]),
    'egpt_attn_prefill': (I32, [P, I64, P, I64, P, P, I64, I64, I64, I32, I32, I32, F32, P]),
    'egpt_silu_mul': (I32, [P, I64, P, I64, I64, I64, P]),
    'egpt_gemm_i8_tc_ws_bytes': (SZ, [I64, I64, I64]),
    'egpt_gemm_i8_tc': (I32, [P, I64, P, I64, I64, P, P, I32, I64, I64, U32, P, SZ, P]),
    'egpt_sample': (I32, [P, I32, I64, I64, I64, F32, I64, F32, P, I64, P, P, I64, P, SZ, P]),
    'egpt_decode_step': (I32, [ctypes.POINTER(Qwen3Plan), P]),
    'egpt_step_sync_ws_bytes': (SZ, []),
    'egpt_decode_step_persistent': (I32, [ctypes.POINTER(Qwen3Plan), P]),
    'egpt_decode_step_persistent_check': (I32, [ctypes.POINTER(Qwen3Plan)]),
    'egpt_dataflow_ws_bytes': (SZ, [ctypes.POINTER(Qwen3Plan)]),
    'egpt_dataflow_prepare': (I32, [ctypes.POINTER(Qwen3Plan)]),
    'egpt_decode_step_dataflow': (I32, [ctypes.POINTER(Qwen3Plan), P]),
    'egpt_decode_step_dataflow_check': (I32, [ctypes.POINTER(Qwen3Plan)]),
    'egpt_tp_xchg_bytes': (SZ, [I64]),
    'egpt_tp_xchg_alloc': (I32, [ctypes.POINTER(P), SZ]),
    'egpt_tp_xchg_free': (I32, [P]),
    'egpt_ipc_handle': (I32, [P, P]),
    'egpt_ipc_open': (I32, [P, ctypes.POINTER(P)]),
    'egpt_ipc_close': (I32, [P]),
}

_lib = None


def header_functions(path=HEADER_PATH):
    """Names of the functions declared in the public header (used by the export test)."""
    text = Path(path).read_text()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    return sorted(set(re.findall(r'\b(egpt_[a-z0-9_]+)\s*\(', text)))


def load():
    """Load the library once; raise if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f'{LIB_PATH} is missing: run `python -m efficientgpt_b200.build` (no CPU fallback)')
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error():
    return load().egpt_last_error().decode(errors='replace')


def check(rc, what):
    if rc == EGPT_OK:
        return
    msg = f'{what}: {last_error()} (status {rc})'
    if rc in _VALUE_ERRORS:
        raise ValueError(msg)
    raise RuntimeError(msg)


def device_error(clear=True):
    """Synchronise and return the device error word (0 = ok)."""
    return int(load().egpt_device_error(1 if clear else 0))
