"""bf16 helpers on numpy float32 arrays (test infrastructure; see oracle/__init__.py).

PyTorch's float32 -> bfloat16 cast is round-to-nearest-even on the upper 16 bits (NaN stays NaN); these
helpers reproduce it so the oracle can round at the same points as the reference's eager bf16 model.
"""
import numpy as np


def round_bf16(a):
    """float32 array -> float32 array whose values are the nearest-even bf16 values."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.nan
    return out


def from_bits(bits):
    """uint16 bf16 bit patterns -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_bits(a):
    """float32 -> uint16 bf16 bit patterns (round to nearest even)."""
    return (round_bf16(a).view(np.uint32) >> 16).astype(np.uint16)


def from_torch(t):
    """torch tensor (any float dtype, any device) -> float32 numpy array of the same values."""
    import torch
    return t.detach().to(device='cpu', dtype=torch.float32).numpy()
