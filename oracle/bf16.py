"""bf16 <-> float32 bit conversions in numpy (test infrastructure only)."""
import numpy as np


def bits_to_f32(bits):
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bits(x):
    """float32 -> bf16 bit patterns, round to nearest even; NaN stays NaN (quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    nan = np.isnan(x)
    if nan.any():
        rounded = np.where(nan, ((u >> 16) | 0x40) & 0xFFFF, rounded)
    return rounded.astype(np.uint16)


def round_f32(x):
    """float32 values rounded through bf16 (what `.to(torch.bfloat16)` keeps)."""
    return bits_to_f32(f32_to_bits(x))
