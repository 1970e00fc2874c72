"""bf16 helpers for the numpy oracle (test infrastructure only).

numpy has no bfloat16 type, so bf16 tensors are carried either as uint16 bit
patterns (storage, fixtures) or as float32 arrays whose values are exactly
representable in bf16 (arithmetic). ``round_bf16`` is the single rounding
primitive: IEEE round-to-nearest-even from fp32 to bf16, the rounding every
``.to(tl.bfloat16)`` / ``.bfloat16()`` in the reference performs
(e.g. ``src/moss_tts/_runtime/kernels.py:57,76,80``).
"""
import numpy as np


def round_bf16(x) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); returns float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    # uint32 wrap-around is impossible for finite inputs (|bits| <= 0xFF7FFFFF)
    r = (u + (((u >> 16) & np.uint32(1)) + np.uint32(0x7FFF))) & np.uint32(0xFFFF0000)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, np.uint32(0x7FC00000), r)
    return r.view(np.float32).reshape(x.shape)


def bf16_bits(x) -> np.ndarray:
    """fp32 values -> uint16 bf16 bit patterns (rounding first)."""
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits) -> np.ndarray:
    """uint16 bf16 bit patterns -> exact float32 values."""
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def to_f32(x) -> np.ndarray:
    """Accept either uint16 bf16 bits or float arrays; return float32 values."""
    x = np.asarray(x)
    if x.dtype == np.uint16:
        return from_bf16_bits(x)
    return x.astype(np.float32, copy=False)
