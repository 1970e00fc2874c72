"""int4 / G32 weight formats and dequantization (oracle, test infrastructure only).

Two on-device formats share one byte layout, ``packed uint8 [N, K/2]`` with the
low nibble holding even ``k`` and the high nibble odd ``k``
(reference ``src/moss_tts/calibration.py:190-191``). Viewed little-endian as
``int32 [N, K/8]``, nibble ``j`` of word ``i`` is element ``k = 8*i + j``: the
"8 codes per int32 along K" GPTQ packing.

* signed (the reference's calibrated export): two's-complement codes in [-7, 7],
  ``W = bf16(code * scale)`` (``_runtime/calibrated_backend.py:8-13``,
  ``_runtime/calibrated_quant.py:41-42``).
* zero-point (GPTQ W4A16): unsigned codes ``q`` in [0, 15] with one 4-bit zero
  point ``z`` per group, ``W = bf16((q - z) * scale)``; zero points are packed
  two per byte along the group axis, ``uint8 [N, K/G/2]`` (low nibble = even
  group). The signed format is the special case ``q = code + 8``, ``z = 8``.

Both products are exact in fp32 (|q - z| <= 15 times an 8-bit bf16 mantissa),
so the single fp32 -> bf16 rounding defines the dequantized weight bit-exactly.
"""
import numpy as np

from .numerics import round_bf16, to_f32


def unpack_u4(packed) -> np.ndarray:
    """uint8 [N, K/2] -> uint8 [N, K] nibbles, low nibble first."""
    p = np.asarray(packed).view(np.uint8)
    n = p.shape[0]
    out = np.empty((n, p.shape[1] * 2), dtype=np.uint8)
    out[:, 0::2] = p & 15
    out[:, 1::2] = p >> 4
    return out


def pack_u4(values) -> np.ndarray:
    """uint8 [N, K] nibbles in [0, 15] -> uint8 [N, K/2] (low nibble = even index)."""
    v = np.asarray(values, dtype=np.uint8)
    return (v[:, 0::2] | (v[:, 1::2] << 4)).astype(np.uint8)


def unpack_signed(packed) -> np.ndarray:
    """Two's-complement nibbles -> int8 codes.

    Follows ``src/moss_tts/_runtime/calibrated_backend.py:8-13`` (``unpack_signed``).
    """
    u = unpack_u4(packed).astype(np.int8)
    return np.where(u >= 8, u - 16, u).astype(np.int8)


def signed_to_unsigned(packed) -> np.ndarray:
    """Signed-code bytes -> zero-point bytes with ``q = code + 8`` (so ``z = 8``).

    Flipping bit 3 of a 4-bit two's-complement value adds 8 modulo 16, which
    maps [-8, 7] onto [0, 15] monotonically.
    """
    return (np.asarray(packed).view(np.uint8) ^ np.uint8(0x88)).astype(np.uint8)


def dequantize_signed(signed, scales, group: int = 32) -> np.ndarray:
    """``bf16(code * scale)``, following ``_runtime/calibrated_quant.py:41-42``."""
    c = np.asarray(signed).astype(np.float32)
    s = to_f32(scales)
    n, k = c.shape
    w = c.reshape(n, k // group, group) * s[:, :, None]
    return round_bf16(w.reshape(n, k))


def dequantize_w4(qweight, scales, qzeros, group: int = 32) -> np.ndarray:
    """``bf16((q - z) * scale)`` for the zero-point format.

    ``qweight`` is the packed ``uint8 [N, K/2]`` (or its ``int32 [N, K/8]`` view);
    ``qzeros`` is ``uint8 [N, K/G/2]`` or ``None`` for the implicit ``z = 8``.
    Restates the reference's dequantization (``_runtime/calibrated_quant.py:41-42``)
    with the per-group zero point subtracted before the scale.
    """
    q = unpack_u4(np.ascontiguousarray(qweight).view(np.uint8)).astype(np.float32)
    n, k = q.shape
    g = k // group
    if qzeros is None:
        z = np.full((n, g), 8.0, dtype=np.float32)
    else:
        z = unpack_u4(np.ascontiguousarray(qzeros).view(np.uint8)).astype(np.float32)[:, :g]
    s = to_f32(scales)
    w = (q.reshape(n, g, group) - z[:, :, None]) * s[:, :, None]
    return round_bf16(w.reshape(n, k))
