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


def gptq_prepare(weight, inputs, damping: float = 0.01, actorder: bool = True):
    """The Hessian set-up of ``calibrated_quant.gptq`` (``_runtime/calibrated_quant.py:52-62``):
    ``H = 2/m X^T X``, dead columns (zero diagonal) get ``H[d, d] = 1`` and zero weights, the
    act-order permutation (diagonal descending), damping by ``damping * mean(diag)``, and the
    upper Cholesky factor of ``H^-1``. Returns ``(w [N, K] fp32 permuted, hinv [K, K] fp32,
    perm int64 [K])``.

    This is dense linear algebra (Cholesky, inverse), not the quantization arithmetic, so it is
    run with the same torch CPU calls the reference makes: identical inputs give identical
    factors, which is what lets the column loop below be compared bit for bit.
    """
    import torch

    w32 = torch.from_numpy(to_f32(weight).copy())
    x = torch.from_numpy(np.asarray(inputs, dtype=np.float32))
    h = (x.T @ x) * (2 / x.shape[0])
    dead = h.diagonal() == 0
    h[dead, dead] = 1
    w32[:, dead] = 0
    k = w32.shape[1]
    perm = torch.argsort(h.diagonal(), descending=True) if actorder else torch.arange(k)
    w32 = w32[:, perm].contiguous()
    h = h[perm][:, perm].contiguous()
    h.diagonal().add_(damping * h.diagonal().mean())
    hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(h)), upper=True).contiguous()
    return w32.numpy(), hinv.numpy(), perm.numpy()


def gptq_block(chunk, hinv, perm, scales, start: int, group: int = 32):
    """The column loop of one GPTQ block (``_runtime/calibrated_quant.py:67-82``, torch backend;
    the Triton ``_column`` kernel, ``calibrated_quant.py:15-33``, does the same per column).

    ``chunk`` fp32 ``[N, B]`` (columns ``start .. start+B`` of the permuted weights) is updated in
    place; returns ``(codes int8 [N, B] in permuted column order, errors fp32 [N, B])``. Every
    step is one IEEE fp32 operation rounded on its own, in the reference's order:
    ``code = clamp(rint(w / s), -7, 7)``, ``q = bf16(code * s)``, ``e = (w - q) / hinv[c, c]``,
    ``chunk[:, c:] -= e * hinv[c, c:]`` (a product, then a difference).
    """
    n, b = chunk.shape
    s_all = to_f32(scales)
    codes = np.empty((n, b), dtype=np.int8)
    errors = np.zeros((n, b), dtype=np.float32)
    for c in range(b):
        col = start + c
        scale = s_all[:, int(perm[col]) // group]
        value = chunk[:, c].copy()
        code = np.clip(np.rint(value / scale), -7, 7).astype(np.float32)
        q = round_bf16(code * scale)
        err = ((value - q) / hinv[col, col]).astype(np.float32)
        codes[:, c] = code.astype(np.int8)
        chunk[:, c:] -= (err[:, None] * hinv[col, col:start + b][None, :]).astype(np.float32)
        errors[:, c] = err
    return codes, errors


def gptq(weight, inputs, group: int = 32, damping: float = 0.01, actorder: bool = True, block: int = 128,
         scales=None):
    """Whole ``calibrated_quant.gptq`` (``_runtime/calibrated_quant.py:45-85``): static scales
    (``static_scales``) unless given, the Hessian set-up, the per-block column loop and the
    trailing update ``w[:, end:] -= errors @ hinv[start:end, end:]`` (torch CPU matmul, as the
    reference). Returns ``(signed int8 [N, K] in original column order, scales bf16 bits)``."""
    import torch

    n, k = np.asarray(weight).shape
    if scales is None:
        scales = static_scales(weight, group)
    w, hinv, perm = gptq_prepare(weight, inputs, damping, actorder)
    signed = np.empty((n, k), dtype=np.int8)
    for start in range(0, k, block):
        end = start + block
        chunk = np.ascontiguousarray(w[:, start:end])
        codes, errors = gptq_block(chunk, hinv, perm, scales, start, group)
        signed[:, perm[start:end]] = codes
        if end < k:
            upd = torch.from_numpy(errors) @ torch.from_numpy(np.ascontiguousarray(hinv[start:end, end:]))
            w[:, end:] -= upd.numpy()
    return signed, np.asarray(scales)


def static_scales(weight, group: int = 32) -> np.ndarray:
    """``bf16(max(absmax over the group, 1e-8) / 7)`` per group of ``group`` input columns
    (``_runtime/calibrated_quant.py:36-38``); returns uint16 bf16 bits."""
    from .numerics import bf16_bits

    w = to_f32(weight)
    n, k = w.shape
    a = np.abs(w).reshape(n, k // group, group).max(-1)
    return bf16_bits(np.maximum(a, np.float32(1e-8)) / np.float32(7))
