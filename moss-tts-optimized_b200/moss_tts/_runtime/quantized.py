"""W4A16 G32 quantized linear: the B200 replacement of the reference's dp4a projections.

Signatures follow the reference's quantized-linear modules
(``src/moss_tts/_runtime/dp4a_packing.py:94-106`` ``linear``,
``dp4a_norm_projection.py:99-117`` fused norm ``linear``, ``int4_dp4a.py:56``) with
the activation kept in bf16 (W4A16): ``prequantized`` int8 activations belong to
the reference's W4A8 approximation and are rejected.

Weights: ``packed`` uint8 ``[N, K/2]`` (or its int32 ``[N, K/8]`` view), ``scales``
bf16 ``[N, K/32]``, optional ``zeros`` uint8 ``[N, K/64]`` (None = symmetric codes
stored with ``q = code + 8``, see ``calibrated_backend.to_zero_point``).
"""
import torch

from . import native
from .kernels import _bf16, _cuda


def _weights(packed, scales, zeros, group):
    if group != 32:
        raise ValueError("Only G32 groups are supported")
    if packed.dtype == torch.int32:
        packed = packed.view(torch.uint8)
    if packed.dtype != torch.uint8 or packed.ndim != 2:
        raise ValueError("packed weights must be uint8 [N, K/2] or int32 [N, K/8]")
    n, k = packed.shape[0], packed.shape[1] * 2
    if scales.dtype != torch.bfloat16 or scales.shape != (n, k // group):
        raise ValueError("scales must be bf16 [N, K/32]")
    if zeros is not None and (zeros.dtype != torch.uint8 or zeros.shape != (n, k // (2 * group))):
        raise ValueError("zeros must be uint8 [N, K/64]")
    if packed.data_ptr() % 16:
        raise ValueError("packed weights must be 16-byte aligned")
    return packed, n, k


_WORKSPACES: dict = {}


def gemm_workspace(device, batch: int, n: int, k: int, paired: bool = False) -> torch.Tensor:
    """Zero-filled workspace of ``mt_w4a16_gemm`` for this shape, cached per device and grown
    on demand (the kernel leaves its tickets zero, so calls ordered on one stream share it)."""
    nbytes = native.w4a16_gemm_workspace(batch, n, k, native.LINEAR_PAIRED if paired else 0)
    dev = torch.device(device)
    ws = _WORKSPACES.get(dev)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
        _WORKSPACES[dev] = ws
    return ws


def linear(x, packed, scales, zeros=None, *, group=32, paired=False, prequantized=None, pdl=False):
    """``y = x @ dequant(W).T`` in bf16 with fp32 accumulation, for 1..128 activation rows.

    ``paired=True`` treats rows ``[0, N/2)`` as gate and ``[N/2, N)`` as up and returns
    ``bf16(bf16(silu(gate)) * up)`` with ``N/2`` columns (``dp4a_packing.py:85-89``).
    Up to 8 rows run the CUDA-core GEMV; 9..128 rows run the
    tcgen05 tensor-core GEMM (N % 128 == 0, K % 256 == 0) with a cached workspace.
    """
    if prequantized is not None:
        raise ValueError("W4A16 takes bf16 activations; int8 prequantized inputs are not used")
    x = x.contiguous()
    packed, n, k = _weights(packed, scales, zeros, group)
    _cuda(x, packed, scales, zeros)
    _bf16(x)
    rows = x.numel() // x.shape[-1]
    if x.shape[-1] != k or not 1 <= rows <= 128:
        raise ValueError("Expected 1..128 contiguous bf16 activation rows of width K")
    out_n = n // 2 if paired else n
    y = torch.empty((*x.shape[:-1], out_n), device=x.device, dtype=x.dtype)
    mode = native.LINEAR_PAIRED if paired else 0
    flags = native.FLAG_PDL if pdl else 0
    if rows <= 8:
        native.call("mt_w4a16_linear", x.data_ptr(), None, None, 0.0, None, packed.data_ptr(),
                    scales.data_ptr(), native.ptr(zeros), y.data_ptr(), rows, n, k, group, mode, flags,
                    native.stream_of(x))
        return y
    if n % 128 or k % 256:
        raise ValueError("More than 8 rows need N a multiple of 128 and K a multiple of 256")
    ws = gemm_workspace(x.device, rows, n, k, paired)
    native.call("mt_w4a16_gemm", x.data_ptr(), packed.data_ptr(), scales.data_ptr(), native.ptr(zeros),
                y.data_ptr(), rows, n, k, mode, ws.data_ptr(), flags, native.stream_of(x))
    return y


def norm_linear(x, residual, norm_weight, eps, packed, scales, zeros=None, *, paired=False,
                group=32, pdl=False):
    """Residual add + RMSNorm prologue fused into the projection.

    Mirrors ``dp4a_norm_projection.linear`` (``dp4a_norm_projection.py:99-117``):
    returns ``(summed, y)`` where ``summed = bf16(x + residual)`` (or ``x`` when
    ``residual`` is None) and ``y = linear(rmsnorm(summed), W)``.
    """
    x = x.contiguous()
    packed, n, k = _weights(packed, scales, zeros, group)
    _cuda(x, residual, norm_weight, packed, scales, zeros)
    _bf16(x, residual, norm_weight)
    rows = x.numel() // x.shape[-1]
    if x.shape[-1] != k or not 1 <= rows <= 8 or norm_weight.numel() != k:
        raise ValueError("Expected 1..8 bf16 rows of width K and a [K] norm weight")
    if residual is not None and residual.shape != x.shape:
        raise ValueError("residual shape differs from x")
    summed = torch.empty_like(x) if residual is not None else x
    out_n = n // 2 if paired else n
    y = torch.empty((*x.shape[:-1], out_n), device=x.device, dtype=x.dtype)
    mode = native.LINEAR_NORM | (native.LINEAR_ADD if residual is not None else 0)
    mode |= native.LINEAR_PAIRED if paired else 0
    native.call("mt_w4a16_linear", x.data_ptr(), native.ptr(residual), norm_weight.data_ptr(),
                float(eps), summed.data_ptr() if residual is not None else None, packed.data_ptr(),
                scales.data_ptr(), native.ptr(zeros), y.data_ptr(), rows, n, k, group, mode,
                native.FLAG_PDL if pdl else 0, native.stream_of(x))
    return summed, y


def interleave_nibbles(packed):
    """The reference's load-time nibble interleave (``dp4a_packing.py:15-19``): within every
    4-byte word, codes 0..3 move to the low nibbles and codes 4..7 to the high nibbles."""
    n, k2 = packed.shape
    if packed.dtype != torch.uint8 or k2 % 4:
        raise ValueError("Expected signed-nibble pairs with K divisible by eight")
    unsigned = torch.stack([packed & 15, packed >> 4], dim=-1).reshape(n, -1, 8)
    return (unsigned[:, :, :4] | (unsigned[:, :, 4:] << 4)).reshape(n, k2).contiguous()


def deinterleave_nibbles(packed):
    """Inverse of ``interleave_nibbles``: back to code k in nibble ``k & 1`` of byte ``k / 2``."""
    n, k2 = packed.shape
    if packed.dtype != torch.uint8 or k2 % 4:
        raise ValueError("Expected signed-nibble pairs with K divisible by eight")
    words = packed.reshape(n, -1, 4)
    unsigned = torch.cat([words & 15, words >> 4], dim=-1).reshape(n, -1, 8)
    return (unsigned[:, :, 0::2] | (unsigned[:, :, 1::2] << 4)).reshape(n, k2).contiguous()


_SIGNED: dict = {}


def from_signed(packed, scales, *, group: int = 32, interleaved: bool = False):
    """Reference-format weights -> this library's W4 operands ``(qweight, bf16 scales)``.

    The reference stores two's-complement codes in [-7, 7] (``calibration.py:190-191``) with
    fp32 or bf16 scales (``calibrated_backend.py:51``, ``dp4a_packing.py:149-155``); flipping
    bit 3 of every nibble gives ``q = code + 8`` with the implicit zero point 8, so the
    dequantized weights are unchanged bit for bit. Scales must be exactly representable in
    bf16 (the reference's own check before it narrows them). The converted copy is made once
    per source tensor and reused while the source is alive and unmodified.
    """
    if group != 32:
        raise ValueError("Only G32 groups are supported")
    if packed.dtype != torch.uint8 or packed.ndim != 2:
        raise ValueError("packed weights must be uint8 [N, K/2] signed nibbles")
    n, k = packed.shape[0], packed.shape[1] * 2
    if scales.shape != (n, k // group) or scales.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("scales must be float32 or bfloat16 [N, K/32]")
    key = (id(packed), packed._version, id(scales), scales._version, bool(interleaved))
    hit = _SIGNED.get(id(packed))
    if hit is not None and hit[0] == key:
        return hit[1], hit[2]
    if scales.dtype != torch.bfloat16:
        if not torch.equal(scales, scales.bfloat16().float()):
            raise ValueError("Scales are not exactly representable in bf16")
        scales = scales.bfloat16()
    codes = deinterleave_nibbles(packed) if interleaved else packed
    qweight = (codes ^ 0x88).contiguous()
    scales = scales.contiguous()
    import weakref
    if hit is None:
        weakref.finalize(packed, _SIGNED.pop, id(packed), None)
    _SIGNED[id(packed)] = (key, qweight, scales)
    return qweight, scales


def dequantize_packed(packed, scales, zeros=None, group=32):
    """Bit-exact ``bf16((q - z) * s)`` of a packed W4 matrix, ``[N, K]``."""
    packed, n, k = _weights(packed, scales, zeros, group)
    _cuda(packed, scales, zeros)
    out = torch.empty((n, k), device=packed.device, dtype=torch.bfloat16)
    native.call("mt_dequant_w4", packed.data_ptr(), scales.data_ptr(), native.ptr(zeros),
                out.data_ptr(), n, k, group, native.stream_of(packed))
    return out
