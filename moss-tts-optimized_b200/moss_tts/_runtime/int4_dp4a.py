"""``int4_dp4a`` of the reference, as W4A16 on the B200 kernels.

``int4_dp4a(x, packed, scales, group=128, warps=4, reciprocal=False, prequantized=None,
grouped_activation=False)`` keeps the reference's signature and errors
(``src/moss_tts/_runtime/int4_dp4a.py:56-74``): one contiguous bf16 row against signed-nibble
weights with per-group scales, output ``[..., N]`` bf16. The reference quantizes the
activation to int8 first (``int4_dp4a.py:21-30``); this keeps it bf16 (W4A16, fp32
accumulation), so ``prequantized`` is rejected and ``reciprocal`` / ``grouped_activation``
(choices of that int8 quantizer) only pass their reference validation. The kernels use G32
groups, the reference's calibrated format; other group sizes are rejected.
"""
import torch

from . import native
from .kernels import _cuda
from .quantized import from_signed


def int4_dp4a(x, packed, scales, group=128, warps=4, reciprocal=False, prequantized=None,
              grouped_activation=False):
    n, k2 = packed.shape
    k = k2 * 2
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.numel() != k:
        raise ValueError("Expected one contiguous BF16 activation row")
    if prequantized is not None:
        raise ValueError("Invalid prequantized activation: W4A16 takes the bf16 activation")
    if grouped_activation and not reciprocal:
        raise ValueError("Grouped activation uses explicit reciprocal rounding")
    if group != 32:
        raise ValueError("Only G32 groups are supported")
    if warps not in (1, 2, 4, 8):
        raise ValueError("Unsupported warp count")
    _cuda(x, packed, scales)
    qweight, s = from_signed(packed, scales, group=group)
    out = torch.empty((*x.shape[:-1], n), device=x.device, dtype=x.dtype)
    native.call("mt_w4a16_linear", x.data_ptr(), None, None, 0.0, None, qweight.data_ptr(), s.data_ptr(), None,
                out.data_ptr(), 1, n, k, group, 0, 0, native.stream_of(x))
    return out
