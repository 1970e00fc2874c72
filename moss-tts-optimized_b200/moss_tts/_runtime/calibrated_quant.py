"""``calibrated_quant`` of the reference: static G32 scales and bit-exact dequantization.

Same names and signatures as ``src/moss_tts/_runtime/calibrated_quant.py``:

* ``static_scales(weight, group=32)`` = ``bf16(max(absmax over the group, 1e-8) / 7)``
  (``calibrated_quant.py:36-38``), one scale per group of ``group`` input columns;
* ``dequantize(signed, scales, group)`` = ``bf16(float(code) * float(scale))``
  (``calibrated_quant.py:41-42``) for int8 codes ``[N, K]`` in [-8, 7], computed by the
  library's bit-exact dequantization kernel (the codes are packed to nibbles with ``q = code
  + 8`` and zero point 8 on the way; the product is exact in fp32, so one rounding defines
  every output bit).

The GPTQ solver of the same reference module (``gptq``, ``calibrated_quant.py:45-85``) is
offline calibration and lives in ``gptq_solver``.
"""
import torch

from . import native
from .kernels import _cuda


def static_scales(weight, group=32):
    n, k = weight.shape
    if k % group:
        raise ValueError("K must be a multiple of the group size")
    _cuda(weight)
    if weight.dtype not in (torch.bfloat16, torch.float32, torch.float16):
        raise ValueError("floating-point weights required")
    if group != 32:
        raise ValueError("Only G32 groups are supported")
    out = torch.empty((n, k // group), device=weight.device, dtype=torch.bfloat16)
    w = weight.contiguous()
    native.call("mt_static_scales", w.data_ptr(), {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2}[w.dtype],
                out.data_ptr(), n, k, native.stream_of(w))
    return out


def dequantize(signed, scales, group):
    """``bf16(code * scale)`` of int8 codes ``[N, K]`` with per-group scales ``[N, K / group]``."""
    if signed.dtype != torch.int8 or signed.ndim != 2:
        raise ValueError("int8 codes [N, K] required")
    n, k = signed.shape
    if group != 32 or k % 64:
        raise ValueError("Only G32 groups over K divisible by 64 are supported")
    if scales.shape != (n, k // group):
        raise ValueError("scales must be [N, K / group]")
    _cuda(signed, scales)
    if scales.dtype != torch.bfloat16:
        if not torch.equal(scales.float(), scales.float().bfloat16().float()):
            raise ValueError("Scales are not exactly representable in bf16")
        scales = scales.bfloat16()
    c = signed.contiguous().view(torch.uint8)
    qweight = (((c[:, 0::2] & 15) | ((c[:, 1::2] & 15) << 4)) ^ 0x88).contiguous()
    out = torch.empty((n, k), device=signed.device, dtype=torch.bfloat16)
    native.call("mt_dequant_w4", qweight.data_ptr(), scales.contiguous().data_ptr(), None, out.data_ptr(), n, k,
                group, native.stream_of(signed))
    return out
