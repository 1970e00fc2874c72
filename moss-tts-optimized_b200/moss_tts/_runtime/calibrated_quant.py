"""``calibrated_quant`` of the reference: static G32 scales and bit-exact dequantization.

Same names and signatures as ``src/moss_tts/_runtime/calibrated_quant.py``:

* ``static_scales(weight, group=32)`` = ``bf16(max(absmax over the group, 1e-8) / 7)``
  (``calibrated_quant.py:36-38``), one scale per group of ``group`` input columns;
* ``dequantize(signed, scales, group)`` = ``bf16(float(code) * float(scale))``
  (``calibrated_quant.py:41-42``) for int8 codes ``[N, K]`` in [-8, 7], computed by the
  library's bit-exact dequantization kernel (the codes are packed to nibbles with ``q = code
  + 8`` and zero point 8 on the way; the product is exact in fp32, so one rounding defines
  every output bit).

* ``gptq(weight, inputs, group=32, damping=.01, actorder=True, block=128, backend='triton',
  scales_override=None)`` (``calibrated_quant.py:45-85``): the Hessian set-up and the trailing
  block updates are the reference's torch calls (Cholesky, matmul) on the device; the column
  loop of each 128-column block is one launch of ``mt_gptq_block`` instead of one Triton
  ``_column`` launch per column. ``backend`` accepts the reference's ``'triton'`` (the fused
  column kernel) and ``'cuda'``; the codes are bit-identical to the reference's column loop on
  the same block inputs.
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


@torch.inference_mode()
def gptq(weight, inputs, group=32, damping=.01, actorder=True, block=128, backend="triton", scales_override=None):
    """Signed G32 codes ``int8 [N, K]`` in [-7, 7] and their static bf16 scales, by GPTQ error
    feedback over calibration inputs ``[m, K]`` (``calibrated_quant.py:45-85``)."""
    n, k = weight.shape
    if k % block or k % group:
        raise ValueError("Dimensions must be divisible by group/block sizes")
    if inputs.ndim != 2 or inputs.shape[1] != k:
        raise ValueError("Calibration input shape mismatch")
    if backend not in ("triton", "cuda"):
        raise ValueError("Unknown GPTQ backend")
    if block > 128:
        raise ValueError("GPTQ blocks of at most 128 columns are supported")
    _cuda(weight, inputs)
    scales = static_scales(weight, group) if scales_override is None else scales_override
    if (scales.shape != (n, k // group) or scales.dtype != torch.bfloat16 or scales.device != weight.device
            or not scales.is_contiguous() or not torch.isfinite(scales).all() or not (scales > 0).all()):
        raise ValueError("Invalid static group scales")
    x = inputs.float()
    h = (x.T @ x) * (2 / x.shape[0])
    dead = h.diagonal() == 0
    h[dead, dead] = 1
    w = weight.float().clone()
    w[:, dead] = 0
    perm = torch.argsort(h.diagonal(), descending=True) if actorder else torch.arange(k, device=w.device)
    w = w[:, perm].contiguous()
    h = h[perm][:, perm].contiguous()
    h.diagonal().add_(damping * h.diagonal().mean())
    hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(h)), upper=True).contiguous()
    del h, x
    perm = perm.to(torch.int64).contiguous()
    signed = torch.empty((n, k), device=w.device, dtype=torch.int8)
    s = native.stream_of(w)
    for start in range(0, k, block):
        end = start + block
        chunk = w[:, start:end].contiguous()
        errors = torch.empty_like(chunk)
        native.call("mt_gptq_block", chunk.data_ptr(), errors.data_ptr(), signed.data_ptr(), scales.data_ptr(),
                    hinv.data_ptr(), perm.data_ptr(), start, block, n, k, group, s)
        if end < k:
            w[:, end:] -= errors @ hinv[start:end, end:]
    return signed, scales
