"""``dp4a_norm_projection`` of the reference, as W4A16 on the B200 kernels.

``linear(x, residual, norm_weight, eps, w, s, *, fused=False, rows=4, integer_groups=1,
integer_rows=1, debug=False)`` keeps the reference's signature, validation and return
shape (``src/moss_tts/_runtime/dp4a_norm_projection.py:99-117``): the bf16 residual add and
RMSNorm prologue feed the projection in the same launch, and ``fused=True`` is the paired
gate/up with SiLU·up. The reference's third result for ``fused`` is the int8 quantization of
the output for its W4A8 down projection; here the down projection takes the bf16 output, so
that slot is ``None`` and ``dp4a_packing.project(mlp, "down", y, None)`` consumes it as the
reference's ``hidden`` loop does (``dp4a_norm_projection.py:138-163``). ``debug`` returned the
int8 intermediates of the W4A8 path and is rejected.
"""
import torch

from . import native
from .quantized import from_signed

SELECTED = {"qkv": {"rows": 8, "integer_groups": 1, "integer_rows": 1},
            "up": {"rows": 32, "integer_groups": 2, "integer_rows": 4}}


def linear(x, residual, norm_weight, eps, w, s, *, fused=False, rows=4, integer_groups=1, integer_rows=1,
           debug=False):
    n2, k2 = w.shape
    n = n2 // 2 if fused else n2
    if x.numel() != 4096 or x.dtype != torch.bfloat16 or k2 != 2048 or n <= 0 or norm_weight.numel() != 4096:
        raise ValueError("One BF16 K4096 activation row required")
    if integer_groups not in (1, 2, 4) or integer_rows not in (1, 2, 4) or rows not in ((32, 64) if fused else (4, 8, 16)):
        raise ValueError("Unsupported fusion tile")
    if fused and n2 % 64:
        raise ValueError("Complete gate/up output quantization groups required")
    tensors = (x, norm_weight, w, s) + (() if residual is None else (residual,))
    if not x.is_cuda or any(t.device != x.device or not t.is_contiguous() for t in tensors):
        raise ValueError("Contiguous CUDA inputs required")
    if norm_weight.dtype != torch.bfloat16 or residual is not None and (residual.dtype != x.dtype or residual.shape != x.shape) \
            or w.dtype != torch.uint8 or s.shape != (n2, 128) or s.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("Invalid norm, residual or grouped weight buffers")
    if debug:
        raise ValueError("debug returns the W4A8 int8 intermediates, which W4A16 does not form")
    qweight, scales = from_signed(w, s)
    summed = torch.empty_like(x) if residual is not None else x
    y = torch.empty((*x.shape[:-1], n), device=x.device, dtype=x.dtype)
    mode = native.LINEAR_NORM | (native.LINEAR_ADD if residual is not None else 0) | (native.LINEAR_PAIRED if fused else 0)
    native.call("mt_w4a16_linear", x.data_ptr(), native.ptr(residual), norm_weight.data_ptr(), float(eps),
                summed.data_ptr() if residual is not None else None, qweight.data_ptr(), scales.data_ptr(), None,
                y.data_ptr(), 1, n2, 4096, 32, mode, 0, native.stream_of(x))
    return (summed, y, None) if fused else (summed, y)
