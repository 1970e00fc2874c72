"""``dp4a_packing`` of the reference, as W4A16 on the B200 kernels.

Same module name and call signatures as ``src/moss_tts/_runtime/dp4a_packing.py``:
``pack_interleaved`` / ``unpack_interleaved`` (``:15-27``), ``linear`` (``:94-106``),
``project`` (``:109-125``) and ``install_packing`` (``:128-160``). Weights stay in the
reference's format -- two's-complement nibbles in [-7, 7], optionally interleaved, with
fp32 or bf16 G32 scales -- and are handed to the W4A16 GEMV with the implicit zero point 8
(``quantized.from_signed``). The activation stays bf16: the reference's int8 activation
(``prequantized``) belongs to its W4A8 approximation and is rejected. The reference's
tile knobs (``rows``, ``warps``) are validated and otherwise unused.
"""
import json
from pathlib import Path

import torch

from . import native
from .kernels import _cuda
from .quantized import deinterleave_nibbles, from_signed, interleave_nibbles

_TILES = (1, 2, 4, 8)


def pack_interleaved(packed):
    """Codes 0..3 of every 8 into the low nibbles, 4..7 into the high (``dp4a_packing.py:15-19``)."""
    return interleave_nibbles(packed)


def unpack_interleaved(packed):
    """Interleaved nibbles -> int8 codes in [-8, 7] (``dp4a_packing.py:22-27``)."""
    plain = deinterleave_nibbles(packed)
    lo, hi = (plain & 15).to(torch.int8), (plain >> 4).to(torch.int8)
    codes = torch.stack([lo, hi], dim=-1).reshape(plain.shape[0], -1)
    return torch.where(codes >= 8, codes - 16, codes)


def linear(x, packed, scales, *, group=32, rows=1, warps=1, interleaved=False, paired=False,
           prequantized=None):
    """One bf16 activation row times signed-nibble G32 weights, ``y = bf16(x . W^T)`` with
    fp32 accumulation; ``paired`` returns ``bf16(bf16(silu(gate)) * up)`` over the two halves
    (``dp4a_packing.py:85-89``). Output ``[..., N]`` (``N / 2`` when paired)."""
    n, k2 = packed.shape
    k = k2 * 2
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.numel() != k:
        raise ValueError("One contiguous BF16 input row required")
    if prequantized is not None:
        raise ValueError("W4A16 takes the bf16 activation; int8 prequantized inputs are not used")
    if rows not in _TILES or warps not in _TILES:
        raise ValueError("Unsupported tile")
    if paired and n % 8:
        raise ValueError("Paired gate/up needs N divisible by eight")
    _cuda(x, packed, scales)
    qweight, s = from_signed(packed, scales, group=group, interleaved=interleaved)
    out_n = n // 2 if paired else n
    out = torch.empty((*x.shape[:-1], out_n), device=x.device, dtype=x.dtype)
    native.call("mt_w4a16_linear", x.data_ptr(), None, None, 0.0, None, qweight.data_ptr(), s.data_ptr(), None,
                out.data_ptr(), 1, n, k, group, native.LINEAR_PAIRED if paired else 0, 0, native.stream_of(x))
    return out


def project(module, name, x, prequantized=None):
    """Projection ``name`` (``qkv``, ``out``, ``up`` = fused gate/up, ``down``) of an installed
    module (``dp4a_packing.py:109-125``): reads ``module._quant_<name>`` / ``_quant_<name>_scale``,
    the tile plan ``module._dp4a_packing[name]`` and ``module._dp4a_group``."""
    if getattr(module, "_short_scale_projection", None) == name or getattr(module, "_scaled_dp4a", None):
        raise ValueError("Short-scale and scaled DP4A layouts are W4A8-only; install the plain G32 export")
    cfg = (getattr(module, "_dp4a_packing", None) or {}).get(name, {})
    if cfg.get("activation_load", "standard") != "standard":
        raise ValueError("Direct activation loads are W4A8-only")
    return linear(x, getattr(module, "_quant_" + name), getattr(module, "_quant_" + name + "_scale"),
                  group=getattr(module, "_dp4a_group", 32), rows=cfg.get("rows", 1), warps=cfg.get("warps", 1),
                  interleaved=cfg.get("scheme") == "interleaved", paired=name == "up", prequantized=prequantized)


def install_packing(modules, plan_path):
    """Apply a ``dp4a_packing_v1`` plan to installed modules (``dp4a_packing.py:128-160``): same
    plan validation, scale narrowing checked for every projection before any layout changes.
    ``modules`` are the attention and MLP modules carrying ``_quant_*`` buffers."""
    plan = json.loads(Path(plan_path).read_text())
    if plan.get("format") != "dp4a_packing_v1" or plan.get("group") != 32 or plan.get("codebooks") != 32:
        raise ValueError("Unsupported packing plan")
    cfgs = plan["projections"]
    if set(cfgs) != {"qkv", "out", "up", "down"}:
        raise ValueError("Incomplete packing plan")
    for cfg in cfgs.values():
        if cfg["scheme"] not in ("prmt", "interleaved") or cfg["scale_dtype"] not in ("bfloat16", "float32") \
                or cfg["rows"] not in _TILES or cfg["warps"] not in _TILES:
            raise ValueError("Invalid packing configuration")
        if cfg.get("activation_load", "standard") not in ("standard", "direct"):
            raise ValueError("Invalid activation load mode")
        if cfg.get("activation_load") == "direct" and cfg["scheme"] != "interleaved":
            raise ValueError("Direct loads require interleaved weights")
    if any(getattr(m, "_dp4a_packing", None) for m in modules):
        raise ValueError("Weights are already repacked")
    targets = [(m, name) for m in modules for name in (("qkv", "out") if hasattr(m, "_quant_qkv") else ("up", "down"))]
    for m, name in targets:
        s = getattr(m, "_quant_" + name + "_scale")
        if cfgs[name]["scale_dtype"] == "bfloat16" and not torch.equal(s.float(), s.bfloat16().float()):
            raise ValueError("Requested BF16 scale storage would change values")
    for m, name in targets:
        cfg = cfgs[name]
        if cfg["scheme"] == "interleaved":
            setattr(m, "_quant_" + name, pack_interleaved(getattr(m, "_quant_" + name)))
        if cfg["scale_dtype"] == "bfloat16":
            setattr(m, "_quant_" + name + "_scale", getattr(m, "_quant_" + name + "_scale").bfloat16())
    for m in modules:
        names = ("qkv", "out") if hasattr(m, "_quant_qkv") else ("up", "down")
        m._dp4a_packing = {name: cfgs[name] for name in names}
    return plan
