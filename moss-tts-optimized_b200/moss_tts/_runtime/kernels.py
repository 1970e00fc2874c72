"""Decode operators with the reference's module-level signatures, on B200 CUDA kernels.

Mirrors ``src/moss_tts/_runtime/kernels.py`` of the reference: ``embedding_sum``,
``rmsnorm``, ``add_rmsnorm``, ``linear_decode``, ``silu_mul`` and
``qk_rope_decode`` keep their names, arguments and return values. All launches
go to PyTorch's current CUDA stream, outputs are allocated with ``torch.empty``
(as the reference does), and there is no CPU fallback: the C library must be
built and the tensors must live on a CUDA device.
"""
import torch

from . import native

_ATTN_SPLITS = 16


def _cuda(*tensors):
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("CUDA tensors required (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("All tensors must be on the same CUDA device")
        if not t.is_contiguous():
            raise ValueError("Contiguous tensors required")
    return dev


def _bf16(*tensors):
    for t in tensors:
        if t is not None and t.dtype != torch.bfloat16:
            raise ValueError("bf16 tensors required")


def embedding_sum(ids, text_weight, audio_weight):
    """Text embedding + 32 audio-codebook embeddings, bf16 rounding after each add.

    Same contract as the reference (``kernels.py:21-26``): ``ids`` int64
    ``[..., 1 + n_vq]``, ``text_weight`` ``[V, H]``, ``audio_weight`` ``[n_vq, V_a, H]``.
    """
    ids = ids.contiguous()
    _cuda(ids, text_weight, audio_weight)
    _bf16(text_weight, audio_weight)
    if ids.dtype != torch.long or ids.shape[-1] != audio_weight.shape[0] + 1:
        raise ValueError("ids must be int64 [..., 1 + n_vq]")
    h = text_weight.shape[-1]
    out = torch.empty((*ids.shape[:-1], h), device=ids.device, dtype=text_weight.dtype)
    tokens = ids.numel() // ids.shape[-1]
    native.call("mt_embedding_sum", ids.data_ptr(), text_weight.data_ptr(), audio_weight.data_ptr(),
                out.data_ptr(), tokens, h, text_weight.shape[0], audio_weight.shape[1],
                audio_weight.shape[0], None, 0, native.stream_of(ids))
    return out


def rmsnorm(x, weight, eps):
    """Qwen3 RMSNorm over the last dimension (``kernels.py:62-66``)."""
    x = x.contiguous()
    _cuda(x, weight)
    _bf16(x, weight)
    y = torch.empty_like(x)
    native.call("mt_rmsnorm", x.data_ptr(), None, weight.data_ptr(), None, y.data_ptr(),
                x.numel() // x.shape[-1], x.shape[-1], float(eps), 0, native.stream_of(x))
    return y


def add_rmsnorm(x, residual, weight, eps):
    """``(summed, normalized)`` with ``summed = bf16(x + residual)`` (``kernels.py:85-90``)."""
    x, residual = x.contiguous(), residual.contiguous()
    _cuda(x, residual, weight)
    _bf16(x, residual, weight)
    if x.shape != residual.shape:
        raise ValueError("x and residual shapes differ")
    summed, normalized = torch.empty_like(x), torch.empty_like(x)
    native.call("mt_rmsnorm", x.data_ptr(), residual.data_ptr(), weight.data_ptr(), summed.data_ptr(),
                normalized.data_ptr(), x.numel() // x.shape[-1], x.shape[-1], float(eps), 0,
                native.stream_of(x))
    return summed, normalized


def linear_decode(x, w):
    """bf16 GEMV for up to 8 rows (``kernels.py:102-108``); fp32 accumulation."""
    x = x.contiguous()
    _cuda(x, w)
    _bf16(x, w)
    n, k = w.shape
    rows = x.numel() // x.shape[-1]
    if x.shape[-1] != k or rows > 8:
        raise ValueError("linear_decode expects [..., K] with at most 8 rows")
    y = torch.empty((*x.shape[:-1], n), dtype=x.dtype, device=x.device)
    native.call("mt_bf16_linear", x.data_ptr(), None, None, 0.0, None, w.data_ptr(), y.data_ptr(),
                rows, n, k, 0, 0, native.stream_of(x))
    return y


def silu_mul(x):
    """``bf16(bf16(silu(gate)) * up)`` for ``x = gate || up`` (``kernels.py:132-139``)."""
    x = x.contiguous()
    _cuda(x)
    _bf16(x)
    n = x.shape[-1] // 2
    y = torch.empty((*x.shape[:-1], n), dtype=x.dtype, device=x.device)
    native.call("mt_silu_mul", x.data_ptr(), y.data_ptr(), x.numel() // x.shape[-1], n, 0,
                native.stream_of(x))
    return y


class AttentionScratch:
    """Per-device scratch for the split-K decode attention (partials, LSE, tickets)."""

    def __init__(self, device, batch, nq, nkv, splits):
        rep = nq // nkv
        self.splits = splits
        self.partial = torch.empty(batch * nkv * splits * rep * 128, device=device, dtype=torch.float32)
        self.lse = torch.empty(batch * nkv * splits * rep, device=device, dtype=torch.float32)
        self.tickets = torch.zeros(batch * nkv, device=device, dtype=torch.int32)


_scratch = {}


def qk_rope_decode(qkv, q_weight, k_weight, cos, sin, cache, layer_idx, position, eps, backend=None,
                   block=128, warps=4, context_capacity=None, quantize_output=False,
                   native_attention=False, pdl=None):
    """QK-norm + RoPE + KV-cache write + split-K decode attention for one token.

    Same call signature as the reference (``kernels.py:211-251``). ``cos``/``sin`` are the
    bf16 RoPE tables ``[max_len, 128]`` (rows selected on the device by ``position``);
    ``cache`` exposes ``cache.layers[layer_idx].keys/.values`` of shape ``[1, nkv, L, 128]``.
    Returns the attention output ``[1, 1, nq * 128]``. The reference's tile/warp/backend
    knobs select Triton variants and are validated but otherwise unused; int8 output
    quantization (``quantize_output``) belongs to the W4A8 path and is rejected.
    """
    if backend is not None or quantize_output or pdl:
        raise ValueError("Only the native fused B200 attention is available")
    kc, vc = cache.layers[layer_idx].keys, cache.layers[layer_idx].values
    _cuda(qkv, q_weight, k_weight, cos, sin, kc, vc, position)
    _bf16(qkv, q_weight, k_weight, cos, sin, kc, vc)
    if kc.ndim != 4 or kc.shape[0] != 1 or kc.shape[-1] != 128 or vc.shape != kc.shape:
        raise ValueError("KV cache must be [1, nkv, L, 128]")
    nkv, length = kc.shape[1], kc.shape[2]
    nq = qkv.shape[-1] // 128 - 2 * nkv
    if position.dtype != torch.long or position.numel() != 1:
        raise ValueError("position must be a one-element int64 CUDA tensor")
    if cos.shape != (length, 128) or sin.shape != cos.shape:
        raise ValueError("RoPE tables must be [L, 128]")
    capacity = length if context_capacity is None else context_capacity
    if not 0 < capacity <= length:
        raise ValueError("Invalid decode attention capacity")
    key = (qkv.device, nq, nkv)
    scratch = _scratch.get(key)
    if scratch is None:
        scratch = _scratch[key] = AttentionScratch(qkv.device, 1, nq, nkv, _ATTN_SPLITS)
    out = torch.empty((1, 1, nq * 128), device=qkv.device, dtype=qkv.dtype)
    native.call("mt_attention_decode", qkv.data_ptr(), q_weight.data_ptr(), k_weight.data_ptr(),
                cos.data_ptr(), sin.data_ptr(), position.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                out.data_ptr(), scratch.partial.data_ptr(), scratch.lse.data_ptr(),
                scratch.tickets.data_ptr(), 1, nq, nkv, length, scratch.splits, float(eps), None, 0,
                native.stream_of(qkv))
    return out
