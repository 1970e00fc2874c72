"""Decode-step operators of the MOSS-TTS backbone (oracle, test infrastructure only).

Each function restates one reference kernel on the CPU with numpy, keeping the
reference's bf16 rounding points. bf16 tensors are float32 arrays holding
bf16-exact values (see ``numerics``). File:line citations are into the
reference's ``src/moss_tts``.
"""
import numpy as np

from .numerics import round_bf16, to_f32

ATTENTION_SCALE = np.float32(0.08838834764831845)  # 1/sqrt(128), _runtime/kernels.py:183


def linear(x, w) -> np.ndarray:
    """bf16 ``x @ w.T`` with fp32 accumulation and one bf16 rounding of the output.

    The reference scores its G32 export with ``F.linear`` on dequantized weights
    (``calibration.py:185-189``); decode projections (``_runtime/kernels.py:93-108``)
    accumulate in fp32 and store bf16.
    """
    x = to_f32(x)
    w = to_f32(w)
    return round_bf16(np.matmul(x, w.T))


def linear_reordered(x, w, chunks: int) -> np.ndarray:
    """``linear`` with the fp32 sum over K taken in ``chunks`` consecutive pieces, each summed
    on its own and then added in order -- the same value up to fp32 summation order. Tests use
    it to measure how far the reference's own arithmetic moves under a different order."""
    x, w = to_f32(x), to_f32(w)
    k = w.shape[1]
    acc = np.zeros(x.shape[:-1] + (w.shape[0],), dtype=np.float32)
    for c in range(chunks):
        a, b = c * k // chunks, (c + 1) * k // chunks
        acc += np.matmul(x[..., a:b], w[:, a:b].T)
    return round_bf16(acc)


def rmsnorm(x, weight, eps: float) -> np.ndarray:
    """Qwen3 RMSNorm, ``_runtime/kernels.py:50-59``: the normalized value is
    rounded to bf16 before the weight multiply, and the product is rounded again."""
    x = to_f32(x)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    inv = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    z = round_bf16(x * inv)
    return round_bf16(z * to_f32(weight))


def add_rmsnorm(x, residual, weight, eps: float):
    """``_runtime/kernels.py:69-90``: ``summed = bf16(x + residual)`` then RMSNorm.

    Returns ``(summed, normalized)`` like the reference's ``add_rmsnorm``.
    """
    summed = round_bf16(to_f32(x) + to_f32(residual))
    return summed, rmsnorm(summed, weight, eps)


def silu_mul(gate_up) -> np.ndarray:
    """``_runtime/kernels.py:123-139``: ``bf16(bf16(g / (1 + exp(-g))) * u)`` where
    the input is the bf16 ``[..., 2I]`` concatenation ``gate || up``."""
    gu = to_f32(gate_up)
    i = gu.shape[-1] // 2
    g, u = gu[..., :i], gu[..., i:]
    with np.errstate(over="ignore"):
        s = round_bf16(g / (np.float32(1.0) + np.exp(-g)))
    return round_bf16(s * u)


def embedding_sum(ids, text_weight, audio_weight) -> np.ndarray:
    """``_runtime/kernels.py:7-26``: text embedding plus the 32 audio-codebook
    embeddings, rounding to bf16 after every sequential addition.

    ``ids`` is ``[..., 1 + n_vq]``; ``audio_weight`` is ``[n_vq, V_audio, H]``.
    """
    ids = np.asarray(ids, dtype=np.int64)
    flat = ids.reshape(-1, ids.shape[-1])
    out = np.empty((flat.shape[0], text_weight.shape[-1]), dtype=np.float32)
    for t, row in enumerate(flat):
        x = to_f32(text_weight[row[0]])
        for q in range(flat.shape[1] - 1):
            x = round_bf16(x + to_f32(audio_weight[q, row[q + 1]]))
        out[t] = x
    return out.reshape(*ids.shape[:-1], -1)


def rope_inv_freq(head_dim: int = 128, theta: float = 1e6) -> np.ndarray:
    """Default RoPE inverse frequencies as the HF ``Qwen3RotaryEmbedding`` builds them
    (fp32 exponent ``arange(0, d, 2) / d``, fp32 power and reciprocal)."""
    exps = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    base = np.float32(theta).astype(np.float64) ** exps.astype(np.float64)
    return (np.float32(1.0) / base.astype(np.float32)).astype(np.float32)


def rope_table(positions, head_dim: int = 128, theta: float = 1e6):
    """bf16 ``(cos, sin)`` tables ``[P, head_dim]``; the reference evaluates the
    transformers rotary embedding per step (``_runtime/llm.py:231``): fp32
    ``freqs = inv_freq * position``, ``emb = cat(freqs, freqs)``, cos/sin in fp32,
    cast to bf16."""
    inv = rope_inv_freq(head_dim, theta)
    pos = np.asarray(positions, dtype=np.float32).reshape(-1, 1)
    freqs = (pos * inv[None, :]).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1).astype(np.float64)
    cos = round_bf16(np.cos(emb).astype(np.float32))
    sin = round_bf16(np.sin(emb).astype(np.float32))
    return cos, sin


def _head_norm_rope(x, w, cos, sin, eps):
    """One head of ``_runtime/kernels.py:142-170``: head RMSNorm (bf16 rounding of
    the normalized value and of the weighted value), then rotate-half RoPE with
    each product rounded to bf16 and the sum rounded on store."""
    d = x.shape[-1]
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    inv = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    y = round_bf16(round_bf16(x * inv) * w)
    rot = np.concatenate([-y[..., d // 2:], y[..., :d // 2]], axis=-1)
    return round_bf16(round_bf16(y * cos) + round_bf16(rot * sin))


def qk_rope(qkv, q_weight, k_weight, cos, sin, eps: float, n_q: int = 32, n_kv: int = 8,
            head_dim: int = 128):
    """Fused QK-norm + RoPE + cache-row preparation, ``_runtime/kernels.py:142-170``.

    ``qkv`` is the bf16 projection ``[(n_q + 2 n_kv) * d]`` laid out q | k | v;
    ``cos``/``sin`` are the bf16 table rows for this position. Returns
    ``(q [n_q, d], k_row [n_kv, d], v_row [n_kv, d])`` as written by the kernel.
    """
    x = to_f32(qkv)
    d = head_dim
    q = x[: n_q * d].reshape(n_q, d)
    k = x[n_q * d:(n_q + n_kv) * d].reshape(n_kv, d)
    v = x[(n_q + n_kv) * d:(n_q + 2 * n_kv) * d].reshape(n_kv, d)
    c, s = to_f32(cos), to_f32(sin)
    qw, kw = to_f32(q_weight), to_f32(k_weight)
    return _head_norm_rope(q, qw, c, s, eps), _head_norm_rope(k, kw, c, s, eps), v.copy()


def attention_decode(q, k_cache, v_cache, position: int) -> np.ndarray:
    """GQA decode attention over cache rows ``0..position`` with fp32 softmax.

    Restates the split-K kernel pair ``_runtime/kernels.py:173-208`` (and
    ``_runtime/attention_native.cu:31-89``): per split a normalized partial and
    its log-sum-exp, merged with softmax weights; mathematically the full fp32
    softmax computed here. Query head ``h`` reads KV head ``h // (n_q / n_kv)``.
    Output: bf16 ``[n_q * d]``.
    """
    q = to_f32(q)
    n_q, d = q.shape
    n_kv = k_cache.shape[0]
    rep = n_q // n_kv
    out = np.empty((n_q, d), dtype=np.float32)
    for h in range(n_q):
        kh = to_f32(k_cache[h // rep, : position + 1])
        vh = to_f32(v_cache[h // rep, : position + 1])
        logits = (kh @ q[h]).astype(np.float32) * ATTENTION_SCALE
        m = logits.max()
        p = np.exp(logits - m).astype(np.float32)
        out[h] = (p @ vh) / p.sum(dtype=np.float32)
    return round_bf16(out.reshape(-1))


def argmax_first(x, axis=-1):
    """``torch.argmax`` tie rule: the first maximal index."""
    return np.argmax(np.asarray(x), axis=axis)


def heads_greedy(h, text_head, audio_heads, text_ids, audio_length: int, delay_length: int,
                 delay_slot_id: int, audio_end_id: int, n_vq: int = 32, audio_vocab: int = 1024,
                 pad_code: int = 1024):
    """Output heads, greedy selection and delay-pattern masks, ``_runtime/llm.py:268-287``
    with ``greedy=True`` (``sample_topk`` with temperature 0 is ``argmax``, ``llm.py:11-12``).

    Returns ``(next_ids [1 + n_vq] int64, text_logits [2], audio_logits [n_vq, V])``.
    """
    text = linear(h, text_head)
    audio = linear(h, audio_heads).reshape(n_vq, audio_vocab)
    text_token = int(text_ids[int(argmax_first(text))])
    if delay_length >= 0:
        text_token = delay_slot_id
    if delay_length == 32:
        text_token = audio_end_id
    tokens = argmax_first(audio, axis=-1).astype(np.int64)
    ch = np.arange(n_vq)
    valid = (ch < audio_length) & ((delay_length < 0) | (ch >= delay_length))
    tokens = np.where(valid, tokens, pad_code)
    return np.concatenate([[text_token], tokens]).astype(np.int64), text, audio
