"""One batch-1 decode step of the MOSS-TTS backbone (oracle, test infrastructure only).

Restates ``FastLLM.hidden`` with ``fused_residual=True`` (reference
``src/moss_tts/_runtime/llm.py:227-260``) and ``FastLLM._decode`` with
``greedy=True`` (``llm.py:268-287``) on the CPU with numpy, projections
dequantized once up front (``oracle.quant``), bf16 rounding as in ``oracle.ops``.

Weights are the plain dict layout produced by the product's synthetic
generator (``moss_tts._runtime.synthetic``) and accepted by its loader; bf16
tensors are uint16 bit arrays. Configuration is a plain dict with the keys of
``moss_tts._runtime.config.DecoderConfig``.
"""
import numpy as np

from . import ops, quant
from .numerics import to_f32


def dequantize_projection(p, group: int = 32) -> np.ndarray:
    """W4 dict ``{qweight, scales, qzeros}`` or bf16 dict ``{weight}`` -> fp32 values."""
    if "weight" in p:
        return to_f32(p["weight"])
    return quant.dequantize_w4(p["qweight"], p["scales"], p.get("qzeros"), group)


class Decoder:
    """Stateful CPU decoder holding a static KV cache of ``max_length`` rows."""

    def __init__(self, weights: dict, cfg: dict, max_length: int, layers=None, threads: int = 1):
        self.cfg = cfg
        self.max_length = max_length
        g = cfg["group_size"]
        chosen = weights["layers"] if layers is None else weights["layers"][:layers]
        names = ("qkv", "out", "gate_up", "down")
        jobs = [(i, n) for i in range(len(chosen)) for n in names]
        if threads > 1:  # numpy releases the GIL inside its array operations
            from concurrent.futures import ThreadPoolExecutor
            with ThreadPoolExecutor(threads) as ex:
                deq = dict(zip(jobs, ex.map(lambda j: dequantize_projection(chosen[j[0]][j[1]], g), jobs)))
        else:
            deq = {j: dequantize_projection(chosen[j[0]][j[1]], g) for j in jobs}
        self.layers = []
        for i, lw in enumerate(chosen):
            self.layers.append({
                "input_norm": to_f32(lw["input_norm"]), "post_norm": to_f32(lw["post_norm"]),
                "q_norm": to_f32(lw["q_norm"]), "k_norm": to_f32(lw["k_norm"]),
                **{n: deq[(i, n)] for n in names},
            })
        del deq
        n_kv, d = cfg["num_kv_heads"], cfg["head_dim"]
        self.k = np.zeros((len(self.layers), n_kv, max_length, d), dtype=np.float32)
        self.v = np.zeros_like(self.k)
        self.cos, self.sin = ops.rope_table(np.arange(max_length), d, cfg["rope_theta"])
        self.embed_text = weights["embed_text"]
        self.embed_audio = weights["embed_audio"]
        self.final_norm = to_f32(weights["final_norm"])
        self.text_ids = np.array([cfg["audio_assistant_gen_slot_token_id"],
                                  cfg["audio_assistant_delay_slot_token_id"]], dtype=np.int64)
        # FastLLM keeps the two audio-phase rows of the text head and the first
        # 1024 rows of each audio head (llm.py:188-191).
        self.text_head = to_f32(weights["head_text"][self.text_ids])
        self.full_text_head = weights["head_text"]  # bf16 bits [V, H], for prefill / full_step
        av = cfg["audio_vocab_size"]
        self.audio_heads = to_f32(weights["head_audio"][:, :av].reshape(-1, cfg["hidden_size"]))

    _linear = staticmethod(ops.linear)

    def reordered(self, chunks: int) -> "Decoder":
        """A decoder over the same weights (shared, not copied) with its own KV cache whose
        projections sum over K in ``chunks`` pieces (``ops.linear_reordered``): the same
        arithmetic up to fp32 summation order."""
        twin = Decoder.__new__(Decoder)
        twin.__dict__.update(self.__dict__)
        twin.k, twin.v = np.zeros_like(self.k), np.zeros_like(self.v)
        twin._linear = lambda x, w: ops.linear_reordered(x, w, chunks)
        return twin

    def hidden(self, ids, position: int) -> np.ndarray:
        """Final-norm hidden state for one token, ``llm.py:227-260``."""
        cfg = self.cfg
        eps = cfg["rms_norm_eps"]
        emb = ops.embedding_sum(np.asarray(ids).reshape(-1), self.embed_text, self.embed_audio)
        residual = emb
        hidden = ops.rmsnorm(emb, self.layers[0]["input_norm"], eps)
        for i, lw in enumerate(self.layers):
            linear = self._linear
            qkv = linear(hidden, lw["qkv"])
            q, k_row, v_row = ops.qk_rope(qkv, lw["q_norm"], lw["k_norm"], self.cos[position],
                                          self.sin[position], eps, cfg["num_heads"],
                                          cfg["num_kv_heads"], cfg["head_dim"])
            self.k[i, :, position] = k_row
            self.v[i, :, position] = v_row
            att = ops.attention_decode(q, self.k[i], self.v[i], position)
            att = linear(att, lw["out"])
            residual, hidden = ops.add_rmsnorm(att, residual, lw["post_norm"], eps)
            mlp = linear(ops.silu_mul(linear(hidden, lw["gate_up"])), lw["down"])
            norm = self.layers[i + 1]["input_norm"] if i + 1 < len(self.layers) else self.final_norm
            residual, hidden = ops.add_rmsnorm(mlp, residual, norm, eps)
        return hidden

    def step(self, ids, position: int, audio_length: int, delay_length: int):
        """``FastLLM.step`` semantics with greedy sampling.

        Returns ``(next_ids [1 + n_vq], text_logits [2], audio_logits [n_vq, 1024], hidden)``.
        """
        if not 0 <= position < self.max_length:
            raise ValueError("KV capacity exceeded")
        cfg = self.cfg
        h = self.hidden(ids, position)
        nxt, text, audio = ops.heads_greedy(
            h, self.text_head, self.audio_heads, self.text_ids, audio_length, delay_length,
            cfg["audio_assistant_delay_slot_token_id"], cfg["audio_end_token_id"], cfg["n_vq"],
            cfg["audio_vocab_size"], cfg["audio_pad_code"])
        return nxt, text, audio, h

    def prefill(self, ids):
        """``FastLLM.prefill`` (``llm.py:303-318``): the prompt ``ids [n, 1 + n_vq]`` at positions
        0..n-1, causal attention (row t attends rows 0..t), cache filled; the last row's
        final-norm hidden state gives the full text-head logits ``[V]`` and the audio logits
        ``[n_vq, 1024]`` (``llm.py:207``). Row by row, which is the causal pass's arithmetic."""
        ids = np.asarray(ids).reshape(-1, 1 + self.cfg["n_vq"])
        h = None
        for t in range(ids.shape[0]):
            h = self.hidden(ids[t], t)
        text = ops.linear(h, to_f32(self.full_text_head))
        audio = ops.linear(h, self.audio_heads).reshape(self.cfg["n_vq"], -1)
        return text, audio, h

    def fill_cache(self, k, v):
        """Install caller-provided cache rows (``[layers, n_kv, P, d]`` each)."""
        p = k.shape[2]
        self.k[:, :, :p] = to_f32(k)
        self.v[:, :, :p] = to_f32(v)
