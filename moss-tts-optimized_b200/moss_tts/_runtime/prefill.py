"""Batched causal prompt prefill on the decode engine's weights and KV cache.

The reference runs a prompt as one batched backbone pass and returns the last row's logits
(``FastLLM.prefill`` / ``_prefill_forward``, ``src/moss_tts/_runtime/llm.py:204-226, 303-318``):
embedding sum of the ``[n, 33]`` ids, 36 layers over all n rows at positions 0..n-1 with causal
attention, the cache filled for the decode steps that follow, then ``(text logits [1, V] over
the full text head, audio logits [32, 1024])`` of the last row. Here every launch is this
library's CUDA:

    mt_embedding_sum (n rows)
    per layer: mt_rmsnorm (+ residual add) -> W4A16 q|k|v GEMM (tcgen05, 128-row tiles)
               -> mt_prefill_qk_rope_kv (head norm, RoPE, cache rows 0..n-1)
               -> mt_prefill_attention (causal GQA) -> o_proj GEMM -> add + RMSNorm
               -> gate/up GEMM with SiLU*up -> down GEMM
    last row: add + final RMSNorm (mt_rmsnorm) -> full text head and audio heads (bf16 GEMVs)

Projections, three modes:

* ``"bf16"``: bf16 copies of the projection weights, made once by the bit-exact
  ``mt_dequant_w4`` on first use and kept resident, multiplied with a plain bf16 GEMM (cuBLAS
  through ``torch.matmul``, fp32 accumulation); the gate/up product goes through
  ``mt_silu_mul``. This is the reference's own arrangement: its G32 preset keeps BF16 weights
  for the prompt pass (``calibrated_quant.py`` header, ``llm.py:204-226``). 2 bytes per weight
  (13.9 GB for the 8B backbone).
* ``"dequant"``: the same GEMMs, each projection dequantized into one reused bf16 scratch
  matrix (201 MB) right before its GEMM.
* ``"w4"``: the W4A16 tcgen05 GEMM on the GPTQ layout (``mt_w4a16_gemm``), one call per
  128-row tile of the prompt, with the paired SiLU epilogue (no extra memory).

``"auto"`` picks ``"bf16"`` when the device has room for the copies (with 8 GB to spare),
else ``"dequant"``.
"""
import torch

from . import native

GEMM_ROWS = 128


class Prefill:
    """Prompt buffers for up to ``max_tokens`` rows over a (single-GPU, W4A16) ``DecodeEngine``."""

    def __init__(self, engine, max_tokens: int = 512, mode: str = "auto"):
        if mode not in ("auto", "bf16", "dequant", "w4"):
            raise ValueError("mode must be 'auto', 'bf16', 'dequant' or 'w4'")
        eng = engine
        if mode == "auto":
            need = 2 * sum(p.n * p.k for lw in eng.w.layers for p in (lw.qkv, lw.out, lw.gate_up, lw.down))
            free, _ = torch.cuda.mem_get_info(eng.device)
            mode = "bf16" if free > need + (8 << 30) else "dequant"
        self.mode = mode
        self.resident = {}  # id(projection) -> bf16 weights ("bf16" mode)
        if eng.tp.world != 1:
            raise ValueError("prefill runs on one GPU")
        w, cfg = eng.w, eng.cfg
        if not all(p.quantized for lw in w.layers for p in (lw.qkv, lw.out, lw.gate_up, lw.down)):
            raise ValueError("prefill runs the W4A16 projections")
        if w.head_text is None:
            raise ValueError("prefill returns the full text-head logits: load the full text head")
        self.eng, self.cfg, self.max_tokens = eng, cfg, max_tokens
        dev, T, h = eng.device, max_tokens, cfg.hidden_size
        bf = dict(device=dev, dtype=torch.bfloat16)
        self.ids = torch.zeros(T, 1 + cfg.n_vq, device=dev, dtype=torch.long)
        self.x = torch.zeros(T, h, **bf)
        self.res = [torch.zeros(T, h, **bf), torch.zeros(T, h, **bf)]  # residual stream, ping-pong
        self.normed = torch.zeros(T, h, **bf)
        self.qkv = torch.zeros(T, cfg.qkv_size, **bf)
        self.q = torch.zeros(T, cfg.num_heads, cfg.head_dim, **bf)
        self.attn = torch.zeros(T, cfg.num_heads * cfg.head_dim, **bf)
        self.mid = torch.zeros(T, cfg.intermediate_size, **bf)
        self.hidden = torch.zeros(h, **bf)
        self.text_logits = torch.zeros(1, w.head_text.shape[0], **bf)
        self.audio_logits = torch.zeros(cfg.n_vq, cfg.audio_vocab_size, **bf)
        if mode in ("bf16", "dequant"):
            if mode == "dequant":
                largest = max(p.n * p.k for lw in w.layers for p in (lw.qkv, lw.out, lw.gate_up, lw.down))
                self.wscratch = torch.empty(largest, **bf)
            self.gu = torch.zeros(T, w.layers[0].gate_up.n, **bf)
        ws = 256
        for lw in w.layers:
            for p, paired in ((lw.qkv, False), (lw.out, False), (lw.gate_up, True), (lw.down, False)):
                ws = max(ws, native.w4a16_gemm_workspace(GEMM_ROWS, p.n, p.k, native.LINEAR_PAIRED if paired else 0))
        self.workspace = torch.zeros(ws, device=dev, dtype=torch.uint8)
        # one CUDA graph per prompt length (the launches depend on n), captured after the first
        # eager pass of that length (as the reference captures its prefill buckets, llm.py:204-226)
        self.graphs = {}
        self.max_graphs = 8

    def _gemm(self, p, x, y, n, paired=False):
        s = torch.cuda.current_stream(self.eng.device).cuda_stream
        if self.mode in ("bf16", "dequant"):
            w = self.resident.get(id(p)) if self.mode == "bf16" else None
            if w is None:
                w = (torch.empty((p.n, p.k), device=y.device, dtype=torch.bfloat16) if self.mode == "bf16"
                     else self.wscratch[: p.n * p.k].view(p.n, p.k))
                native.call("mt_dequant_w4", p.qweight.data_ptr(), p.scales.data_ptr(), native.ptr(p.qzeros),
                            w.data_ptr(), p.n, p.k, 32, s)
                if self.mode == "bf16":
                    self.resident[id(p)] = w
            if paired:
                torch.matmul(x[:n], w.t(), out=self.gu[:n])
                native.call("mt_silu_mul", self.gu.data_ptr(), y.data_ptr(), n, p.n // 2, 0, s)
            else:
                torch.matmul(x[:n], w.t(), out=y[:n])
            return
        mode = native.LINEAR_PAIRED if paired else 0
        for r0 in range(0, n, GEMM_ROWS):
            rows = min(GEMM_ROWS, n - r0)
            native.call("mt_w4a16_gemm", x[r0].data_ptr(), p.qweight.data_ptr(), p.scales.data_ptr(),
                        native.ptr(p.qzeros), y[r0].data_ptr(), rows, p.n, p.k, mode, self.workspace.data_ptr(), 0, s)

    def run(self, ids) -> tuple[torch.Tensor, torch.Tensor]:
        """Prefill ``ids`` ``[1, n, 33]`` (host or device int64) at positions 0..n-1; returns the
        last row's ``(text logits [1, V], audio logits [32, 1024])`` (device tensors)."""
        eng, cfg, w = self.eng, self.cfg, self.eng.w
        ids = torch.as_tensor(ids)
        if ids.dim() != 3 or ids.shape[0] != 1 or ids.shape[2] != 1 + cfg.n_vq:
            raise ValueError("ids must be [1, n, 1 + n_vq]")
        n = ids.shape[1]
        if not 1 <= n <= self.max_tokens or n >= eng.max_length:
            raise ValueError("Batch must be one and prompt must fit the KV capacity")
        self.ids[:n].copy_(ids[0])
        g = self.graphs.get(n)
        if g is not None:
            g.replay()
            return self.text_logits, self.audio_logits
        if self.mode == "w4" or len(self.graphs) >= self.max_graphs:
            self._launch(n)
            return self.text_logits, self.audio_logits
        # an eager pass on a side stream (it makes the bf16 copies and the GEMM library's state on
        # that stream, and gives this call's result), then the same launches captured there
        cur = torch.cuda.current_stream(eng.device)
        stream = torch.cuda.Stream(eng.device)
        stream.wait_stream(cur)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            self._launch(n)
            with torch.cuda.graph(graph, stream=stream):
                self._launch(n)
        cur.wait_stream(stream)
        self.graphs[n] = graph
        return self.text_logits, self.audio_logits

    def _launch(self, n: int) -> None:
        """Enqueue the prompt pass over ``self.ids[:n]`` on the current stream."""
        eng, cfg, w = self.eng, self.cfg, self.eng.w
        s = torch.cuda.current_stream(eng.device).cuda_stream
        eps = float(cfg.rms_norm_eps)
        h, d = cfg.hidden_size, cfg.head_dim
        native.call("mt_embedding_sum", self.ids.data_ptr(), w.embed_text.data_ptr(), w.embed_audio.data_ptr(),
                    self.x.data_ptr(), n, h, w.embed_text.shape[0], w.embed_audio.shape[1], cfg.n_vq,
                    eng.status.data_ptr(), 0, s)
        # x holds the sublayer output to add; the residual stream alternates between two buffers
        cur = 0
        for i, lw in enumerate(w.layers):
            if i == 0:
                self.res[cur][:n].copy_(self.x[:n])
                native.call("mt_rmsnorm", self.x.data_ptr(), None, lw.input_norm.data_ptr(), None, self.normed.data_ptr(),
                            n, h, eps, 0, s)
            else:
                native.call("mt_rmsnorm", self.x.data_ptr(), self.res[cur].data_ptr(), lw.input_norm.data_ptr(),
                            self.res[1 - cur].data_ptr(), self.normed.data_ptr(), n, h, eps, 0, s)
                cur = 1 - cur
            self._gemm(lw.qkv, self.normed, self.qkv, n)
            k, v = eng.kv[i, 0], eng.kv[i, 1]
            native.call("mt_prefill_qk_rope_kv", self.qkv.data_ptr(), lw.q_norm.data_ptr(), lw.k_norm.data_ptr(),
                        eng.cos.data_ptr(), eng.sin.data_ptr(), 0, self.q.data_ptr(), k.data_ptr(), v.data_ptr(), n,
                        cfg.num_heads, cfg.num_kv_heads, eng.max_length, eps, 0, s)
            native.call("mt_prefill_attention", self.q.data_ptr(), k.data_ptr(), v.data_ptr(), self.attn.data_ptr(), 0,
                        n, cfg.num_heads, cfg.num_kv_heads, eng.max_length, 0, s)
            self._gemm(lw.out, self.attn, self.x, n)
            native.call("mt_rmsnorm", self.x.data_ptr(), self.res[cur].data_ptr(), lw.post_norm.data_ptr(),
                        self.res[1 - cur].data_ptr(), self.normed.data_ptr(), n, h, eps, 0, s)
            cur = 1 - cur
            self._gemm(lw.gate_up, self.normed, self.mid, n, paired=True)
            self._gemm(lw.down, self.mid, self.x, n)
        last = n - 1
        native.call("mt_rmsnorm", self.x[last].data_ptr(), self.res[cur][last].data_ptr(), w.final_norm.data_ptr(),
                    self.res[1 - cur][last].data_ptr(), self.hidden.data_ptr(), 1, h, eps, 0, s)
        native.call("mt_bf16_linear", self.hidden.data_ptr(), None, None, 0.0, None, w.head_text.data_ptr(),
                    self.text_logits.data_ptr(), 1, w.head_text.shape[0], h, 0, 0, s)
        native.call("mt_bf16_linear", self.hidden.data_ptr(), None, None, 0.0, None, w.head_audio.data_ptr(),
                    self.audio_logits.data_ptr(), 1, w.head_audio.shape[0], h, 0, 0, s)
