"""``FastLLM``: the reference's batch-1 decode runtime object, on the B200 engine.

Mirrors ``src/moss_tts/_runtime/llm.py:148-337``: same constructor keywords and
validation, ``step(ids, position, audio_length, delay_length)`` returning the next
``[1, 1, 33]`` ids, ``prefill``, ``full_step``, ``warmup`` (graph capture) and the
``ids`` / ``position`` / ``audio_length`` / ``delay_length`` device buffers. The
reference's Triton/attention-tile knobs select kernels that do not exist here; they
are validated as the reference validates them and otherwise ignored.

``model`` is a ``DecoderWeights`` (device-resident, optionally a tensor-parallel
shard). Sampling: ``greedy=True`` selects argmax on the device inside the heads
kernel; otherwise the reference's top-k / top-p sampler (``llm.py:10-19``: text T 1.5,
top-k 2; audio T 1.7, top-k 25, top-p 0.8) runs as one kernel after it
(``mt_heads_sample``), delay masks included (``llm.py:280-286``), so a sampled step is a
graph of this library's kernels with no host round trip. Its draws come from a
counter-based generator keyed by ``engine.seed`` and the position, not torch's generator:
the distribution is the reference's, the individual draws are not.
"""
import torch
import torch.nn.functional as F

from . import native
from .engine import CONTROL_IDS, DecodeEngine, TensorParallel
from .weights import DecoderWeights


def sample_topk(logits, temperature=1.7, top_k=25, top_p=0.8):
    """Reference sampler (``llm.py:10-19``): temperature, top-k, top-p, multinomial."""
    if temperature <= 0:
        return logits.argmax(-1)
    values, indexes = torch.topk(logits.float() / temperature, min(top_k, logits.shape[-1]), dim=-1)
    probs = values.softmax(-1)
    remove = probs.cumsum(-1) - probs > top_p
    probs = probs.masked_fill(remove, 0)
    sampled = torch.multinomial(probs, 1)
    return indexes.gather(-1, sampled).squeeze(-1)


class FastLLM:
    def __init__(self, model: DecoderWeights, *, max_length=1024, fused=True, graph=True, greedy=False,
                 triton_attention=True, triton_gemv=True, attention_block=128, attention_warps=4,
                 fused_residual=False, fused_gateup=False, tp: TensorParallel | None = None,
                 splits: int | None = None, pdl: bool = True):
        if fused_residual and not fused:
            raise ValueError("Residual fusion requires the fused backbone")
        if fused_gateup and not fused:
            raise ValueError("Gate/up fusion requires a BF16 or 8-bit fused backbone")
        if max_length < 128 or max_length % 128:
            raise ValueError("max_length must be a positive multiple of 128")
        if attention_block not in (16, 32, 64, 128, 256) or max_length % attention_block or attention_warps not in (4, 8):
            raise ValueError("Unsupported attention tile or warp count")
        if not isinstance(model, DecoderWeights):
            raise TypeError("FastLLM takes DecoderWeights (see moss_tts._runtime.weights)")
        model.cfg.validate()
        self.model = model
        self.cfg = model.cfg
        self.max_length = max_length
        self.graph_enabled = graph
        self.greedy = greedy
        self.weight_quantization = "gptq_w4a16" if model.preset == "gptq" else "none"
        self.engine = DecodeEngine(model, max_length, splits=splits, pdl=pdl, tp=tp)
        e = self.engine
        self.ids = e.ids.view(1, 1, CONTROL_IDS)
        self.position, self.audio_length, self.delay_length = e.position, e.audio_length, e.delay_length
        self.channels = torch.arange(self.cfg.n_vq, device=e.device)
        self.graph = None
        self.prefill_graphs = {}
        self.prefill_mode = "auto"  # prefill.Prefill modes: "bf16", "dequant", "w4"

    # The sampler settings of FastLLM._decode (llm.py:280, 284): text (T, top-k, top-p), audio.
    SAMPLING = (1.5, 2, 1.0, 1.7, 25, 0.8)

    def _decode(self):
        self.engine.sampling = None if self.greedy else self.SAMPLING
        self.engine.launch_step()
        return (self.engine.next_ids.view(1, 1, CONTROL_IDS), self.engine.text_logits.view(1, 2),
                self.engine.audio_logits.view(-1, self.cfg.audio_vocab_size))

    @torch.inference_mode()
    def warmup(self):
        """Run the step eagerly, then capture it as one CUDA graph (``llm.py:289-301``)."""
        saved = self.engine.control.clone()
        for _ in range(3):
            self._decode()
        self.engine.control.copy_(saved)
        torch.cuda.synchronize(self.engine.device)
        if self.graph_enabled:
            stream = torch.cuda.Stream(self.engine.device)
            stream.wait_stream(torch.cuda.current_stream(self.engine.device))
            with torch.cuda.stream(stream):
                for _ in range(3):
                    self._decode()
                    self.engine.control.copy_(saved)
            torch.cuda.current_stream(self.engine.device).wait_stream(stream)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.next_ids, self.text_logits, self.audio_logits = self._decode()
            self.engine.control.copy_(saved)

    @torch.inference_mode()
    def step(self, ids, position, audio_length, delay_length):
        """One decode step; returns a device copy of the next ids ``[1, 1, 33]`` (``llm.py:327-337``)."""
        self.engine.set_inputs(ids, position, audio_length, delay_length)
        if self.graph is not None:
            self.graph.replay()
            return self.next_ids.clone()
        return self._decode()[0].clone()

    @torch.inference_mode()
    def step_host(self, ids, position, audio_length, delay_length):
        """``step`` with host input and a pinned host result (one copy each way)."""
        self.engine.set_inputs(ids, position, audio_length, delay_length)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._decode()
        return self.engine.read_next_ids()

    def health(self, clear: bool = True) -> dict:
        """Device-side failure flags of the decode steps so far (``DecodeEngine.health``)."""
        return self.engine.health(clear)

    def _full_text_logits(self):
        head = self.model.head_text
        if head is None:
            raise ValueError("The full text head was not loaded")
        out = torch.empty((1, head.shape[0]), device=head.device, dtype=torch.bfloat16)
        native.call("mt_bf16_linear", self.engine.hidden.data_ptr(), None, None, 0.0, None, head.data_ptr(),
                    out.data_ptr(), 1, head.shape[0], head.shape[1], 0, 0,
                    torch.cuda.current_stream(head.device).cuda_stream)
        return out

    @torch.inference_mode()
    def full_step(self, ids, position):
        """Decode one text-phase token and return the full text-head logits (``llm.py:320-325``)."""
        self.engine.set_inputs(ids, position, 1, -1)
        self.engine.launch_step()
        return self._full_text_logits()

    @torch.inference_mode()
    def prefill(self, ids):
        """Run a ``[1, n, 33]`` prompt as one batched causal pass at positions 0..n-1 (filling
        the KV cache) and return the last row's ``(text logits [1, V], audio logits [32, 1024])``
        (``llm.py:303-318``). W4A16 weights on one GPU run the batched prefill kernels
        (``prefill.Prefill``); otherwise the prompt goes through the decode step row by row."""
        ids = torch.as_tensor(ids)
        if ids.dim() != 3 or ids.shape[0] != 1 or ids.shape[1] >= self.max_length:
            raise ValueError("Batch must be one and prompt must fit the KV capacity")
        e = self.engine
        batched = e.tp.world == 1 and self.model.head_text is not None and all(
            p.quantized for lw in self.model.layers for p in (lw.qkv, lw.out, lw.gate_up, lw.down))
        if batched:
            from .prefill import Prefill
            n = ids.shape[1]
            runner = self.prefill_graphs.get("runner")
            if runner is None or runner.max_tokens < n or runner.mode != self.prefill_mode:
                runner = self.prefill_graphs["runner"] = Prefill(e, max_tokens=max(512, n), mode=self.prefill_mode)
            return runner.run(ids.to(e.device))
        for t in range(ids.shape[1]):
            e.set_inputs(ids[0, t], t, 1, -1)
            e.launch_step()
        return self._full_text_logits(), e.audio_logits.view(-1, self.cfg.audio_vocab_size)
