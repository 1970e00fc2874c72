"""The 32 decode steps after ``audio_start`` as one CUDA graph (the reference's
``first_audio_graph.FirstAudioGraph``, ``src/moss_tts/_runtime/first_audio_graph.py:30-93``).

The delay schedule cannot emit ``audio_end`` in the 32 steps after ``audio_start``, so they
can run with no host decision in between. One replay runs 32 times: the full decode step of
``FastLLM`` (this library's kernels; greedy ids from the heads kernel or the device sampler),
then ``mt_decode_advance`` (next ids fed back, position and audio length + 1, delay
bookkeeping as the reference's ``_advance``, ``first_audio_graph.py:14-27``) and a copy of the
step's ids into ``history[step]``. ``status`` holds ``(text id, audio length, delay length,
position)`` after the last step.

``head_prefixes`` is accepted for the reference's signature: the reference computes only the
first ``8 (step // 8 + 1)`` codebook heads in these steps, the rest being masked to the pad
code by the delay pattern; here every step computes all heads (the outputs are the same).
``capacity`` bounds the positions a replay may reach (``position + 32 <= capacity``).
"""
import time

import torch

from .engine import CONTROL_IDS


class FirstAudioGraph:
    def __init__(self, llm, capacity, *, head_prefixes=True, save_logits=False):
        if llm.graph is None or capacity % 32 or not 32 <= capacity <= llm.max_length:
            raise ValueError("A warmed LLM and valid context capacity are required")
        self.llm, self.capacity = llm, capacity
        self.head_prefixes, self.save_logits = head_prefixes, save_logits
        e = llm.engine
        dev = e.device
        self.history = torch.empty((32, CONTROL_IDS), device=dev, dtype=torch.long)
        self.status = torch.empty(4, device=dev, dtype=torch.long)
        self.text_history = torch.empty((32, 2), device=dev, dtype=torch.bfloat16) if save_logits else None
        self.audio_history = (torch.empty((32, llm.cfg.n_vq, llm.cfg.audio_vocab_size), device=dev,
                                          dtype=torch.bfloat16) if save_logits else None)
        self.graph = None
        self.metadata = {}

    def _body(self):
        llm, e = self.llm, self.llm.engine
        for step in range(32):
            _, text, audio = llm._decode()
            if self.save_logits:
                self.text_history[step].copy_(text.flatten())
                self.audio_history[step].copy_(audio.view_as(self.audio_history[step]))
            self.history[step].copy_(e.next_ids)
            e.launch_advance()
        # (text id, audio length, delay length, position) as the reference's _advance leaves them
        self.status[0:1].copy_(e.ids[0:1])
        self.status[1:2].copy_(e.audio_length)
        self.status[2:3].copy_(e.delay_length)
        self.status[3:4].copy_(e.position)

    def _initialize(self, ids, position, delay=-1):
        e = self.llm.engine
        e.ids.copy_(ids.reshape(-1))
        e.position.fill_(position)
        e.audio_length.fill_(1)
        e.delay_length.fill_(delay)

    @torch.inference_mode()
    def warmup(self):
        if self.graph is not None:
            raise RuntimeError("First-audio graph already captured")
        llm, e = self.llm, self.llm.engine
        saved = e.control.clone()
        first = torch.full((CONTROL_IDS,), llm.cfg.audio_pad_code, device=e.device, dtype=torch.long)
        first[0] = llm.cfg.audio_start_token_id
        torch.cuda.synchronize(e.device)
        before, reserved, start = torch.cuda.memory_allocated(), torch.cuda.memory_reserved(), time.perf_counter()
        try:
            stream = torch.cuda.Stream(e.device)
            stream.wait_stream(torch.cuda.current_stream(e.device))
            with torch.cuda.stream(stream):
                self._initialize(first, 0)
                self._body()
            torch.cuda.current_stream(e.device).wait_stream(stream)
            self._initialize(first, 0)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._body()
            torch.cuda.synchronize(e.device)
            self.metadata = {"capacity": self.capacity, "steps": 32, "codebooks": llm.cfg.n_vq,
                             "head_prefixes": self.head_prefixes, "save_logits": self.save_logits,
                             "capture_seconds": time.perf_counter() - start,
                             "additional_live_bytes": torch.cuda.memory_allocated() - before,
                             "additional_reserved_bytes": torch.cuda.memory_reserved() - reserved}
        finally:
            e.control.copy_(saved)

    @torch.inference_mode()
    def run(self, ids, position, *, delay=-1):
        """Replay the 32 steps from ``ids`` (CUDA int64 ``[1, 1, 33]``, the audio-start row) at
        ``position``; returns ``(history [32, 33], status [4])`` device tensors."""
        if self.graph is None:
            raise RuntimeError("Warm the first-audio graph before use")
        if not 0 <= position or position + 32 > self.capacity:
            raise ValueError("Initial interval exceeds captured context capacity")
        e = self.llm.engine
        if tuple(ids.shape) != (1, 1, CONTROL_IDS) or ids.dtype != torch.long or ids.device != e.device:
            raise ValueError("Expected a CUDA int64 audio-start row with all 32 channels")
        if delay not in (-1, 0):
            raise ValueError("Only fresh audio or an immediate-delay validation probe is supported")
        self._initialize(ids, position, delay)
        self.graph.replay()
        return self.history, self.status
