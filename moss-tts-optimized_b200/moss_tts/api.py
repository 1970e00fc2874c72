"""Public API: ``MossTTS.from_pretrained(preset="gptq"|"bf16")`` backed by the B200 decode engine.

Mirrors ``src/moss_tts/api.py`` of the reference: keyword arguments, validation before
anything is loaded (``ValueError``), ``RuntimeError`` without a CUDA device, a single
active request per model, ``metrics``, ``close`` and context-manager use. Differences:

* the SM90/Triton gate becomes an sm_100 gate (the kernels are built for sm_100a only);
* the gptq preset accepts any ``max_length`` multiple of 128 (the reference pins 1024);
* checkpoints are read from the local Hugging Face cache (``cache_dir``); there is no
  network download; ``from_random`` builds a random-init model of the same shapes;
* the audio codec, text processor and voice encoder are not part of this package (they
  are outside the decode hot path): ``stream``/``clone_voice`` run only when the engine
  object passed to the constructor provides them, as the reference's tests do.
"""
import threading
import time
from contextlib import contextmanager
from pathlib import Path
from typing import Literal

from .types import AudioChunk, Voice  # noqa: F401


class MossTTS:
    sample_rate = 48000
    codebooks = 32

    def __init__(self, engine, encoder=None, *, device, preset: str):
        self._engine = engine
        self._encoder = encoder
        self.device = device
        self.preset = preset
        self._lock = threading.Lock()
        self._closed = False
        self._last_metrics = {}

    @staticmethod
    def _validate(preset, calibration_path, max_length, cpu_threads):
        if preset not in ("bf16", "gptq"):
            raise ValueError("preset must be 'bf16' or 'gptq'")
        if (preset == "gptq") != (calibration_path is not None):
            raise ValueError("Provide calibration_path exactly when preset='gptq'")
        if not isinstance(max_length, int) or max_length < 128 or max_length % 128:
            raise ValueError("max_length must be a positive multiple of 128")
        if not isinstance(cpu_threads, int) or cpu_threads < 1:
            raise ValueError("cpu_threads must be positive")
        if preset == "gptq":
            folder = Path(calibration_path)
            if not (folder / "config.json").is_file():
                raise ValueError("calibration_path must be a calibrated G32 export directory")
            from ._runtime.calibrated_backend import validate_export
            validate_export(folder)

    @staticmethod
    def _device(device):
        import torch
        target = torch.device(device)
        if target.type != "cuda" or not torch.cuda.is_available():
            raise RuntimeError("MOSS-TTS 8B streaming requires an NVIDIA CUDA device")
        if target.index is None:
            target = torch.device("cuda", torch.cuda.current_device())
        if torch.cuda.get_device_capability(target) != (10, 0):
            raise ValueError("The B200 kernels are built for sm_100a (Blackwell B200) only")
        return target

    @classmethod
    def from_pretrained(cls, *, preset: Literal["bf16", "gptq"] = "bf16", calibration_path=None,
                        device: str = "cuda:0", cache_dir=None, local_files_only: bool = False,
                        max_length: int = 1024, cpu_threads: int = 4) -> "MossTTS":
        """Load the pinned 8B checkpoint from the local cache and capture the decode graph."""
        cls._validate(preset, calibration_path, max_length, cpu_threads)
        import torch
        target = cls._device(device)
        from ._runtime.checkpoint import config_from_json, find_snapshot, load_checkpoint
        from ._runtime.llm import FastLLM
        torch.set_num_threads(cpu_threads)
        folder = find_snapshot(cache_dir)
        cfg = config_from_json(folder / "config.json")
        calibrated = None
        if preset == "gptq":
            from ._runtime.calibrated_backend import load_export
            shapes = {"qkv": [cfg.qkv_size, cfg.hidden_size], "out": [cfg.hidden_size, cfg.hidden_size],
                      "up": [2 * cfg.intermediate_size, cfg.hidden_size],
                      "down": [cfg.hidden_size, cfg.intermediate_size]}
            calibrated = load_export(calibration_path, shapes, cfg.num_layers)
        with torch.cuda.device(target), torch.inference_mode():
            weights = load_checkpoint(folder, target, calibrated, cfg)
            llm = FastLLM(weights, max_length=max_length, fused_residual=True, fused_gateup=preset == "bf16")
            llm.warmup()
        return cls(llm, None, device=target, preset=preset)

    @classmethod
    def from_random(cls, *, preset: Literal["bf16", "gptq"] = "gptq", device: str = "cuda:0",
                    max_length: int = 1024, seed: int = 0, layers: int | None = None,
                    greedy: bool = True) -> "MossTTS":
        """Random-init model of the pinned shapes (no checkpoint), decode graph captured."""
        if preset not in ("bf16", "gptq"):
            raise ValueError("preset must be 'bf16' or 'gptq'")
        if not isinstance(max_length, int) or max_length < 128 or max_length % 128:
            raise ValueError("max_length must be a positive multiple of 128")
        import torch
        target = cls._device(device)
        from ._runtime.config import DecoderConfig
        from ._runtime.llm import FastLLM
        from ._runtime.weights import DecoderWeights
        cfg = DecoderConfig() if layers is None else DecoderConfig().with_(num_layers=layers)
        with torch.cuda.device(target), torch.inference_mode():
            weights = DecoderWeights.random(cfg, target, seed, preset)
            llm = FastLLM(weights, max_length=max_length, greedy=greedy, fused_residual=True)
            llm.warmup()
        return cls(llm, None, device=target, preset=preset)

    @property
    def llm(self):
        """The decode runtime (``FastLLM``) behind this model."""
        return self._engine

    @contextmanager
    def _request(self):
        if not self._lock.acquire(blocking=False):
            raise RuntimeError("This model is busy; finish or close the active stream first")
        try:
            if self._closed:
                raise RuntimeError("This model is closed")
            yield
        finally:
            self._lock.release()

    def clone_voice(self, audio_path):
        if self._encoder is None:
            raise NotImplementedError("Voice encoding (the audio codec) is not part of the B200 decode package")
        with self._request():
            return Voice(codes=self._encoder.encode(audio_path))

    def stream(self, text: str, *, voice=None, language: str = "English", max_new_tokens: int = 400,
               seed: int = 1234):
        """Validate like the reference (``api.py:171-181``) and stream from the engine."""
        if not isinstance(text, str) or not text.strip():
            raise ValueError("text must be a nonempty string")
        if not isinstance(language, str) or not language.strip():
            raise ValueError("language must be a nonempty string")
        if not isinstance(max_new_tokens, int) or max_new_tokens < 33:
            raise ValueError("At least 33 generated steps are required for all 32 codebooks")
        if not isinstance(seed, int) or not 0 <= seed < 2**32:
            raise ValueError("seed must be an integer in [0, 2**32)")
        if voice is not None and not isinstance(voice, Voice):
            raise TypeError("voice must be returned by clone_voice()")
        if not hasattr(self._engine, "stream"):
            raise NotImplementedError("Text-to-PCM streaming needs the codec and text processor, which are "
                                      "outside the B200 decode package; drive FastLLM.step directly")

        def generate():
            started = time.perf_counter()
            with self._request():
                emitted = 0
                first = None
                for chunk in self._engine.stream(text, None if voice is None else voice.codes, language,
                                                 max_new_tokens):
                    elapsed = (time.perf_counter() - started) * 1000
                    first = elapsed if first is None else first
                    yield AudioChunk(chunk.pcm, emitted, elapsed, chunk.sample_rate)
                    emitted += 1
                self._last_metrics = {**getattr(self._engine, "last_metrics", {}), "ttfa_ms": first,
                                      "total_ms": (time.perf_counter() - started) * 1000,
                                      "output_chunks": emitted}

        return generate()

    @property
    def metrics(self) -> dict:
        from copy import deepcopy
        if self._closed:
            raise RuntimeError("This model is closed")
        return deepcopy(self._last_metrics)

    def close(self) -> None:
        if not self._lock.acquire(blocking=False):
            raise RuntimeError("Close the active stream before closing this model")
        try:
            if not self._closed:
                codec = getattr(self._engine, "codec", None)
                if codec is not None and hasattr(codec, "close"):
                    codec.close()
                self._closed = True
                self._encoder = None
                self._engine = None
        finally:
            self._lock.release()

    def __enter__(self) -> "MossTTS":
        if self._closed:
            raise RuntimeError("This model is closed")
        return self

    def __exit__(self, *_exc) -> None:
        self.close()
