"""Public result types (mirror ``src/moss_tts/types.py`` of the reference)."""
from dataclasses import dataclass


@dataclass(frozen=True)
class Voice:
    """Reusable reference-voice codes returned by ``MossTTS.clone_voice``."""
    codes: object


@dataclass(frozen=True)
class AudioChunk:
    """One streamed PCM chunk: float samples in [-1, 1], index and elapsed milliseconds."""
    pcm: object
    index: int
    elapsed_ms: float
    sample_rate: int = 48000

    def pcm16(self) -> bytes:
        import torch
        return (self.pcm.clamp(-1, 1) * 32767).round().to(torch.int16).cpu().numpy().tobytes()
