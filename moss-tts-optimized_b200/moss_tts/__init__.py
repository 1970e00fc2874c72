"""MOSS-TTS v1.5 8B batch-1 decode on NVIDIA B200 (sm_100a).

Drop-in for the decode hot path of kadirnar/MOSS-TTS-optimized: the public
entry ``MossTTS.from_pretrained(preset="gptq"|"bf16")`` and the module-level
operator signatures of ``moss_tts._runtime.kernels`` and the quantized linear,
backed by hand-written CUDA kernels loaded through a C-ABI shared library.
Importing the package does not import torch (as the reference's does not).
"""

__all__ = ["MossTTS", "AudioChunk", "Voice"]


def __getattr__(name):
    if name == "MossTTS":
        from .api import MossTTS
        return MossTTS
    if name in ("AudioChunk", "Voice"):
        from . import types as _types
        return getattr(_types, name)
    raise AttributeError(name)
