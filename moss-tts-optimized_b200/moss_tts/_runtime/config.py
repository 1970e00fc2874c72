"""Decoder configuration for the MOSS-TTS v1.5 8B backbone (Qwen3-8B shaped).

Defaults mirror the reference's pinned model: ``MossTTSDelayConfig``
(``src/moss_tts/_model/configuration_moss_tts.py:64-103``) over a Qwen3 language
config with hidden 4096, intermediate 12288, 36 layers, 32 query / 8 KV heads of
dimension 128, RoPE theta 1e6 and RMSNorm eps 1e-6, and the architecture check
of ``FastLLM`` (``src/moss_tts/_runtime/llm.py:162-163``).
"""
from dataclasses import asdict, dataclass, replace


@dataclass(frozen=True)
class DecoderConfig:
    hidden_size: int = 4096
    intermediate_size: int = 12288
    num_layers: int = 36
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    vocab_size: int = 155648
    n_vq: int = 32
    audio_vocab_size: int = 1024
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6
    group_size: int = 32
    pad_token_id: int = 151643
    im_start_token_id: int = 151644
    im_end_token_id: int = 151645
    audio_user_slot_token_id: int = 151654
    audio_assistant_gen_slot_token_id: int = 151656
    audio_assistant_delay_slot_token_id: int = 151662
    audio_start_token_id: int = 151652
    audio_end_token_id: int = 151653
    audio_pad_code: int = 1024

    @property
    def qkv_size(self) -> int:
        return (self.num_heads + 2 * self.num_kv_heads) * self.head_dim

    def as_dict(self) -> dict:
        return asdict(self)

    def with_(self, **changes) -> "DecoderConfig":
        return replace(self, **changes)

    def validate(self) -> None:
        """The decode kernels are specialised to this architecture, as the
        reference's are (``llm.py:162-163``)."""
        if (self.hidden_size, self.head_dim, self.num_heads, self.num_kv_heads, self.n_vq,
                self.audio_vocab_size) != (4096, 128, 32, 8, 32, 1024):
            raise ValueError("These specialized kernels require the MOSS-TTS-v1.5 Qwen3-8B "
                             "architecture")
        if self.group_size != 32:
            raise ValueError("Only G32 quantization groups are supported")
        if self.intermediate_size % 256:
            raise ValueError("intermediate_size must be a multiple of 256")


def small_vocab(cfg: DecoderConfig, vocab: int = 2048, layers: int = 2) -> DecoderConfig:
    """A test-sized variant: full hidden width and heads, fewer layers, a small text
    vocabulary with the special token ids remapped inside it."""
    base = vocab - 16
    return cfg.with_(
        num_layers=layers, vocab_size=vocab, pad_token_id=base, im_start_token_id=base + 1,
        im_end_token_id=base + 2, audio_user_slot_token_id=base + 3,
        audio_assistant_gen_slot_token_id=base + 4, audio_assistant_delay_slot_token_id=base + 5,
        audio_start_token_id=base + 6, audio_end_token_id=base + 7)
