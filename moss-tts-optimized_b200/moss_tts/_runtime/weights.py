"""Device-resident decoder weights for the B200 decode engine.

Layout in HBM (one GPU, or one tensor-parallel shard):
* per layer: RMSNorm weights (bf16 [H], q/k norm [128]); four projections, each
  either W4 (``qweight`` uint8 [N, K/2], ``scales`` bf16 [N, K/32], ``qzeros`` uint8
  [N, K/64] or None) or bf16 (``weight`` [N, K]): fused q|k|v [6144, 4096], o
  [4096, 4096], gate||up [24576, 4096], down [4096, 12288] -- the fused layout of the
  reference's ``fuse_backbone`` (``src/moss_tts/_runtime/llm.py:133-145``);
* text and audio embeddings (bf16 [V, H] and [32, 1025, H]);
* decode heads as ``FastLLM`` keeps them (``llm.py:188-191``): the two audio-phase
  text-head rows [2, H] and the first 1024 rows of each audio head [32 * 1024, H];
  the full text head [V, H] for ``full_step``.
"""
from dataclasses import dataclass, field

import numpy as np
import torch

from .config import DecoderConfig


def _t(a, device, dtype=None):
    if a is None:
        return None
    if isinstance(a, torch.Tensor):
        t = a
    else:
        arr = np.ascontiguousarray(a)
        if arr.dtype == np.uint16:
            t = torch.from_numpy(arr.view(np.int16)).view(torch.bfloat16)
        else:
            t = torch.from_numpy(arr)
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.to(device).contiguous()


@dataclass
class Projection:
    n: int
    k: int
    qweight: torch.Tensor | None = None  # uint8 [N, K/2]
    scales: torch.Tensor | None = None   # bf16 [N, K/32]
    qzeros: torch.Tensor | None = None   # uint8 [N, K/64] or None (z = 8)
    weight: torch.Tensor | None = None   # bf16 [N, K] (bf16 preset)
    packed: dict = field(default_factory=dict, repr=False, compare=False)  # paired -> packed tiles

    @property
    def quantized(self) -> bool:
        return self.qweight is not None

    def packed_tiles(self, paired: bool = False) -> torch.Tensor:
        """Tile-major copy of the W4 weights for ``mt_w4a16_linear_packed``, made on first
        use on the weights' device (the load-time repack; ``paired`` interleaves the gate
        and up halves tile by tile)."""
        key = bool(paired)
        if key not in self.packed:
            from . import native
            mode = native.LINEAR_PAIRED if paired else 0
            nbytes, _ = native.w4a16_packed_size(self.n, self.k, self.qzeros is not None, mode)
            buf = torch.empty(nbytes, dtype=torch.uint8, device=self.qweight.device)
            native.call("mt_w4a16_pack", self.qweight.data_ptr(), self.scales.data_ptr(),
                        native.ptr(self.qzeros), self.n, self.k, mode, buf.data_ptr(),
                        torch.cuda.current_stream(buf.device).cuda_stream)
            self.packed[key] = buf
        return self.packed[key]

    @classmethod
    def from_host(cls, p: dict, device) -> "Projection":
        if "weight" in p:
            w = _t(p["weight"], device, torch.bfloat16)
            return cls(w.shape[0], w.shape[1], weight=w)
        qw = _t(p["qweight"], device)
        if qw.dtype == torch.int32:
            qw = qw.view(torch.uint8)
        return cls(qw.shape[0], qw.shape[1] * 2, qweight=qw, scales=_t(p["scales"], device, torch.bfloat16),
                   qzeros=_t(p.get("qzeros"), device))

    def rows(self, start: int, stop: int) -> "Projection":
        """Output-row slice (column-parallel shard)."""
        def s(t):
            return None if t is None else t[start:stop].contiguous()
        return Projection(stop - start, self.k, s(self.qweight), s(self.scales), s(self.qzeros), s(self.weight))

    def cols(self, start: int, stop: int) -> "Projection":
        """Input-column slice (row-parallel shard); boundaries must align to 64."""
        if start % 64 or stop % 64:
            raise ValueError("K shards must align to 64 (two quantization groups)")
        def s(t, div):
            return None if t is None else t[:, start // div:stop // div].contiguous()
        return Projection(self.n, stop - start, s(self.qweight, 2), s(self.scales, 32), s(self.qzeros, 64),
                          s(self.weight, 1))

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.qweight, self.scales, self.qzeros, self.weight)
                   if t is not None)


@dataclass
class LayerWeights:
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    qkv: Projection
    out: Projection
    gate_up: Projection
    down: Projection

    def nbytes(self) -> int:
        return sum(p.nbytes() for p in (self.qkv, self.out, self.gate_up, self.down))


@dataclass
class DecoderWeights:
    cfg: DecoderConfig
    layers: list
    final_norm: torch.Tensor
    embed_text: torch.Tensor
    embed_audio: torch.Tensor
    head_text_rows: torch.Tensor   # [2, H] rows (gen_slot, delay_slot)
    head_audio: torch.Tensor       # [n_vq * 1024, H]
    head_text: torch.Tensor | None = None  # [V, H], full text head (full_step)
    preset: str = "gptq"
    meta: dict = field(default_factory=dict)

    @property
    def device(self):
        return self.final_norm.device

    @classmethod
    def from_host(cls, cfg: DecoderConfig, w: dict, device="cuda", preset="gptq") -> "DecoderWeights":
        """Upload the plain host dict (``synthetic.decoder_weights`` layout)."""
        layers = []
        for lw in w["layers"]:
            layers.append(LayerWeights(
                _t(lw["input_norm"], device), _t(lw["post_norm"], device), _t(lw["q_norm"], device),
                _t(lw["k_norm"], device), Projection.from_host(lw["qkv"], device),
                Projection.from_host(lw["out"], device), Projection.from_host(lw["gate_up"], device),
                Projection.from_host(lw["down"], device)))
        ids = [cfg.audio_assistant_gen_slot_token_id, cfg.audio_assistant_delay_slot_token_id]
        head_text = _t(w["head_text"], device)
        av = cfg.audio_vocab_size
        head_audio = _t(np.ascontiguousarray(np.asarray(w["head_audio"])[:, :av]).reshape(-1, cfg.hidden_size)
                        if not isinstance(w["head_audio"], torch.Tensor)
                        else w["head_audio"][:, :av].reshape(-1, cfg.hidden_size), device)
        return cls(cfg, layers, _t(w["final_norm"], device), _t(w["embed_text"], device),
                   _t(w["embed_audio"], device), head_text[ids].contiguous(), head_audio, head_text,
                   preset)

    @classmethod
    def random(cls, cfg: DecoderConfig, device="cuda", seed: int = 0, preset: str = "gptq",
               zero_points: bool = True, full_text_head: bool = True) -> "DecoderWeights":
        """Random-init weights generated directly on the device (benchmark-sized models).

        Same distributions as ``synthetic.decoder_weights`` but drawn from torch's device
        generator, so a full 36-layer model is ready in seconds; not bit-identical to the
        host generator (tests use the host generator)."""
        g = torch.Generator(device=device).manual_seed(seed)
        h, i, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim

        def normal(shape, std=0.02, mean=0.0):
            return (torch.randn(shape, generator=g, device=device) * std + mean).to(torch.bfloat16)

        def proj(n, k):
            if preset == "bf16":
                return Projection(n, k, weight=normal((n, k), 0.0125))
            qw = torch.randint(0, 256, (n, k // 2), generator=g, device=device, dtype=torch.uint8)
            sc = (torch.randn((n, k // 32), generator=g, device=device).abs() * 0.02 / 7 + 1e-4).to(torch.bfloat16)
            qz = None
            if zero_points:
                z = torch.randint(6, 10, (n, k // 32), generator=g, device=device, dtype=torch.uint8)
                qz = (z[:, 0::2] | (z[:, 1::2] << 4)).contiguous()
            return Projection(n, k, qw, sc, qz)

        layers = []
        for _ in range(cfg.num_layers):
            layers.append(LayerWeights(normal((h,), 0.02, 1.0), normal((h,), 0.02, 1.0),
                                       normal((d,), 0.02, 1.0), normal((d,), 0.02, 1.0),
                                       proj(cfg.qkv_size, h), proj(h, cfg.num_heads * d),
                                       proj(2 * i, h), proj(h, i)))
        head_text = normal((cfg.vocab_size, h)) if full_text_head else None
        ids = [cfg.audio_assistant_gen_slot_token_id, cfg.audio_assistant_delay_slot_token_id]
        rows = head_text[ids].contiguous() if head_text is not None else normal((2, h))
        return cls(cfg, layers, normal((h,), 0.02, 1.0), normal((cfg.vocab_size, h)),
                   normal((cfg.n_vq, cfg.audio_vocab_size + 1, h)), rows,
                   normal((cfg.n_vq * cfg.audio_vocab_size, h)), head_text, preset)

    def layer_bytes(self) -> int:
        return sum(layer.nbytes() for layer in self.layers)
