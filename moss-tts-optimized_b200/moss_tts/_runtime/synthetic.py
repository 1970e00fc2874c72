"""Seeded random-init weights of the MOSS-TTS decoder shapes (no checkpoints needed).

Host-side numpy generation, so the same seed yields the same bytes on any
machine (the CPU oracle and the GPU path see identical weights). Layout is the
plain dict accepted by ``moss_tts._runtime.weights.DecoderWeights.from_host``:

* bf16 tensors are ``uint16`` bit arrays;
* int4/G32 projections are ``{"qweight": uint8 [N, K/2], "scales": uint16 [N, K/32],
  "qzeros": uint8 [N, K/64] | None}`` -- codes low nibble first along K (the
  reference's packing, ``src/moss_tts/calibration.py:190-191``), one zero point
  per group packed two per byte;
* bf16 projections are ``{"weight": uint16 [N, K]}``.

Distributions follow the benchmark specification: codes uniform in [0, 15],
zero points uniform in [6, 9], scales ``|N(0, 0.02)| / 7 + 1e-4`` rounded to
bf16, norm weights ``1 + N(0, 0.02)``, embeddings and heads ``N(0, 0.02)``
(the HF ``initializer_range``).
"""
import numpy as np

from .config import DecoderConfig


def f32_to_bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    # finite inputs never wrap: the largest finite pattern is 0xFF7FFFFF
    u = (u + (((u >> 16) & np.uint32(1)) + np.uint32(0x7FFF))) >> np.uint32(16)
    return u.astype(np.uint16).reshape(x.shape)


def bf16_bits_to_f32(bits) -> np.ndarray:
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32).reshape(b.shape)


def _normal_bf16(rng, shape, std=0.02, mean=0.0):
    return f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
                            + np.float32(mean))


def quantized(rng, n: int, k: int, group: int = 32, zero_points: bool = True) -> dict:
    """One W4/G32 projection ``[n, k]`` in the zero-point format."""
    if k % (2 * group):
        raise ValueError("K must be a multiple of 2 * group")
    qweight = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    scales = np.abs(rng.standard_normal((n, k // group), dtype=np.float32)) * np.float32(0.02)
    scales = f32_to_bf16_bits(scales / np.float32(7.0) + np.float32(1e-4))
    qzeros = None
    if zero_points:
        z = rng.integers(6, 10, size=(n, k // group), dtype=np.uint8)
        qzeros = (z[:, 0::2] | (z[:, 1::2] << 4)).astype(np.uint8)
    return {"qweight": qweight, "scales": scales, "qzeros": qzeros}


def bf16_projection(rng, n: int, k: int, std: float = 0.0125) -> dict:
    """One bf16 projection ``[n, k]`` (the bf16 preset); the default std matches
    the W4 weights' spread so activations keep the same scale."""
    return {"weight": _normal_bf16(rng, (n, k), std)}


def decoder_weights(cfg: DecoderConfig, seed: int = 0, *, preset: str = "gptq",
                    zero_points: bool = True, layers: int | None = None) -> dict:
    """Random-init weights for ``cfg`` (``layers`` overrides ``cfg.num_layers``)."""
    if preset not in ("gptq", "bf16"):
        raise ValueError("preset must be 'gptq' or 'bf16'")
    rng = np.random.Generator(np.random.PCG64(seed))
    h, i, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    n_layers = cfg.num_layers if layers is None else layers
    shapes = {"qkv": (cfg.qkv_size, h), "out": (h, cfg.num_heads * d),
              "gate_up": (2 * i, h), "down": (h, i)}

    def projection(name):
        n, k = shapes[name]
        if preset == "gptq":
            return quantized(rng, n, k, cfg.group_size, zero_points)
        return bf16_projection(rng, n, k)

    out = {"layers": []}
    for _ in range(n_layers):
        layer = {"input_norm": _normal_bf16(rng, (h,), 0.02, 1.0),
                 "post_norm": _normal_bf16(rng, (h,), 0.02, 1.0),
                 "q_norm": _normal_bf16(rng, (d,), 0.02, 1.0),
                 "k_norm": _normal_bf16(rng, (d,), 0.02, 1.0)}
        for name in ("qkv", "out", "gate_up", "down"):
            layer[name] = projection(name)
        out["layers"].append(layer)
    av = cfg.audio_vocab_size + 1
    out["final_norm"] = _normal_bf16(rng, (h,), 0.02, 1.0)
    out["embed_text"] = _normal_bf16(rng, (cfg.vocab_size, h))
    out["embed_audio"] = _normal_bf16(rng, (cfg.n_vq, av, h))
    out["head_text"] = _normal_bf16(rng, (cfg.vocab_size, h))
    out["head_audio"] = _normal_bf16(rng, (cfg.n_vq, av, h))
    return out


def activation(seed: int, shape, std: float = 1.0) -> np.ndarray:
    """Seeded bf16 activations ``N(0, std)`` as uint16 bits."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return _normal_bf16(rng, shape, std)
