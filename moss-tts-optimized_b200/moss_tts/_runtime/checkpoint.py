"""Read the MOSS-TTS v1.5 safetensors checkpoint into ``DecoderWeights``.

Parameter names are those of the reference's bundled ``MossTTSDelayModel``
(``src/moss_tts/_model/modeling_moss_tts.py:165-191``) over transformers' ``Qwen3Model``:
``language_model.layers.{i}.self_attn.{q,k,v,o}_proj.weight``, ``...q_norm/k_norm``,
``...input_layernorm/post_attention_layernorm``, ``...mlp.{gate,up,down}_proj.weight``,
``language_model.norm``, ``language_model.embed_tokens``, ``emb_ext.{q}`` and
``lm_heads.{0..32}``. Projections are fused the way ``fuse_backbone`` fuses them
(``src/moss_tts/_runtime/llm.py:133-145``): q|k|v and gate||up. With a calibrated G32
export (``calibrated_backend.load_export``) the four projections are replaced by W4 codes.
"""
import json
from pathlib import Path

import torch

from .config import DecoderConfig
from .weights import DecoderWeights, LayerWeights, Projection

MODEL_ID = "OpenMOSS-Team/MOSS-TTS-v1.5"
TTS_REVISION = "cdd3b911b1585e3f2dbc7775ef10f9926f58850a"


def config_from_json(path) -> DecoderConfig:
    data = json.loads(Path(path).read_text())
    lc = data.get("language_config", {})
    rope = (lc.get("rope_parameters") or {}).get("rope_theta", lc.get("rope_theta", 1e6))
    keys = {f for f in DecoderConfig.__dataclass_fields__}
    cfg = DecoderConfig(
        hidden_size=lc.get("hidden_size", 4096), intermediate_size=lc.get("intermediate_size", 12288),
        num_layers=lc.get("num_hidden_layers", 36), num_heads=lc.get("num_attention_heads", 32),
        num_kv_heads=lc.get("num_key_value_heads", 8), head_dim=lc.get("head_dim", 128),
        vocab_size=lc.get("vocab_size", 155648), rope_theta=float(rope),
        rms_norm_eps=lc.get("rms_norm_eps", 1e-6),
        **{k: v for k, v in data.items() if k in keys and k not in ("hidden_size", "vocab_size")})
    return cfg


def find_snapshot(cache_dir=None) -> Path:
    """Locate the pinned revision in a Hugging Face cache (no download: offline)."""
    import os
    roots = [Path(cache_dir)] if cache_dir else []
    roots += [Path(os.environ.get("HF_HUB_CACHE", "")), Path(os.environ.get("HF_HOME", "~/.cache/huggingface")).expanduser() / "hub"]
    for root in roots:
        snap = root / ("models--" + MODEL_ID.replace("/", "--")) / "snapshots" / TTS_REVISION
        if (snap / "config.json").is_file():
            return snap
    raise FileNotFoundError(f"{MODEL_ID}@{TTS_REVISION} is not in the local cache; pass cache_dir")


def load_checkpoint(folder, device="cuda", calibrated_layers=None, cfg: DecoderConfig | None = None,
                    full_text_head: bool = True) -> DecoderWeights:
    from safetensors import safe_open
    folder = Path(folder)
    cfg = cfg or config_from_json(folder / "config.json")
    tensors = {}
    for f in sorted(folder.glob("*.safetensors")):
        with safe_open(str(f), framework="pt") as st:
            for k in st.keys():
                tensors[k] = st.get_tensor(k)

    def get(name):
        t = tensors[name]
        return t.to(torch.bfloat16).to(device).contiguous()

    layers = []
    for i in range(cfg.num_layers):
        p = f"language_model.layers.{i}."
        if calibrated_layers is not None:
            cal = calibrated_layers[i]
            proj = {k: Projection.from_host(cal[k], device) for k in ("qkv", "out", "gate_up", "down")}
        else:
            def cat(*names):
                return torch.cat([get(p + n) for n in names], 0).contiguous()
            mats = {"qkv": cat("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight"),
                    "out": get(p + "self_attn.o_proj.weight"),
                    "gate_up": cat("mlp.gate_proj.weight", "mlp.up_proj.weight"),
                    "down": get(p + "mlp.down_proj.weight")}
            proj = {k: Projection(m.shape[0], m.shape[1], weight=m) for k, m in mats.items()}
        layers.append(LayerWeights(get(p + "input_layernorm.weight"), get(p + "post_attention_layernorm.weight"),
                                   get(p + "self_attn.q_norm.weight"), get(p + "self_attn.k_norm.weight"),
                                   proj["qkv"], proj["out"], proj["gate_up"], proj["down"]))
    av = cfg.audio_vocab_size
    head_text = get("lm_heads.0.weight")
    ids = [cfg.audio_assistant_gen_slot_token_id, cfg.audio_assistant_delay_slot_token_id]
    head_audio = torch.cat([get(f"lm_heads.{q + 1}.weight")[:av] for q in range(cfg.n_vq)], 0).contiguous()
    embed_audio = torch.stack([get(f"emb_ext.{q}.weight") for q in range(cfg.n_vq)]).contiguous()
    return DecoderWeights(cfg, layers, get("language_model.norm.weight"), get("language_model.embed_tokens.weight"),
                          embed_audio, head_text[ids].contiguous(), head_audio,
                          head_text if full_text_head else None,
                          "gptq" if calibrated_layers is not None else "bf16")
