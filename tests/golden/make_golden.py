"""Write the golden fixtures in this folder from the reference's own CPU code.

Run in a container that has the reference source (read-only), with
``$MOSS_TTS_REFERENCE`` set to the reference checkout (the folder holding ``src/moss_tts``):

    MOSS_TTS_REFERENCE=<reference checkout> python tests/golden/make_golden.py

The reference package is imported from ``$MOSS_TTS_REFERENCE/src`` (its module
name is ``moss_tts``); this repository's seeded synthetic-weight generator is
loaded by file path under a private package name, so both can coexist. Every
fixture is produced by calling reference functions -- ``calibrated_backend.
unpack_signed``, ``calibrated_quant.static_scales`` / ``dequantize``,
``dp4a_packing.pack_interleaved``, ``calibrated_quant.gptq`` (torch backend), ``llm.sample_topk``, the bundled
``MossTTSDelayModel`` and transformers' ``Qwen3`` modules -- on seeded inputs,
or (for the zero-point format, which the reference does not implement) by the
one-line restatement of ``calibrated_quant.dequantize`` with the zero point
subtracted. Outputs are bf16 bit patterns (uint16) in ``.npz`` files, small
enough to commit; large weights are regenerated from their seeds by the tests.

The GPU box never runs this script: the fixtures travel, the reference does not.
"""
import importlib
import os
import sys
import types
import zlib
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
if not os.environ.get("MOSS_TTS_REFERENCE"):
    raise SystemExit("set MOSS_TTS_REFERENCE to the reference checkout (the folder holding src/moss_tts)")
REFERENCE = Path(os.environ["MOSS_TTS_REFERENCE"])
sys.path.insert(0, str(REFERENCE / "src"))

from moss_tts._model.configuration_moss_tts import MossTTSDelayConfig  # noqa: E402
from moss_tts._model.modeling_moss_tts import MossTTSDelayModel  # noqa: E402
from moss_tts._runtime import calibrated_backend, calibrated_quant, dp4a_packing  # noqa: E402
from moss_tts._runtime.llm import sample_topk  # noqa: E402
from transformers import Qwen3Config  # noqa: E402
from transformers.cache_utils import DynamicCache  # noqa: E402
from transformers.models.qwen3 import modeling_qwen3  # noqa: E402


def _load_b200_runtime():
    """Import this repo's ``moss_tts/_runtime`` under the private name ``b200rt``."""
    pkg = types.ModuleType("b200rt")
    pkg.__path__ = [str(REPO / "moss-tts-optimized_b200" / "moss_tts" / "_runtime")]
    sys.modules["b200rt"] = pkg
    return (importlib.import_module("b200rt.config"), importlib.import_module("b200rt.synthetic"))


config_mod, synthetic = _load_b200_runtime()
torch.set_num_threads(os.cpu_count() or 1)
BF16 = torch.bfloat16


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(BF16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(a) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(BF16)


def crc(t: torch.Tensor) -> int:
    return zlib.crc32(bits(t).tobytes())


def zero_point_dequant(qweight_u8, scales_bits, qzeros_u8, group=32) -> torch.Tensor:
    """Restatement of ``calibrated_quant.dequantize`` (``_runtime/calibrated_quant.py:41-42``)
    for unsigned codes with per-group zero points: ``bf16((q - z) * s)``."""
    p = torch.from_numpy(qweight_u8)
    q = torch.stack([p & 15, p >> 4], dim=-1).reshape(p.shape[0], -1)
    zp = torch.from_numpy(qzeros_u8)
    z = torch.stack([zp & 15, zp >> 4], dim=-1).reshape(zp.shape[0], -1)
    s = from_bits(scales_bits)
    return ((q.int() - z.int().repeat_interleave(group, dim=1)).float()
            * s.float().repeat_interleave(group, dim=1)).bfloat16()


def quant_fixture():
    out = {}
    # (a) the reference's signed export path: static scales from a weight, codes in
    # [-7, 7], packed as calibration.py:344-345 does, unpacked and dequantized by the
    # reference's own functions.
    g = torch.Generator().manual_seed(11)
    w = (torch.randn(64, 256, generator=g) * 0.02).bfloat16()
    scales = calibrated_quant.static_scales(w, 32)
    signed = (w.float().view(64, 8, 32) / scales.float()[:, :, None]).round().clamp(-7, 7)
    signed = signed.reshape(64, 256).to(torch.int8)
    unsigned = signed.to(torch.uint8) & 15
    packed = (unsigned[:, ::2] | (unsigned[:, 1::2] << 4)).contiguous()
    unpacked = calibrated_backend.unpack_signed(packed)
    out["signed_packed"] = packed.numpy()
    out["signed_scales"] = bits(scales)
    out["signed_codes"] = unpacked.numpy()
    out["signed_dequant"] = bits(calibrated_quant.dequantize(unpacked, scales, 32))
    out["signed_interleaved"] = dp4a_packing.pack_interleaved(packed).numpy()
    # (b) zero-point format from the synthetic generator, small and config-0 sized.
    rng = np.random.Generator(np.random.PCG64(21))
    small = synthetic.quantized(rng, 96, 512, 32, True)
    out["zp_qweight"], out["zp_scales"], out["zp_qzeros"] = (
        small["qweight"], small["scales"], small["qzeros"])
    out["zp_dequant"] = bits(zero_point_dequant(small["qweight"], small["scales"], small["qzeros"]))
    rng = np.random.Generator(np.random.PCG64(0))
    big = synthetic.quantized(rng, 12288, 4096, 32, True)
    wbig = zero_point_dequant(big["qweight"], big["scales"], big["qzeros"])
    out["config0_dequant_crc32"] = np.array([crc(wbig)], dtype=np.uint64)
    return out, big, wbig


def linear_fixture(big, wbig):
    out = {}
    # config 0: x ~ N(0,1) bf16 [1, 4096] (seed 1), weights seed 0 (quant_fixture).
    x = from_bits(synthetic.activation(1, (1, 4096)))
    out["config0_y"] = bits(torch.nn.functional.linear(x, wbig))
    # small shapes with batch 1, 3 and 8
    rng = np.random.Generator(np.random.PCG64(31))
    small = synthetic.quantized(rng, 384, 1024, 32, True)
    ws = zero_point_dequant(small["qweight"], small["scales"], small["qzeros"])
    for b in (1, 3, 8):
        xb = from_bits(synthetic.activation(100 + b, (b, 1024)))
        out[f"small_x{b}"] = bits(xb)
        out[f"small_y{b}"] = bits(torch.nn.functional.linear(xb, ws))
    out["small_qweight"], out["small_scales"], out["small_qzeros"] = (
        small["qweight"], small["scales"], small["qzeros"])
    return out


def qwen3_config(layers=1, vocab=2048, attn="sdpa"):
    cfg = Qwen3Config(hidden_size=4096, intermediate_size=12288, num_hidden_layers=layers,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                      vocab_size=vocab, rms_norm_eps=1e-6,
                      rope_parameters={"rope_type": "default", "rope_theta": 1e6},
                      max_position_embeddings=8192)
    cfg._attn_implementation = attn
    return cfg


def ops_fixture():
    out = {}
    cfg = qwen3_config()
    # RMSNorm / add-RMSNorm (Qwen3RMSNorm is what FastLLM's Triton norm replaces).
    norm = modeling_qwen3.Qwen3RMSNorm(4096, eps=1e-6)
    w = from_bits(synthetic.activation(40, (4096,), 0.02)).float() + 1.0
    norm.weight.data = w.bfloat16()
    norm = norm.to(BF16)
    x = from_bits(synthetic.activation(41, (3, 4096)))
    r = from_bits(synthetic.activation(42, (3, 4096)))
    out["norm_x"], out["norm_r"], out["norm_w"] = bits(x), bits(r), bits(norm.weight)
    out["rmsnorm_y"] = bits(norm(x))
    summed = x + r
    out["add_sum"], out["add_y"] = bits(summed), bits(norm(summed))
    # RoPE tables from the transformers rotary embedding used by FastLLM (llm.py:231).
    rope = modeling_qwen3.Qwen3RotaryEmbedding(cfg)
    positions = np.concatenate([np.arange(0, 64), np.arange(500, 532), np.arange(1020, 1032),
                                np.arange(2040, 2056), np.arange(4080, 4096)])
    cos, sin = rope(torch.zeros(1, dtype=BF16), torch.from_numpy(positions)[None])
    out["rope_positions"], out["rope_cos"], out["rope_sin"] = positions, bits(cos[0]), bits(sin[0])
    # QK head norm + RoPE at position 77 (Qwen3Attention.forward order).
    qkv = from_bits(synthetic.activation(43, (6144,)))
    qn = from_bits(synthetic.activation(44, (128,), 0.02)).float() + 1.0
    kn = from_bits(synthetic.activation(45, (128,), 0.02)).float() + 1.0
    qnorm = modeling_qwen3.Qwen3RMSNorm(128, eps=1e-6)
    knorm = modeling_qwen3.Qwen3RMSNorm(128, eps=1e-6)
    qnorm.weight.data, knorm.weight.data = qn.bfloat16(), kn.bfloat16()
    qnorm, knorm = qnorm.to(BF16), knorm.to(BF16)
    c, s = rope(torch.zeros(1, dtype=BF16), torch.tensor([[77]]))
    q = qnorm(qkv[:4096].view(1, 1, 32, 128)).transpose(1, 2)
    k = knorm(qkv[4096:5120].view(1, 1, 8, 128)).transpose(1, 2)
    q, k = modeling_qwen3.apply_rotary_pos_emb(q, k, c, s)
    out["rope_qkv"], out["rope_qn"], out["rope_kn"] = bits(qkv), bits(qnorm.weight), bits(knorm.weight)
    out["rope_q"], out["rope_k"] = bits(q[0, :, 0]), bits(k[0, :, 0])
    # SiLU(gate) * up as Qwen3MLP computes it (act on bf16, product in bf16).
    gu = from_bits(synthetic.activation(46, (2, 2 * 12288), 2.0))
    act = torch.nn.functional.silu(gu[:, :12288]) * gu[:, 12288:]
    out["silu_in"], out["silu_out"] = bits(gu), bits(act)
    # Embedding sum: the reference model's _compute_input_embeddings
    # (_model/modeling_moss_tts.py:199-214) over 33 channels.
    rng = np.random.Generator(np.random.PCG64(47))
    text = torch.nn.Embedding(2048, 4096).to(BF16)
    text.weight.data = from_bits(synthetic._normal_bf16(rng, (2048, 4096)))
    ext = torch.nn.ModuleList([torch.nn.Embedding(1025, 4096).to(BF16) for _ in range(32)])
    audio = synthetic._normal_bf16(rng, (32, 1025, 4096))
    for i, e in enumerate(ext):
        e.weight.data = from_bits(audio[i])
    ids = torch.from_numpy(rng.integers(0, 1025, size=(2, 1, 33)))
    ids[..., 0] = torch.from_numpy(rng.integers(0, 2048, size=(2, 1)))
    holder = types.SimpleNamespace(get_input_embeddings=lambda: text, emb_ext=ext)
    emb = MossTTSDelayModel._compute_input_embeddings(holder, ids)
    out["emb_ids"], out["emb_out"] = ids.numpy(), bits(emb)
    return out


def load_layer(layer, lw, group=32):
    """Install synthetic W4 weights (dequantized) into an HF Qwen3DecoderLayer."""
    def deq(p):
        return zero_point_dequant(p["qweight"], p["scales"], p["qzeros"], group)
    a, m = layer.self_attn, layer.mlp
    qkv = deq(lw["qkv"])
    a.q_proj.weight.data, a.k_proj.weight.data, a.v_proj.weight.data = (
        qkv[:4096].clone(), qkv[4096:5120].clone(), qkv[5120:].clone())
    a.o_proj.weight.data = deq(lw["out"])
    gu = deq(lw["gate_up"])
    m.gate_proj.weight.data, m.up_proj.weight.data = gu[:12288].clone(), gu[12288:].clone()
    m.down_proj.weight.data = deq(lw["down"])
    a.q_norm.weight.data, a.k_norm.weight.data = from_bits(lw["q_norm"]), from_bits(lw["k_norm"])
    layer.input_layernorm.weight.data = from_bits(lw["input_norm"])
    layer.post_attention_layernorm.weight.data = from_bits(lw["post_norm"])


def layer_fixture():
    """One decoder-layer decode step at context 96 and at context 2048 (config 2)."""
    out = {}
    dc = config_mod.DecoderConfig()
    weights = synthetic.decoder_weights(dc.with_(vocab_size=16), seed=5, layers=1)
    lw = weights["layers"][0]
    cfg = qwen3_config()
    layer = modeling_qwen3.Qwen3DecoderLayer(cfg, 0).to(BF16)
    load_layer(layer, lw)
    rope = modeling_qwen3.Qwen3RotaryEmbedding(cfg)
    for ctx, seed in ((96, 61), (2048, 62)):
        k = from_bits(synthetic.activation(seed, (1, 8, ctx, 128)))
        v = from_bits(synthetic.activation(seed + 100, (1, 8, ctx, 128)))
        x = from_bits(synthetic.activation(seed + 200, (1, 1, 4096)))
        cache = DynamicCache(config=cfg)
        cache.update(k, v, 0)
        pos = torch.tensor([[ctx]])
        with torch.no_grad():
            y = layer(x, attention_mask=None, position_ids=pos, past_key_values=cache,
                      use_cache=True, position_embeddings=rope(x, pos), cache_position=pos[0])
        y = y[0] if isinstance(y, tuple) else y
        kk, vv = cache.layers[0].keys, cache.layers[0].values
        out[f"ctx{ctx}_y"] = bits(y.reshape(-1))
        out[f"ctx{ctx}_krow"] = bits(kk[0, :, ctx])
        out[f"ctx{ctx}_vrow"] = bits(vv[0, :, ctx])
    return out


def mlp_fixture():
    """Config 1: RMSNorm -> W4A16 gate/up -> SiLU*up -> W4A16 down, batch 1/4/8."""
    out = {}
    rng = np.random.Generator(np.random.PCG64(71))
    gu = synthetic.quantized(rng, 2 * 12288, 4096, 32, True)
    dn = synthetic.quantized(rng, 4096, 12288, 32, True)
    nw = synthetic._normal_bf16(rng, (4096,), 0.02, 1.0)
    cfg = qwen3_config()
    mlp = modeling_qwen3.Qwen3MLP(cfg).to(BF16)
    w = zero_point_dequant(gu["qweight"], gu["scales"], gu["qzeros"])
    mlp.gate_proj.weight.data, mlp.up_proj.weight.data = w[:12288].clone(), w[12288:].clone()
    mlp.down_proj.weight.data = zero_point_dequant(dn["qweight"], dn["scales"], dn["qzeros"])
    norm = modeling_qwen3.Qwen3RMSNorm(4096, eps=1e-6).to(BF16)
    norm.weight.data = from_bits(nw)
    for b in (1, 4, 8):
        x = from_bits(synthetic.activation(80 + b, (b, 4096)))
        with torch.no_grad():
            out[f"b{b}_y"] = bits(mlp(norm(x)))
    return out


def audio_schedule(step: int):
    """(audio_length, delay_length) used by the decode fixture: audio grows for 30
    steps, then the delay counter runs, reaching 32 at step 62."""
    audio_length = min(step + 1, 32)
    delay = -1 if step < 30 else step - 30
    return audio_length, delay


def reference_model(dc, weights):
    """The reference's MossTTSDelayModel (bf16, CPU, SDPA attention) holding the synthetic weights."""
    qcfg = qwen3_config(layers=dc.num_layers, vocab=dc.vocab_size)
    mcfg = MossTTSDelayConfig(language_config=qcfg.to_dict(), n_vq=32, audio_vocab_size=1024,
                              pad_token_id=dc.pad_token_id, im_start_token_id=dc.im_start_token_id,
                              im_end_token_id=dc.im_end_token_id,
                              audio_user_slot_token_id=dc.audio_user_slot_token_id,
                              audio_assistant_gen_slot_token_id=dc.audio_assistant_gen_slot_token_id,
                              audio_assistant_delay_slot_token_id=dc.audio_assistant_delay_slot_token_id,
                              audio_start_token_id=dc.audio_start_token_id,
                              audio_end_token_id=dc.audio_end_token_id)
    mcfg.language_config._attn_implementation = "sdpa"
    model = MossTTSDelayModel(mcfg).to(BF16).eval()
    for layer, lw in zip(model.language_model.layers, weights["layers"]):
        load_layer(layer, lw)
    model.language_model.norm.weight.data = from_bits(weights["final_norm"])
    model.language_model.embed_tokens.weight.data = from_bits(weights["embed_text"])
    for i, e in enumerate(model.emb_ext):
        e.weight.data = from_bits(weights["embed_audio"][i])
    model.lm_heads[0].weight.data = from_bits(weights["head_text"])
    for i in range(32):
        model.lm_heads[i + 1].weight.data = from_bits(weights["head_audio"][i])
    return model, mcfg


def prefill_fixture(n=40):
    """FastLLM.prefill of an n-token prompt (llm.py:303-318 without a captured bucket): the
    2-layer model of the decode fixture runs the whole prompt as one causal pass at positions
    0..n-1; the last row gives the full text-head logits and the 32 x 1024 audio logits."""
    dc = config_mod.small_vocab(config_mod.DecoderConfig(), vocab=2048, layers=2)
    weights = synthetic.decoder_weights(dc, seed=7)
    model, _ = reference_model(dc, weights)
    rng = np.random.Generator(np.random.PCG64(79))
    ids = torch.full((1, n, 33), 1024, dtype=torch.long)
    ids[0, :, 0] = torch.from_numpy(rng.integers(0, dc.vocab_size - 16, size=n))
    ids[0, :, 1:] = torch.from_numpy(rng.integers(0, 1025, size=(n, 32)))
    audio_heads = torch.cat([h.weight[:1024] for h in model.lm_heads[1:]], 0)
    with torch.no_grad():
        emb = model._compute_input_embeddings(ids)
        pos = torch.arange(n)
        h = model.language_model(inputs_embeds=emb, position_ids=pos[None], use_cache=False).last_hidden_state[0, -1]
        text = torch.nn.functional.linear(h, model.lm_heads[0].weight)
        audio = torch.nn.functional.linear(h, audio_heads).view(32, 1024)
    return {"ids": ids.numpy(), "hidden": bits(h), "text": bits(text), "audio": bits(audio)}


def decode_fixture(steps=64):
    """Teacher-forced greedy decode of a 2-layer, full-width, small-vocab model through
    the reference's MossTTSDelayModel, with FastLLM's head/mask semantics."""
    dc = config_mod.small_vocab(config_mod.DecoderConfig(), vocab=2048, layers=2)
    weights = synthetic.decoder_weights(dc, seed=7)
    model, mcfg = reference_model(dc, weights)
    # FastLLM's decode heads (llm.py:188-191).
    text_ids = torch.tensor([dc.audio_assistant_gen_slot_token_id,
                             dc.audio_assistant_delay_slot_token_id])
    audio_heads = torch.cat([h.weight[:1024] for h in model.lm_heads[1:]], 0)
    text_head = model.lm_heads[0].weight[text_ids]
    channels = torch.arange(32)
    rng = np.random.Generator(np.random.PCG64(73))
    ids = torch.full((1, 1, 33), 1024, dtype=torch.long)
    ids[0, 0, 0] = int(rng.integers(0, dc.vocab_size - 16))
    ids[0, 0, 1:] = torch.from_numpy(rng.integers(0, 1024, size=32))
    cache = DynamicCache(config=mcfg.language_config)
    rec = {k: [] for k in ("ids", "next", "text", "audio_top2", "hidden", "audio_logits")}
    rec_steps = list(range(0, steps, 8)) + [steps - 1]
    for step in range(steps):
        audio_length, delay = audio_schedule(step)
        pos = torch.tensor([step])
        with torch.no_grad():
            emb = model._compute_input_embeddings(ids)
            h = model.language_model(inputs_embeds=emb, past_key_values=cache, cache_position=pos,
                                     position_ids=pos[None], use_cache=True).last_hidden_state[0, -1]
            text = torch.nn.functional.linear(h, text_head)
            audio = torch.nn.functional.linear(h, audio_heads).view(32, 1024)
        # llm.py:280-287 with greedy=True (sample_topk with temperature 0 is argmax)
        text_token = text_ids[sample_topk(text, 0)]
        if delay >= 0:
            text_token = torch.tensor(dc.audio_assistant_delay_slot_token_id)
        if delay == 32:
            text_token = torch.tensor(dc.audio_end_token_id)
        audio_tokens = sample_topk(audio, 0)
        valid = (channels < audio_length) & ((delay < 0) | (channels >= delay))
        audio_tokens = torch.where(valid, audio_tokens, 1024)
        nxt = torch.cat([text_token.reshape(1), audio_tokens]).reshape(1, 1, 33)
        top2 = audio.float().topk(2, dim=-1).values
        rec["ids"].append(ids.reshape(-1).numpy().copy())
        rec["next"].append(nxt.reshape(-1).numpy().copy())
        rec["text"].append(bits(text))
        rec["audio_top2"].append((top2[:, 0] - top2[:, 1]).numpy())
        if step in rec_steps:
            rec["hidden"].append(bits(h))
            rec["audio_logits"].append(bits(audio))
        ids = nxt
    out = {k: np.stack(v) for k, v in rec.items()}
    out["hidden_steps"] = np.array(rec_steps)
    return out


def sampling_fixture(draws=20000):
    """``llm.sample_topk`` with the decode step's settings (audio: T 1.7, top-k 25, top-p 0.8;
    text: T 1.5, top-k 2, top-p 1.0) drawn ``draws`` times per row on seeded bf16 logits: the
    reference's empirical counts per token."""
    g = torch.Generator().manual_seed(51)
    audio = (torch.randn(6, 1024, generator=g) * torch.tensor([1.0, 2.0, 3.0, 4.0, 6.0, 0.5])[:, None]).bfloat16()
    text = (torch.randn(4, 2, generator=g) * 2.0).bfloat16()
    torch.manual_seed(52)
    out = {"audio_logits": bits(audio), "text_logits": bits(text), "draws": np.array([draws])}
    picks = sample_topk(audio.repeat(draws, 1), 1.7).view(draws, 6)
    out["audio_counts"] = np.stack([np.bincount(picks[:, r].numpy(), minlength=1024) for r in range(6)]).astype(np.int32)
    picks = sample_topk(text.repeat(draws, 1), 1.5, 2, 1.0).view(draws, 4)
    out["text_counts"] = np.stack([np.bincount(picks[:, r].numpy(), minlength=2) for r in range(4)]).astype(np.int32)
    return out


def gptq_fixture():
    """``calibrated_quant.gptq`` (torch backend, the reference's own column loop) on seeded
    weights and calibration inputs: two 128-column blocks with act-order and one dead input
    column, and one block without act-order."""
    out = {}
    for name, (n, k, actorder, seed) in {"act": (48, 256, True, 41), "plain": (32, 128, False, 42)}.items():
        g = torch.Generator().manual_seed(seed)
        w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
        x = torch.randn(192, k, generator=g) * torch.linspace(0.2, 2.0, k)
        if actorder:
            x[:, 5] = 0  # a dead input column: zero Hessian diagonal
        signed, scales = calibrated_quant.gptq(w, x, group=32, actorder=actorder, backend="torch")
        out[f"{name}_weight"] = bits(w)
        out[f"{name}_inputs"] = x.numpy()
        out[f"{name}_signed"] = signed.numpy()
        out[f"{name}_scales"] = bits(scales)
    return out


def main():
    if sys.argv[1:] == ["prefill"]:  # only the prefill fixture
        np.savez_compressed(HERE / "prefill.npz", **prefill_fixture())
        return
    if sys.argv[1:] == ["gptq"]:  # only the GPTQ fixture
        np.savez_compressed(HERE / "gptq.npz", **gptq_fixture())
        return
    if sys.argv[1:] == ["sampling"]:  # only the sampler fixture
        np.savez_compressed(HERE / "sampling.npz", **sampling_fixture())
        return
    q, big, wbig = quant_fixture()
    np.savez_compressed(HERE / "quant.npz", **q)
    np.savez_compressed(HERE / "linear.npz", **linear_fixture(big, wbig))
    del big, wbig
    np.savez_compressed(HERE / "ops.npz", **ops_fixture())
    np.savez_compressed(HERE / "layer.npz", **layer_fixture())
    np.savez_compressed(HERE / "mlp.npz", **mlp_fixture())
    np.savez_compressed(HERE / "decode.npz", **decode_fixture())
    np.savez_compressed(HERE / "prefill.npz", **prefill_fixture())
    np.savez_compressed(HERE / "gptq.npz", **gptq_fixture())
    np.savez_compressed(HERE / "sampling.npz", **sampling_fixture())
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
