"""The calibrated G32 export on disk: writer, validation and loader (CPU only).

A small export in the reference's format (``src/moss_tts/calibration.py:156-212``:
``config.json`` with ``complete``/``group``/``tts_revision`` and per-file SHA-256, and one
``{packed, scales, shape, group}`` file per layer and projection) is written by
``calibrated_backend.write_export`` and by hand exactly as the reference's exporter writes it,
then read by ``load_export``. The loaded zero-point form must dequantize bit for bit to what
the reference's ``calibrated_quant.dequantize`` of the signed codes gives (the oracle's
``dequantize_signed``), and every validation step of ``install_calibrated`` / ``api.py:83-98``
must refuse a broken export before anything is installed.
"""
import json

import numpy as np
import pytest
import torch

from oracle import quant

from moss_tts._runtime import calibrated_backend as cb

SHAPES = {"qkv": [96, 64], "out": [64, 64], "up": [128, 64], "down": [64, 64]}


def _layers(n_layers, seed=0):
    g = torch.Generator().manual_seed(seed)
    layers = []
    for _ in range(n_layers):
        layer = {}
        for name, (n, k) in SHAPES.items():
            signed = torch.randint(-7, 8, (n, k), generator=g, dtype=torch.int8)
            scales = (torch.rand(n, k // 32, generator=g) * 0.01 + 1e-4).bfloat16()
            layer[name] = (signed, scales)
        layers.append(layer)
    return layers


def test_written_export_loads_and_dequantizes_like_the_reference(tmp_path):
    layers = _layers(2)
    cfg = cb.write_export(tmp_path, layers)
    assert cfg["complete"] and json.loads((tmp_path / "config.json").read_text())["complete"]
    loaded = cb.load_export(tmp_path, SHAPES, layers=2)
    for src, got in zip(layers, loaded):
        for name in SHAPES:
            signed, scales = src[name]
            p = got["gate_up" if name == "up" else name]
            assert p["qzeros"] is None and p["scales"].dtype == torch.bfloat16
            want = quant.dequantize_signed(signed.numpy(), scales.float().numpy())
            have = quant.dequantize_w4(p["qweight"].numpy(), p["scales"].view(torch.int16).numpy().view(np.uint16), None)
            assert np.array_equal(want.view(np.uint32), have.view(np.uint32)), name


def test_reference_written_files_load(tmp_path):
    """Files saved the way the reference's exporter saves them (fp32-free bf16 scales, packed
    low nibble first, calibration.py:190-201), with a reference-style config."""
    layers = _layers(1, seed=3)
    config = {"complete": True, "group": 32, "tts_revision": cb.TTS_REVISION, "projections": {}}
    for name, (signed, scales) in layers[0].items():
        unsigned = signed.to(torch.uint8) & 15
        packed = (unsigned[:, ::2] | (unsigned[:, 1::2] << 4)).contiguous()
        torch.save({"packed": packed, "scales": scales, "shape": list(signed.shape), "group": 32},
                   tmp_path / f"00_{name}.pt")
    (tmp_path / "config.json").write_text(json.dumps(config))
    loaded = cb.load_export(tmp_path, SHAPES, layers=1)
    assert torch.equal(loaded[0]["qkv"]["qweight"], cb.to_zero_point(torch.load(tmp_path / "00_qkv.pt")["packed"]))


def test_broken_exports_are_refused_before_loading(tmp_path):
    cb.write_export(tmp_path, _layers(2, seed=1))
    config = json.loads((tmp_path / "config.json").read_text())
    with pytest.raises(ValueError, match="shape/group mismatch"):
        cb.load_export(tmp_path, {**SHAPES, "down": [64, 128]}, layers=2)
    # a corrupted file no longer matches its recorded checksum
    path = tmp_path / "01_out.pt"
    data = bytearray(path.read_bytes())
    data[-20] ^= 0xFF
    path.write_bytes(bytes(data))
    with pytest.raises(ValueError, match="Checksum mismatch"):
        cb.load_export(tmp_path, SHAPES, layers=2)
    (tmp_path / "01_out.pt").unlink()
    with pytest.raises(ValueError, match="1 projections missing"):
        cb.validate_export(tmp_path, layers=2)
    (tmp_path / "config.json").write_text(json.dumps({**config, "complete": False}))
    with pytest.raises(ValueError, match="incomplete"):
        cb.validate_export(tmp_path, layers=2)
    (tmp_path / "config.json").write_text(json.dumps({**config, "tts_revision": "0" * 40}))
    with pytest.raises(ValueError, match="pinned 8B revision"):
        cb.validate_export(tmp_path, layers=2)


def test_non_bf16_scales_are_refused(tmp_path):
    layers = _layers(1, seed=2)
    signed, scales = layers[0]["out"]
    cb.write_export(tmp_path, layers)
    torch.save({"packed": torch.zeros(64, 32, dtype=torch.uint8), "scales": scales.float() + 1e-7,
                "shape": [64, 64], "group": 32}, tmp_path / "00_out.pt")
    with pytest.raises(ValueError, match="bf16"):
        cb.load_export(tmp_path, SHAPES, layers=1, verify=False)
