"""Load the reference's calibrated G32 export into B200 W4A16 projections.

On-disk format (reference ``src/moss_tts/calibration.py:156-212``): a directory with
``config.json`` (``complete``, ``group == 32``, ``tts_revision``) and 144 files
``{layer:02d}_{qkv,out,up,down}.pt``, each ``{"packed": uint8 [N, K/2] two's-complement
codes in [-7, 7], "scales": [N, K/32], "shape": [N, K], "group": 32}`` where ``up`` is the
concatenated gate||up projection. Validation mirrors ``calibrated_backend.install_calibrated``
(``_runtime/calibrated_backend.py:30-56``) and ``api.py:83-98``: everything is checked
before any tensor is installed.

The symmetric codes become the zero-point format by flipping bit 3 of every nibble
(``q = code + 8``) with an implicit zero point of 8, so the same W4A16 kernel serves
both formats and the dequantized weights are unchanged bit for bit.
"""
import json
from pathlib import Path

import torch

TTS_REVISION = "cdd3b911b1585e3f2dbc7775ef10f9926f58850a"  # reference models.py:7
PROJECTIONS = ("qkv", "out", "up", "down")


def unpack_signed(packed):
    """Two's-complement nibbles -> int8 codes (reference ``calibrated_backend.py:8-13``)."""
    lo = (packed & 15).to(torch.int8)
    hi = (packed >> 4).to(torch.int8)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    return torch.stack([lo, hi], dim=-1).reshape(packed.shape[0], -1)


def to_zero_point(packed):
    """Signed-code bytes -> unsigned codes ``q = code + 8`` (zero point 8)."""
    return packed ^ 0x88


def validate_export(folder, layers: int = 36) -> dict:
    folder = Path(folder)
    config = json.loads((folder / "config.json").read_text())
    if config.get("complete") is False:
        raise ValueError("The calibrated export is incomplete")
    if config.get("group") != 32 or config.get("tts_revision") != TTS_REVISION:
        raise ValueError("A G32 export of the pinned 8B revision is required")
    missing = [folder / f"{i:02d}_{p}.pt" for i in range(layers) for p in PROJECTIONS
               if not (folder / f"{i:02d}_{p}.pt").is_file()]
    if missing:
        raise ValueError(f"Incomplete calibrated export: {len(missing)} projections missing")
    return config


def load_export(folder, shapes: dict, layers: int = 36, device="cpu") -> list[dict]:
    """Read and check all projections; returns per-layer ``{name: {qweight, scales, qzeros}}``.

    ``shapes`` maps projection name to the expected ``[N, K]``; scales must be exactly
    representable in bf16 (the reference's ``install_packing`` check, ``dp4a_packing.py:149-152``).
    """
    folder = Path(folder)
    config = validate_export(folder, layers)
    out = []
    for i in range(layers):
        layer = {}
        for name in PROJECTIONS:
            saved = torch.load(folder / f"{i:02d}_{name}.pt", map_location="cpu", weights_only=True)
            if list(saved["shape"]) != list(shapes[name]) or saved["group"] != config["group"]:
                raise ValueError(f"Projection shape/group mismatch: {i} {name}")
            scales = saved["scales"]
            if not torch.equal(scales.float(), scales.bfloat16().float()):
                raise ValueError("Scales are not exactly representable in bf16")
            layer["gate_up" if name == "up" else name] = {
                "qweight": to_zero_point(saved["packed"].to(torch.uint8)).contiguous(),
                "scales": scales.bfloat16().contiguous(), "qzeros": None}
        out.append(layer)
    if device != "cpu":
        out = [{k: {n: (t.to(device) if t is not None else None) for n, t in p.items()}
                for k, p in layer.items()} for layer in out]
    return out
