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


def _sha256(path: Path) -> str:
    import hashlib
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 22), b""):
            h.update(block)
    return h.hexdigest()


def load_export(folder, shapes: dict, layers: int = 36, device="cpu", verify: bool = True) -> list[dict]:
    """Read and check all projections; returns per-layer ``{name: {qweight, scales, qzeros}}``.

    ``shapes`` maps projection name to the expected ``[N, K]``; scales must be exactly
    representable in bf16 (the reference's ``install_packing`` check, ``dp4a_packing.py:149-152``).
    With ``verify``, every file whose SHA-256 the export's ``config.json`` records
    (``calibration.py:204-209``) is checked against it before it is read.
    """
    folder = Path(folder)
    config = validate_export(folder, layers)
    recorded = config.get("projections", {})
    out = []
    for i in range(layers):
        layer = {}
        for name in PROJECTIONS:
            path = folder / f"{i:02d}_{name}.pt"
            digest = recorded.get(f"{i:02d}_{name}", {}).get("sha256")
            if verify and digest and _sha256(path) != digest:
                raise ValueError(f"Checksum mismatch: {path.name}")
            saved = torch.load(path, map_location="cpu", weights_only=True)
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


def write_export(folder, layers: list, extra: dict | None = None) -> dict:
    """Write a calibrated G32 export in the reference's on-disk format (``calibration.py:156-212``).

    ``layers[i]`` maps ``qkv`` / ``out`` / ``up`` (gate||up) / ``down`` to ``(signed, scales)``:
    int8 codes ``[N, K]`` in [-7, 7] and bf16 scales ``[N, K/32]``. As the reference does, the
    config is first written with ``complete: false``, each projection is saved to a ``.tmp`` file
    and moved into place, its SHA-256 recorded, and ``complete: true`` written last, so an
    interrupted export is never mistaken for a complete one.
    """
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    config = {"complete": False, "group": 32, "static_bf16_scales": True, "code_range": [-7, 7], "codebooks": 32,
              "tts_revision": TTS_REVISION, "torch": torch.__version__, "projections": {}, **(extra or {})}
    config_path = folder / "config.json"
    config_path.write_text(json.dumps(config, indent=2) + "\n")
    for index, layer in enumerate(layers):
        for projection in PROJECTIONS:
            signed, scales = layer[projection]
            if signed.dtype != torch.int8 or signed.ndim != 2 or signed.shape[1] % 2:
                raise ValueError("signed codes must be int8 [N, K]")
            if int(signed.abs().max()) > 7:
                raise ValueError("codes must lie in [-7, 7]")
            unsigned = signed.to(torch.uint8) & 15
            packed = (unsigned[:, ::2] | (unsigned[:, 1::2] << 4)).contiguous()
            name = f"{index:02d}_{projection}"
            destination = folder / f"{name}.pt"
            temporary = destination.with_suffix(".tmp")
            torch.save({"packed": packed.cpu(), "scales": scales.cpu(), "shape": list(signed.shape), "group": 32},
                       temporary)
            temporary.replace(destination)
            config["projections"][name] = {"sha256": _sha256(destination)}
    config["complete"] = True
    config_path.write_text(json.dumps(config, indent=2) + "\n")
    return config
