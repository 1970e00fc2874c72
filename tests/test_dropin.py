"""The reference's quantized-linear module surface on CPU (no GPU, no launches).

``dp4a_packing``, ``dp4a_norm_projection``, ``int4_dp4a`` and ``calibrated_quant`` keep the
reference's names and argument checks; every check below fires before anything touches the
device, and valid CPU tensors are refused (there is no CPU path). The nibble interleave is
pinned to the fixture the reference's own ``pack_interleaved`` wrote.
"""
import numpy as np
import pytest
import torch

from conftest import golden

from moss_tts._runtime import calibrated_quant, dp4a_norm_projection, dp4a_packing, int4_dp4a


def test_interleave_matches_reference_fixture():
    g = golden("quant")
    packed = torch.from_numpy(g["signed_packed"])
    inter = dp4a_packing.pack_interleaved(packed)
    assert np.array_equal(inter.numpy(), g["signed_interleaved"])
    assert np.array_equal(dp4a_packing.unpack_interleaved(inter).numpy(), g["signed_codes"])
    from moss_tts._runtime.quantized import deinterleave_nibbles
    assert torch.equal(deinterleave_nibbles(inter), packed)


def test_linear_argument_checks_match_reference():
    packed = torch.zeros(16, 64, dtype=torch.uint8)
    scales = torch.ones(16, 4)
    x = torch.zeros(128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="One contiguous BF16 input row required"):
        dp4a_packing.linear(x.float(), packed, scales)
    with pytest.raises(ValueError, match="One contiguous BF16 input row required"):
        dp4a_packing.linear(torch.zeros(64, dtype=torch.bfloat16), packed, scales)
    with pytest.raises(ValueError, match="prequantized"):
        dp4a_packing.linear(x, packed, scales, prequantized=(torch.zeros(128, dtype=torch.int8), torch.ones(4)))
    with pytest.raises(ValueError, match="tile"):
        dp4a_packing.linear(x, packed, scales, rows=3)
    with pytest.raises(ValueError, match="CUDA"):
        dp4a_packing.linear(x, packed, scales)  # no CPU fallback


def test_project_reads_module_attributes_and_rejects_w4a8_layouts():
    class Mlp:
        pass
    m = Mlp()
    m._quant_down = torch.zeros(16, 64, dtype=torch.uint8)
    m._quant_down_scale = torch.ones(16, 4)
    m._dp4a_group = 32
    m._scaled_dp4a = {"down": {}}
    with pytest.raises(ValueError, match="W4A8-only"):
        dp4a_packing.project(m, "down", torch.zeros(128, dtype=torch.bfloat16))
    del m._scaled_dp4a
    with pytest.raises(ValueError, match="CUDA"):
        dp4a_packing.project(m, "down", torch.zeros(128, dtype=torch.bfloat16))


def test_norm_projection_checks_match_reference():
    x = torch.zeros(4096, dtype=torch.bfloat16)
    nw = torch.ones(4096, dtype=torch.bfloat16)
    w = torch.zeros(64, 2048, dtype=torch.uint8)
    s = torch.ones(64, 128)
    with pytest.raises(ValueError, match="One BF16 K4096 activation row required"):
        dp4a_norm_projection.linear(x[:2048], None, nw, 1e-6, w, s)
    with pytest.raises(ValueError, match="Unsupported fusion tile"):
        dp4a_norm_projection.linear(x, None, nw, 1e-6, w, s, rows=32)
    with pytest.raises(ValueError, match="Contiguous CUDA inputs required"):
        dp4a_norm_projection.linear(x, None, nw, 1e-6, w, s)


def test_int4_dp4a_and_calibrated_quant_checks():
    x = torch.zeros(128, dtype=torch.bfloat16)
    packed = torch.zeros(8, 64, dtype=torch.uint8)
    with pytest.raises(ValueError, match="Expected one contiguous BF16 activation row"):
        int4_dp4a.int4_dp4a(x[:64], packed, torch.ones(8, 4), group=32)
    with pytest.raises(ValueError, match="Grouped activation uses explicit reciprocal rounding"):
        int4_dp4a.int4_dp4a(x, packed, torch.ones(8, 4), group=32, grouped_activation=True)
    with pytest.raises(ValueError, match="G32"):
        int4_dp4a.int4_dp4a(x, packed, torch.ones(8, 1), group=128)
    with pytest.raises(ValueError, match="int8 codes"):
        calibrated_quant.dequantize(torch.zeros(4, 64, dtype=torch.uint8), torch.ones(4, 2), 32)
    with pytest.raises(ValueError, match="CUDA"):
        calibrated_quant.dequantize(torch.zeros(4, 64, dtype=torch.int8), torch.ones(4, 2), 32)
    with pytest.raises(ValueError, match="CUDA"):
        calibrated_quant.static_scales(torch.zeros(4, 64), 32)
    w = torch.zeros(4, 256)
    with pytest.raises(ValueError, match="Dimensions must be divisible"):
        calibrated_quant.gptq(w[:, :200], torch.zeros(8, 200))
    with pytest.raises(ValueError, match="Calibration input shape mismatch"):
        calibrated_quant.gptq(w, torch.zeros(8, 128))
    with pytest.raises(ValueError, match="Unknown GPTQ backend"):
        calibrated_quant.gptq(w, torch.zeros(8, 256), backend="torch")
    with pytest.raises(ValueError, match="CUDA"):
        calibrated_quant.gptq(w, torch.zeros(8, 256))
