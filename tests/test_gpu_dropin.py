"""The reference's quantized-linear module surface on a B200, against the oracle.

``dp4a_packing.linear`` / ``project``, ``dp4a_norm_projection.linear``, ``int4_dp4a`` and
``calibrated_quant.dequantize`` / ``static_scales`` take the reference's signed-nibble
export format and run on this library's kernels. Dequantization and static scales are
bit-exact against fixtures the reference's own functions wrote; projections are within
max-abs 2e-2 / rel 1e-2 of the oracle's dequantize-then-matmul.
"""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import ops, quant
from oracle.numerics import from_bf16_bits

from moss_tts._runtime import calibrated_quant, dp4a_norm_projection, dp4a_packing, int4_dp4a

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _check(got, want, label):
    got = got.float().cpu().numpy().reshape(-1).astype(np.float64)
    want = np.asarray(want, dtype=np.float64).reshape(-1)
    err = np.abs(got - want)
    print(f"{label}: max abs err {err.max():.3g}, max rel {np.max(err / np.maximum(np.abs(want), 1e-6)):.3g}")
    assert np.all(err <= ATOL + RTOL * np.abs(want)), (label, err.max())


def _bf16(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def _signed(seed, n, k, dev):
    """Random reference-format weights: codes in [-7, 7] as two's-complement nibbles, bf16 scales."""
    rng = np.random.Generator(np.random.PCG64(seed))
    codes = rng.integers(-7, 8, size=(n, k), dtype=np.int8)
    u = codes.astype(np.uint8) & 15
    packed = (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)
    scales = (np.abs(rng.standard_normal((n, k // 32))) * 0.02 / 7 + 1e-4).astype(np.float32)
    scales = torch.from_numpy(scales).bfloat16().float()  # bf16-exact fp32, as install_calibrated keeps them
    w = quant.dequantize_signed(codes, scales.numpy())
    return torch.from_numpy(packed).to(dev), scales.to(dev), w


def test_calibrated_quant_is_bit_exact_against_reference(cuda_device):
    g = golden("quant")
    codes = torch.from_numpy(g["signed_codes"]).to(cuda_device)
    scales = _bf16(g["signed_scales"], cuda_device)
    out = calibrated_quant.dequantize(codes, scales, 32)
    assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), g["signed_dequant"])
    # the fixture's weight matrix, regenerated: torch.randn(64, 256, seed 11) * 0.02 in bf16
    gen = torch.Generator().manual_seed(11)
    w = (torch.randn(64, 256, generator=gen) * 0.02).bfloat16().to(cuda_device)
    s = calibrated_quant.static_scales(w, 32)
    assert np.array_equal(s.cpu().view(torch.int16).numpy().view(np.uint16), g["signed_scales"])


@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("paired", [False, True])
def test_dp4a_packing_linear_against_oracle(cuda_device, interleaved, paired):
    dev = cuda_device
    n, k = 512, 1024
    packed, scales, w = _signed(5 + paired, n, k, dev)
    x = torch.randn(k, generator=torch.Generator().manual_seed(3)).bfloat16()
    if interleaved:
        packed = dp4a_packing.pack_interleaved(packed)
    y = dp4a_packing.linear(x.to(dev), packed, scales, interleaved=interleaved, paired=paired)
    ref = ops.linear(x.float().numpy(), w)
    if paired:
        ref = ops.silu_mul(ref)
    _check(y, ref, f"dp4a_packing.linear paired={paired} interleaved={interleaved}")
    y2 = dp4a_packing.linear(x.to(dev), packed, scales, interleaved=interleaved, paired=paired)  # cached operands
    assert torch.equal(y, y2)


def test_project_and_int4_dp4a_against_oracle(cuda_device):
    dev = cuda_device

    class Attention:
        pass
    m = Attention()
    m._quant_out, m._quant_out_scale, w = _signed(9, 256, 512, dev)
    m._dp4a_group = 32
    m._dp4a_packing = {"out": {"scheme": "prmt", "rows": 4, "warps": 2}}
    x = torch.randn(512, generator=torch.Generator().manual_seed(4)).bfloat16()
    ref = ops.linear(x.float().numpy(), w)
    _check(dp4a_packing.project(m, "out", x.to(dev)), ref, "project(out)")
    _check(int4_dp4a.int4_dp4a(x.to(dev), m._quant_out, m._quant_out_scale, group=32), ref, "int4_dp4a")


@pytest.mark.parametrize("fused", [False, True])
def test_norm_projection_against_oracle(cuda_device, fused):
    dev = cuda_device
    n2 = 512
    packed, scales, w = _signed(13 + fused, n2, 4096, dev)
    gen = torch.Generator().manual_seed(6)
    x = torch.randn(4096, generator=gen).bfloat16()
    r = torch.randn(4096, generator=gen).bfloat16()
    nw = (torch.randn(4096, generator=gen) * 0.02 + 1).bfloat16()
    out = dp4a_norm_projection.linear(x.to(dev), r.to(dev), nw.to(dev), 1e-6, packed, scales, fused=fused,
                                      rows=32 if fused else 8)
    summed, hn = ops.add_rmsnorm(x.float().numpy(), r.float().numpy(), nw.float().numpy(), 1e-6)
    ref = ops.linear(hn, w)
    if fused:
        ref = ops.silu_mul(ref)
        assert len(out) == 3 and out[2] is None
    assert np.array_equal(out[0].float().cpu().numpy(), summed)
    _check(out[1], ref, f"dp4a_norm_projection.linear fused={fused}")
