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


def _gptq_blocks_on_device(dev, weight, inputs, scales, actorder):
    """Drive ``mt_gptq_block`` and the oracle's column loop from the same block inputs (the
    oracle's Hessian set-up; the trailing update by the oracle's torch CPU matmul for both), and
    require identical codes, errors and updated blocks."""
    from moss_tts._runtime import native

    w, hinv, perm = quant.gptq_prepare(weight, inputs, 0.01, actorder)
    n, k = w.shape
    hinv_d = torch.from_numpy(hinv).to(dev)
    perm_d = torch.from_numpy(perm.astype(np.int64)).to(dev)
    scales_d = _bf16(scales, dev)
    codes_d = torch.zeros((n, k), dtype=torch.int8, device=dev)
    ref_codes = np.zeros((n, k), dtype=np.int8)
    for start in range(0, k, 128):
        chunk = np.ascontiguousarray(w[:, start:start + 128])
        chunk_d = torch.from_numpy(chunk).to(dev)
        err_d = torch.empty_like(chunk_d)
        native.call("mt_gptq_block", chunk_d.data_ptr(), err_d.data_ptr(), codes_d.data_ptr(), scales_d.data_ptr(),
                    hinv_d.data_ptr(), perm_d.data_ptr(), start, 128, n, k, 32, native.stream_of(chunk_d))
        codes, errors = quant.gptq_block(chunk, hinv, perm, scales, start, 32)
        ref_codes[:, perm[start:start + 128]] = codes
        assert np.array_equal(err_d.cpu().numpy().view(np.uint32), errors.view(np.uint32)), start
        assert np.array_equal(chunk_d.cpu().numpy().view(np.uint32), chunk.view(np.uint32)), start
        if start + 128 < k:
            w[:, start + 128:] -= (torch.from_numpy(errors) @ torch.from_numpy(
                np.ascontiguousarray(hinv[start:start + 128, start + 128:]))).numpy()
    assert np.array_equal(codes_d.cpu().numpy(), ref_codes)
    return ref_codes


def test_gptq_block_kernel_is_bit_exact(cuda_device):
    """The column-loop kernel against the oracle's (itself pinned to the reference's gptq): the
    reference fixture's two cases, then 300 rows (a ragged last 16-row CTA) x 512 columns."""
    g = golden("gptq")
    for name, actorder in (("act", True), ("plain", False)):
        codes = _gptq_blocks_on_device(cuda_device, g[f"{name}_weight"], g[f"{name}_inputs"],
                                       g[f"{name}_scales"], actorder)
        assert np.array_equal(codes, g[f"{name}_signed"]), name
    gen = torch.Generator().manual_seed(77)
    w = (torch.randn(300, 512, generator=gen) * 0.03).bfloat16()
    x = (torch.randn(256, 512, generator=gen) * torch.linspace(0.1, 3.0, 512)).numpy()
    wb = w.view(torch.int16).numpy().view(np.uint16)
    _gptq_blocks_on_device(cuda_device, wb, x, quant.static_scales(wb), True)


def test_gptq_on_device_against_reference(cuda_device):
    """Whole ``calibrated_quant.gptq`` on the device against the reference's codes. The Hessian
    factors and trailing updates come from device linear algebra, whose summation order differs
    from the CPU's, so a code can differ at a rounding near-tie: at most 1% of the codes, by
    one step, and the layer's calibration loss ``||(W - Q) X^T||`` within 1% of the reference's."""
    g = golden("gptq")
    for name, actorder in (("act", True), ("plain", False)):
        w = _bf16(g[f"{name}_weight"], cuda_device)
        x = torch.from_numpy(g[f"{name}_inputs"]).to(cuda_device)
        signed, scales = calibrated_quant.gptq(w, x, actorder=actorder)
        torch.cuda.synchronize()
        assert np.array_equal(scales.cpu().view(torch.int16).numpy().view(np.uint16), g[f"{name}_scales"])
        got, want = signed.cpu().numpy().astype(np.int32), g[f"{name}_signed"].astype(np.int32)
        differ = int((got != want).sum())
        wf, xf = from_bf16_bits(g[f"{name}_weight"]).astype(np.float64), g[f"{name}_inputs"].astype(np.float64)
        loss = [np.linalg.norm((wf - quant.dequantize_signed(c, g[f"{name}_scales"])) @ xf.T)
                for c in (got, want)]
        print(f"gptq {name}: {differ} of {got.size} codes differ, loss {loss[0]:.5g} vs reference {loss[1]:.5g}")
        assert differ <= got.size // 100 and np.abs(got - want).max() <= 1
        assert loss[0] <= loss[1] * 1.01


def test_gptq_layer_timing(cuda_device):
    """One 4096 x 4096 projection with 512 calibration rows: the 32 block launches and trailing
    updates, timed (the reference launches its column kernel 4096 times for this layer)."""
    gen = torch.Generator().manual_seed(3)
    w = (torch.randn(4096, 4096, generator=gen) * 0.02).bfloat16().to(cuda_device)
    x = torch.randn(512, 4096, generator=gen).to(cuda_device)
    calibrated_quant.gptq(w, x)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    signed, _ = calibrated_quant.gptq(w, x)
    t1.record()
    torch.cuda.synchronize()
    print(f"gptq 4096 x 4096, 512 calibration rows: {t0.elapsed_time(t1):.2f} ms")
    assert int(signed.abs().max()) <= 7
