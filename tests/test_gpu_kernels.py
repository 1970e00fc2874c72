"""Kernel parity on a B200: each C-ABI entry point against the oracle and the golden fixtures.

Bars (from the north star): dequantized bf16 weights bit-exact; projections and layer
outputs within max-abs 2e-2 / relative 1e-2 of the oracle (bf16 in, fp32 accumulate);
integer/index outputs (embedding sums of bf16 adds, cache rows, token ids) exact.
"""
import itertools
import zlib

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import ops, quant
from oracle.numerics import bf16_bits, from_bf16_bits

from moss_tts._runtime import kernels, quantized, synthetic

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def dev_bf16(bits, device):
    a = np.ascontiguousarray(bits, dtype=np.uint16)
    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)


def host_bits(t):
    return t.detach().to("cpu").contiguous().view(torch.int16).numpy().view(np.uint16)


def close(y_bits, ref, atol=ATOL, rtol=RTOL):
    y = from_bf16_bits(y_bits).astype(np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(y - ref)
    bad = err > atol + rtol * np.abs(ref)
    print(f"max abs err {err.max():.4g} (bar {atol:g} + {rtol:g} |ref|)")
    assert not bad.any(), f"max err {err.max():.4g} at {np.argmax(err)}; {bad.sum()} outside tolerance"
    return err.max()


def upload_w4(p, device):
    return (torch.from_numpy(np.ascontiguousarray(p["qweight"])).to(device),
            dev_bf16(p["scales"], device),
            None if p.get("qzeros") is None else torch.from_numpy(np.ascontiguousarray(p["qzeros"])).to(device))


# ------------------------------------------------------------------ dequantization
def test_dequant_bit_exact_zero_point(cuda_device):
    g = golden("quant")
    qw, sc, qz = upload_w4({"qweight": g["zp_qweight"], "scales": g["zp_scales"], "qzeros": g["zp_qzeros"]},
                           cuda_device)
    w = quantized.dequantize_packed(qw, sc, qz)
    assert np.array_equal(host_bits(w), g["zp_dequant"])


def test_dequant_bit_exact_reference_signed_export(cuda_device):
    g = golden("quant")
    qw = torch.from_numpy(quant.signed_to_unsigned(g["signed_packed"])).to(cuda_device)
    w = quantized.dequantize_packed(qw, dev_bf16(g["signed_scales"], cuda_device), None)
    assert np.array_equal(host_bits(w), g["signed_dequant"])


def test_dequant_config0_checksum(cuda_device):
    g = golden("quant")
    rng = np.random.Generator(np.random.PCG64(0))
    big = synthetic.quantized(rng, 12288, 4096, 32, True)
    w = quantized.dequantize_packed(*upload_w4(big, cuda_device))
    assert zlib.crc32(host_bits(w).tobytes()) == int(g["config0_dequant_crc32"][0])


# ------------------------------------------------------------------ W4A16 linear
def test_w4a16_config0_matches_reference(cuda_device):
    g = golden("linear")
    rng = np.random.Generator(np.random.PCG64(0))
    big = synthetic.quantized(rng, 12288, 4096, 32, True)
    x = dev_bf16(synthetic.activation(1, (1, 4096)), cuda_device)
    y = quantized.linear(x, *upload_w4(big, cuda_device))
    close(host_bits(y), from_bf16_bits(g["config0_y"]))
    # and against the oracle's dequantize-then-matmul
    w = quant.dequantize_w4(big["qweight"], big["scales"], big["qzeros"])
    close(host_bits(y), ops.linear(from_bf16_bits(synthetic.activation(1, (1, 4096))), w))


@pytest.mark.parametrize("b", [1, 3, 8])
def test_w4a16_small_batches(cuda_device, b):
    g = golden("linear")
    p = {"qweight": g["small_qweight"], "scales": g["small_scales"], "qzeros": g["small_qzeros"]}
    y = quantized.linear(dev_bf16(g[f"small_x{b}"], cuda_device), *upload_w4(p, cuda_device))
    close(host_bits(y), from_bf16_bits(g[f"small_y{b}"]))


@pytest.mark.parametrize("n,k,zeros", [(4096, 12288, True), (512, 512, True), (4096, 1536, True),
                                       (6144, 4096, False), (64, 128, True), (1024, 3072, False)])
def test_w4a16_shapes_against_oracle(cuda_device, n, k, zeros):
    rng = np.random.Generator(np.random.PCG64(n * 7 + k))
    p = synthetic.quantized(rng, n, k, 32, zeros)
    xb = synthetic.activation(n + k, (1, k))
    y = quantized.linear(dev_bf16(xb, cuda_device), *upload_w4(p, cuda_device))
    ref = ops.linear(from_bf16_bits(xb), quant.dequantize_w4(p["qweight"], p["scales"], p["qzeros"]))
    close(host_bits(y), ref)


@pytest.mark.parametrize("b", [1, 2, 5, 8])
def test_w4a16_paired_silu_and_norm(cuda_device, b):
    rng = np.random.Generator(np.random.PCG64(90 + b))
    p = synthetic.quantized(rng, 2 * 1536, 4096, 32, True)
    x = synthetic.activation(91, (b, 4096))
    r = synthetic.activation(92, (b, 4096))
    nw = synthetic.activation(93, (4096,), 0.02)
    nw = bf16_bits(from_bf16_bits(nw) + 1.0)
    w = quant.dequantize_w4(p["qweight"], p["scales"], p["qzeros"])
    # add + norm + paired projection
    summed, y = quantized.norm_linear(dev_bf16(x, cuda_device), dev_bf16(r, cuda_device),
                                      dev_bf16(nw, cuda_device), 1e-6, *upload_w4(p, cuda_device),
                                      paired=True)
    s_ref, h_ref = ops.add_rmsnorm(from_bf16_bits(x), from_bf16_bits(r), from_bf16_bits(nw), 1e-6)
    assert np.array_equal(host_bits(summed), bf16_bits(s_ref))
    close(host_bits(y), ops.silu_mul(ops.linear(h_ref, w)))
    # norm only, unpaired
    s2, y2 = quantized.norm_linear(dev_bf16(x, cuda_device), None, dev_bf16(nw, cuda_device), 1e-6,
                                   *upload_w4(p, cuda_device))
    close(host_bits(y2), ops.linear(ops.rmsnorm(from_bf16_bits(x), from_bf16_bits(nw), 1e-6), w))


def test_mlp_config1(cuda_device):
    """Config 1: RMSNorm -> gate/up -> SiLU*up -> down at batch 1, 4, 8 vs the HF reference."""
    g = golden("mlp")
    rng = np.random.Generator(np.random.PCG64(71))
    gu = synthetic.quantized(rng, 2 * 12288, 4096, 32, True)
    dn = synthetic.quantized(rng, 4096, 12288, 32, True)
    nw = synthetic._normal_bf16(rng, (4096,), 0.02, 1.0)
    gu_d, dn_d = upload_w4(gu, cuda_device), upload_w4(dn, cuda_device)
    for b in (1, 4, 8):
        x = dev_bf16(synthetic.activation(80 + b, (b, 4096)), cuda_device)
        _, mid = quantized.norm_linear(x, None, dev_bf16(nw, cuda_device), 1e-6, *gu_d, paired=True)
        y = quantized.linear(mid, *dn_d)
        close(host_bits(y), from_bf16_bits(g[f"b{b}_y"]))


# ------------------------------------------------------------------ small operators
def test_rmsnorm_add_rmsnorm(cuda_device):
    g = golden("ops")
    x, r, w = (dev_bf16(g[k], cuda_device) for k in ("norm_x", "norm_r", "norm_w"))
    y = kernels.rmsnorm(x, w, 1e-6)
    assert np.mean(host_bits(y) == g["rmsnorm_y"]) > 0.999
    close(host_bits(y), from_bf16_bits(g["rmsnorm_y"]), 1e-2, 8e-3)
    s, y2 = kernels.add_rmsnorm(x, r, w, 1e-6)
    assert np.array_equal(host_bits(s), g["add_sum"])
    assert np.mean(host_bits(y2) == g["add_y"]) > 0.999


def test_silu_mul(cuda_device):
    g = golden("ops")
    y = kernels.silu_mul(dev_bf16(g["silu_in"], cuda_device))
    assert np.mean(host_bits(y) == g["silu_out"]) > 0.995
    close(host_bits(y), from_bf16_bits(g["silu_out"]))
    # the 8-wide kernel (n % 8 == 0) and the scalar one (n = 1004): the same bits as the oracle but
    # where expf and numpy's exp round differently before the bf16 rounding
    for rows, n in ((37, 12288), (3, 1004)):
        xb = synthetic.activation(rows + n, (rows, 2 * n), 2.0)
        y = host_bits(kernels.silu_mul(dev_bf16(xb, cuda_device)))
        ref = ops.silu_mul(from_bf16_bits(xb))
        assert np.mean(y == bf16_bits(ref)) > 0.995, (rows, n)
        close(y, ref)


def test_embedding_sum_exact(cuda_device):
    g = golden("ops")
    rng = np.random.Generator(np.random.PCG64(47))
    text = dev_bf16(synthetic._normal_bf16(rng, (2048, 4096)), cuda_device)
    audio = dev_bf16(synthetic._normal_bf16(rng, (32, 1025, 4096)), cuda_device)
    ids = torch.from_numpy(g["emb_ids"]).to(cuda_device)
    y = kernels.embedding_sum(ids, text, audio)
    assert np.array_equal(host_bits(y), g["emb_out"])


def test_linear_decode_bf16(cuda_device):
    rng = np.random.Generator(np.random.PCG64(5))
    w = synthetic._normal_bf16(rng, (1030 // 2 * 2 - 2, 4096))
    for b in (1, 3):
        x = synthetic.activation(6 + b, (b, 4096))
        y = kernels.linear_decode(dev_bf16(x, cuda_device), dev_bf16(w, cuda_device))
        close(host_bits(y), ops.linear(from_bf16_bits(x), from_bf16_bits(w)))


@pytest.mark.parametrize("n,k,paired,zeros,batch", [
    (6144, 4096, False, True, 16), (24576, 4096, True, True, 32), (4096, 12288, False, True, 64),
    (4096, 4096, False, False, 48), (768, 4096, False, True, 9), (3072, 4096, True, False, 64),
    (4096, 512, False, True, 128), (256, 256, True, True, 17), (4096, 1536, False, True, 33)])
def test_tcgen05_gemm_matches_oracle(cuda_device, n, k, paired, zeros, batch):
    """Batched W4A16 projection on the tcgen05 tensor cores: oracle parity (dequantise then
    bf16 x bf16 with fp32 accumulation), split-K tickets back to zero, repeat calls bitwise
    equal, ragged batches (padded MMA columns), with and without zero points, fused pair."""
    from moss_tts._runtime import native
    rng = np.random.Generator(np.random.PCG64(n + 7 * k + batch))
    p = synthetic.quantized(rng, n, k, 32, zeros)
    qw, sc, qz = upload_w4(p, cuda_device)
    xb = synthetic.activation(31 + batch, (batch, k))
    x = dev_bf16(xb, cuda_device)
    mode = native.LINEAR_PAIRED if paired else 0
    nbytes = native.w4a16_gemm_workspace(batch, n, k, mode)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    n_out = n // 2 if paired else n
    outs = []
    for flags in (0, 0, 1):
        y = torch.empty((batch, n_out), device=cuda_device, dtype=torch.bfloat16)
        native.call("mt_w4a16_gemm", x.data_ptr(), qw.data_ptr(), sc.data_ptr(), native.ptr(qz), y.data_ptr(),
                    batch, n, k, mode, ws.data_ptr(), flags, torch.cuda.current_stream().cuda_stream)
        outs.append(host_bits(y))
    torch.cuda.synchronize()
    assert native.error_word(clear=True) == 0
    assert int(ws[:16384].view(torch.int32).abs().sum()) == 0
    ref = ops.linear(from_bf16_bits(xb), quant.dequantize_w4(p["qweight"], p["scales"], p["qzeros"]))
    if paired:
        ref = ops.silu_mul(ref)
    close(outs[0], ref)
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


@pytest.mark.parametrize("n,k,paired,zeros,batch", [
    (24576, 4096, True, True, 32), (4096, 12288, False, True, 16), (768, 4096, False, False, 9),
    (4096, 1536, False, True, 64), (256, 256, True, True, 17)])
def test_tcgen05_gemm_packed_layout_matches_gptq_layout(cuda_device, n, k, paired, zeros, batch):
    """The load-time packed layout gives bitwise the same results as the GPTQ layout (same
    arithmetic, different staging), and both match the oracle."""
    from moss_tts._runtime import native
    rng = np.random.Generator(np.random.PCG64(3 * n + k + batch))
    p = synthetic.quantized(rng, n, k, 32, zeros)
    qw, sc, qz = upload_w4(p, cuda_device)
    mode = native.LINEAR_PAIRED if paired else 0
    packed = torch.empty(native.w4a16_gemm_pack_size(n, k, mode), dtype=torch.uint8, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    native.call("mt_w4a16_gemm_pack", qw.data_ptr(), sc.data_ptr(), native.ptr(qz), n, k, mode, packed.data_ptr(), s)
    xb = synthetic.activation(61 + batch, (batch, k))
    x = dev_bf16(xb, cuda_device)
    ws = torch.zeros(native.w4a16_gemm_workspace(batch, n, k, mode), dtype=torch.uint8, device=cuda_device)
    n_out = n // 2 if paired else n
    y_gptq = torch.empty((batch, n_out), device=cuda_device, dtype=torch.bfloat16)
    native.call("mt_w4a16_gemm", x.data_ptr(), qw.data_ptr(), sc.data_ptr(), native.ptr(qz), y_gptq.data_ptr(),
                batch, n, k, mode, ws.data_ptr(), 0, s)
    outs = []
    for flags in (0, 1):
        y = torch.empty_like(y_gptq)
        native.call("mt_w4a16_gemm_packed", x.data_ptr(), packed.data_ptr(), y.data_ptr(), batch, n, k, mode,
                    ws.data_ptr(), flags, s)
        outs.append(host_bits(y))
    torch.cuda.synchronize()
    assert native.error_word(clear=True) == 0
    assert np.array_equal(outs[0], host_bits(y_gptq)) and np.array_equal(outs[0], outs[1])
    ref = ops.linear(from_bf16_bits(xb), quant.dequantize_w4(p["qweight"], p["scales"], p["qzeros"]))
    close(outs[0], ops.silu_mul(ref) if paired else ref)
    assert int(ws[:16384].view(torch.int32).abs().sum()) == 0


def test_tcgen05_gemm_shapes_share_one_workspace(cuda_device):
    """Projections of different shapes interleaved on one workspace (as the batched decode step
    uses it): every call still matches the oracle."""
    from moss_tts._runtime import native
    batch = 24
    shapes = [(6144, 4096, False), (4096, 4096, False), (24576, 4096, True), (4096, 12288, False)]
    rng = np.random.Generator(np.random.PCG64(77))
    mats = [(synthetic.quantized(rng, n, k, 32, True), n, k, paired) for n, k, paired in shapes]
    ws = torch.zeros(max(native.w4a16_gemm_workspace(batch, n, k, 4 if pr else 0) for _, n, k, pr in mats),
                     dtype=torch.uint8, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    for rep in range(2):
        for i, (p, n, k, paired) in enumerate(mats):
            qw, sc, qz = upload_w4(p, cuda_device)
            xb = synthetic.activation(50 + i, (batch, k))
            n_out = n // 2 if paired else n
            y = torch.empty((batch, n_out), device=cuda_device, dtype=torch.bfloat16)
            native.call("mt_w4a16_gemm", dev_bf16(xb, cuda_device).data_ptr(), qw.data_ptr(), sc.data_ptr(),
                        qz.data_ptr(), y.data_ptr(), batch, n, k, 4 if paired else 0, ws.data_ptr(), 1, s)
            ref = ops.linear(from_bf16_bits(xb), quant.dequantize_w4(p["qweight"], p["scales"], p["qzeros"]))
            close(host_bits(y), ops.silu_mul(ref) if paired else ref)
    assert int(ws[:16384].view(torch.int32).abs().sum()) == 0


def test_quantized_linear_routes_large_batches_to_tcgen05(cuda_device):
    """quantized.linear keeps the reference signature for 9..128 rows (tcgen05 GEMM)."""
    rng = np.random.Generator(np.random.PCG64(91))
    p = synthetic.quantized(rng, 1024, 1024, 32, True)
    qw, sc, qz = upload_w4(p, cuda_device)
    xb = synthetic.activation(92, (2, 12, 1024))
    y = quantized.linear(dev_bf16(xb, cuda_device), qw, sc, qz)
    assert y.shape == (2, 12, 1024)
    ref = ops.linear(from_bf16_bits(xb).reshape(24, 1024), quant.dequantize_w4(p["qweight"], p["scales"], p["qzeros"]))
    close(host_bits(y).reshape(24, 1024), ref)


@pytest.mark.parametrize("n,k,mode", [(6144, 4096, 1), (4096, 4096, 3), (24576, 4096, 7), (4096, 12288, 0),
                                      (4096, 6144, 0), (4096, 1536, 0), (3072, 4096, 5), (4096, 512, 0),
                                      (1032, 2048, 4), (80000, 512, 0), (20, 256, 1)])
def test_bf16_linear_batch1_matches_oracle(cuda_device, n, k, mode):
    """Batch-1 bf16 GEMV streamed through shared memory (every (rows per stage, chunks per thread)
    variant, each prologue mode, ragged last stages, fewer rows than SMs, and a matrix large
    enough to need two launches): oracle parity, summed output exact, PDL and repeat calls
    bitwise equal, and agreement with the register-pipelined kernel (flag bit 1)."""
    from moss_tts._runtime import native
    rng = np.random.Generator(np.random.PCG64(7 * n + k + mode))
    wb = synthetic._normal_bf16(rng, (n, k))
    xb, rb = synthetic.activation(21 + n, (1, k)), synthetic.activation(22 + n, (1, k))
    nw = bf16_bits(from_bf16_bits(synthetic.activation(23, (k,), 0.02)) + 1.0)
    x, r, w, g = (dev_bf16(a, cuda_device) for a in (xb, rb, wb, nw))
    n_out = n // 2 if mode & 4 else n
    s = torch.cuda.current_stream().cuda_stream

    def run(flags):
        y = torch.empty((1, n_out), device=cuda_device, dtype=torch.bfloat16)
        summed = torch.zeros_like(x)
        native.call("mt_bf16_linear", x.data_ptr(), r.data_ptr() if mode & 2 else None,
                    g.data_ptr() if mode & 1 else None, 1e-6, summed.data_ptr() if mode & 2 else None,
                    w.data_ptr(), y.data_ptr(), 1, n, k, mode, flags, s)
        return host_bits(y), host_bits(summed)

    y0, s0 = run(0)
    y1, _ = run(0)
    ypdl, _ = run(1)
    yreg, _ = run(2)
    xin = from_bf16_bits(xb)
    if mode & 2:
        s_ref, h = ops.add_rmsnorm(xin, from_bf16_bits(rb), from_bf16_bits(nw), 1e-6)
        assert np.array_equal(s0, bf16_bits(s_ref))
    elif mode & 1:
        h = ops.rmsnorm(xin, from_bf16_bits(nw), 1e-6)
    else:
        h = xin
    ref = ops.linear(h, from_bf16_bits(wb))
    if mode & 4:
        ref = ops.silu_mul(ref)
    close(y0, ref)
    close(yreg, ref)
    assert np.array_equal(y0, y1) and np.array_equal(y0, ypdl)


# ------------------------------------------------------------------ attention
class _Cache:
    class _Layer:
        def __init__(self, k, v):
            self.keys, self.values = k, v

    def __init__(self, k, v):
        self.layers = [self._Layer(k, v)]


def _rope(device, length):
    from moss_tts._runtime.engine import rope_tables
    cos, sin = rope_tables(length)
    return cos.to(device), sin.to(device)


def test_rope_tables_match_transformers():
    """Bit-exact against transformers' Qwen3 rotary embedding evaluated in this process (both
    use torch's fp32 pow / cos / sin on this host's CPU, whose last bits can differ between
    CPUs); against the fixture made on another host, at most one bf16 ulp anywhere."""
    from transformers import Qwen3Config
    from transformers.models.qwen3 import modeling_qwen3
    from moss_tts._runtime.engine import rope_tables
    g = golden("ops")
    cos, sin = rope_tables(4096)
    pos = torch.from_numpy(g["rope_positions"])
    cfg = Qwen3Config(hidden_size=4096, intermediate_size=12288, num_hidden_layers=1, num_attention_heads=32,
                      num_key_value_heads=8, head_dim=128, vocab_size=2048, rms_norm_eps=1e-6,
                      rope_parameters={"rope_type": "default", "rope_theta": 1e6}, max_position_embeddings=8192)
    c_ref, s_ref = modeling_qwen3.Qwen3RotaryEmbedding(cfg)(torch.zeros(1, dtype=torch.bfloat16), pos[None])
    assert torch.equal(cos[pos], c_ref[0]) and torch.equal(sin[pos], s_ref[0])
    for mine, fixture in ((cos[pos], g["rope_cos"]), (sin[pos], g["rope_sin"])):
        ulps = np.abs(mine.view(torch.int16).numpy().astype(np.int32) - fixture.view(np.int16).astype(np.int32))
        assert ulps.max() <= 1, ulps.max()


@pytest.mark.parametrize("ctx", [0, 1, 31, 96, 777, 2048, 4095])
def test_attention_decode_against_oracle(cuda_device, ctx):
    L = max(ctx + 1, 128)
    g = golden("ops")
    kc = synthetic.activation(300 + ctx, (1, 8, L, 128))
    vc = synthetic.activation(400 + ctx, (1, 8, L, 128))
    qkv = synthetic.activation(500 + ctx, (6144,))
    qn, kn = g["rope_qn"], g["rope_kn"]
    cos, sin = _rope(cuda_device, L)
    kd, vd = dev_bf16(kc, cuda_device), dev_bf16(vc, cuda_device)
    pos = torch.tensor([ctx], device=cuda_device)
    out = kernels.qk_rope_decode(dev_bf16(qkv, cuda_device), dev_bf16(qn, cuda_device),
                                 dev_bf16(kn, cuda_device), cos, sin, _Cache(kd, vd), 0, pos, 1e-6)
    c_ref, s_ref = ops.rope_table([ctx])
    q, krow, vrow = ops.qk_rope(from_bf16_bits(qkv), from_bf16_bits(qn), from_bf16_bits(kn),
                                c_ref[0], s_ref[0], 1e-6)
    kf, vf = from_bf16_bits(kc)[0].copy(), from_bf16_bits(vc)[0].copy()
    kf[:, ctx], vf[:, ctx] = krow, vrow
    # cache rows written by the kernel equal the oracle's rows exactly (bf16 rounding points match)
    assert np.mean(host_bits(kd)[0, :, ctx] == bf16_bits(krow)) > 0.995
    assert np.array_equal(host_bits(vd)[0, :, ctx], bf16_bits(vrow))
    ref = ops.attention_decode(q, kf, vf, ctx)
    close(host_bits(out).reshape(-1), ref)
    # rows other than `ctx` are untouched
    assert np.array_equal(np.delete(host_bits(kd)[0], ctx, axis=1), np.delete(kc[0], ctx, axis=1))


def test_qk_norm_rope_matches_transformers(cuda_device):
    g = golden("ops")
    L = 128
    cos, sin = _rope(cuda_device, L)
    kd = torch.zeros((1, 8, L, 128), device=cuda_device, dtype=torch.bfloat16)
    vd = torch.zeros_like(kd)
    qo = torch.empty((32, 128), device=cuda_device, dtype=torch.bfloat16)
    from moss_tts._runtime import native
    pos = torch.tensor([77], device=cuda_device)
    qkv = dev_bf16(g["rope_qkv"], cuda_device)
    qn, kn = dev_bf16(g["rope_qn"], cuda_device), dev_bf16(g["rope_kn"], cuda_device)  # keep alive
    native.call("mt_qk_rope_kv", qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), cos.data_ptr(),
                sin.data_ptr(), pos.data_ptr(),
                qo.data_ptr(), kd.data_ptr(), vd.data_ptr(), 1, 32, 8, L, 1e-6, None, 0,
                torch.cuda.current_stream().cuda_stream)
    assert np.mean(host_bits(qo) == g["rope_q"]) > 0.995
    close(host_bits(qo), from_bf16_bits(g["rope_q"]))
    close(host_bits(kd)[0, :, 77], from_bf16_bits(g["rope_k"]))


@pytest.mark.parametrize("flags", [0, 2, 1])
def test_attention_ragged_batch(cuda_device, flags):
    """Config 4 shape: several sequences with different live lengths in one launch, through the
    cluster kernel (default), the split-K kernel (flags bit 1) and with PDL (bit 0)."""
    from moss_tts._runtime import native
    g = golden("ops")
    lens = [256, 1000, 4095, 3]
    B, L = len(lens), 4096
    kc = synthetic.activation(700, (B, 8, L, 128))
    vc = synthetic.activation(701, (B, 8, L, 128))
    qkv = synthetic.activation(702, (B, 6144))
    cos, sin = _rope(cuda_device, L)
    kd, vd = dev_bf16(kc, cuda_device), dev_bf16(vc, cuda_device)
    pos = torch.tensor(lens, device=cuda_device)
    out = torch.empty((B, 4096), device=cuda_device, dtype=torch.bfloat16)
    splits = 20
    partial = torch.empty(B * 8 * splits * 4 * 128, device=cuda_device)
    lse = torch.empty(B * 8 * splits * 4, device=cuda_device)
    tickets = torch.zeros(B * 8, device=cuda_device, dtype=torch.int32)
    qn, kn = dev_bf16(g["rope_qn"], cuda_device), dev_bf16(g["rope_kn"], cuda_device)
    native.call("mt_attention_decode", dev_bf16(qkv, cuda_device).data_ptr(), qn.data_ptr(), kn.data_ptr(),
                cos.data_ptr(), sin.data_ptr(), pos.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(),
                partial.data_ptr(), lse.data_ptr(), tickets.data_ptr(), B, 32, 8, L, splits, 1e-6, None, flags,
                torch.cuda.current_stream().cuda_stream)
    assert int(tickets.abs().sum()) == 0
    c_all, s_all = ops.rope_table(lens)
    for b, p in enumerate(lens):
        q, krow, vrow = ops.qk_rope(from_bf16_bits(qkv[b]), from_bf16_bits(g["rope_qn"]),
                                    from_bf16_bits(g["rope_kn"]), c_all[b], s_all[b], 1e-6)
        kf, vf = from_bf16_bits(kc[b]).copy(), from_bf16_bits(vc[b]).copy()
        kf[:, p], vf[:, p] = krow, vrow
        close(host_bits(out[b]), ops.attention_decode(q, kf, vf, p))


@pytest.mark.parametrize("ctx,zeros", [(0, True), (95, True), (600, True), (2048, False), (4095, True)])
def test_attention_oproj_fused_against_oracle(cuda_device, ctx, zeros):
    """Attention with o_proj folded into its tail (mt_attention_oproj_decode): the attention
    output against the oracle as mt_attention_decode's, the projection against the oracle's
    o_proj of the oracle attention (GEMV bar), and against the unfused packed GEMV on the
    kernel's own attention output; repeat calls bitwise equal (the merge counters return to
    zero)."""
    from moss_tts._runtime import native
    L = max(ctx + 1, 128)
    g = golden("ops")
    kc = synthetic.activation(900 + ctx, (1, 8, L, 128))
    vc = synthetic.activation(901 + ctx, (1, 8, L, 128))
    qkv = synthetic.activation(902 + ctx, (6144,))
    rng = np.random.Generator(np.random.PCG64(903 + ctx))
    p = synthetic.quantized(rng, 4096, 4096, 32, zeros)
    qw, sc, qz = upload_w4(p, cuda_device)
    nbytes, _ = native.w4a16_packed_size(4096, 4096, qz is not None, 0)
    packed = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    native.call("mt_w4a16_pack", qw.data_ptr(), sc.data_ptr(), native.ptr(qz), 4096, 4096, 0, packed.data_ptr(), s)
    cos, sin = _rope(cuda_device, L)
    qn, kn = dev_bf16(g["rope_qn"], cuda_device), dev_bf16(g["rope_kn"], cuda_device)
    pos = torch.tensor([ctx], device=cuda_device)
    ws = torch.zeros(8 * 4096 * 4 + 64, dtype=torch.uint8, device=cuda_device)
    outs = []
    for flags in (0, 0, 1):
        kd, vd = dev_bf16(kc, cuda_device), dev_bf16(vc, cuda_device)
        att = torch.empty(4096, device=cuda_device, dtype=torch.bfloat16)
        proj = torch.empty(4096, device=cuda_device, dtype=torch.bfloat16)
        status = torch.zeros(1, device=cuda_device, dtype=torch.int32)
        rc = native.library().mt_attention_oproj_decode(
            dev_bf16(qkv, cuda_device).data_ptr(), qn.data_ptr(), kn.data_ptr(), cos.data_ptr(), sin.data_ptr(),
            pos.data_ptr(), kd.data_ptr(), vd.data_ptr(), att.data_ptr(), packed.data_ptr(), 1 if zeros else 0,
            proj.data_ptr(), 4096, ws.data_ptr(), 32, 8, L, 1e-6, status.data_ptr(), flags, s)
        assert rc == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        outs.append((host_bits(att), host_bits(proj), host_bits(kd), host_bits(vd)))
    assert int(ws[8 * 4096 * 4:].abs().sum()) == 0  # merge counters back at zero
    for o in outs[1:]:
        assert all(np.array_equal(x, y) for x, y in zip(outs[0], o))
    att_bits, proj_bits, kbits, vbits = outs[0]
    c_ref, s_ref = ops.rope_table([ctx])
    q, krow, vrow = ops.qk_rope(from_bf16_bits(qkv), from_bf16_bits(g["rope_qn"]), from_bf16_bits(g["rope_kn"]),
                                c_ref[0], s_ref[0], 1e-6)
    kf, vf = from_bf16_bits(kc)[0].copy(), from_bf16_bits(vc)[0].copy()
    kf[:, ctx], vf[:, ctx] = krow, vrow
    assert np.array_equal(vbits[0, :, ctx], bf16_bits(vrow))
    ref_att = ops.attention_decode(q, kf, vf, ctx)
    close(att_bits.reshape(-1), ref_att)
    wdq = quant.dequantize_w4(p["qweight"], p["scales"], p["qzeros"])
    close(proj_bits, ops.linear(from_bf16_bits(att_bits.reshape(-1)), wdq))
    # the unfused packed GEMV on the same attention output: same rows up to summation order
    y = torch.empty((1, 4096), device=cuda_device, dtype=torch.bfloat16)
    gws = torch.zeros(native.w4a16_packed_size(4096, 4096, qz is not None, 0)[1], dtype=torch.uint8,
                      device=cuda_device)
    native.call("mt_w4a16_linear_packed", dev_bf16(att_bits.reshape(1, -1), cuda_device).data_ptr(), None, None,
                1e-6, None, packed.data_ptr(), 1 if zeros else 0, y.data_ptr(), 4096, 4096, 0, gws.data_ptr(), 0, s)
    diff = np.abs(from_bf16_bits(host_bits(y)).reshape(-1) - from_bf16_bits(proj_bits))
    scale = np.abs(from_bf16_bits(proj_bits)) + 1e-3
    assert float((diff / scale).max()) <= 2 ** -7, float((diff / scale).max())


# ------------------------------------------------------------------ heads
def test_heads_greedy_against_oracle(cuda_device):
    from moss_tts._runtime import native
    rng = np.random.Generator(np.random.PCG64(123))
    H = 4096
    x, r = synthetic.activation(124, (H,)), synthetic.activation(125, (H,))
    nw = bf16_bits(from_bf16_bits(synthetic.activation(126, (H,), 0.02)) + 1.0)
    text_head = synthetic._normal_bf16(rng, (2, H))
    audio = synthetic._normal_bf16(rng, (32 * 1024, H))
    text_ids = torch.tensor([7, 9], device=cuda_device)
    best = torch.zeros(33, device=cuda_device, dtype=torch.int64)
    ticket = torch.zeros(1, device=cuda_device, dtype=torch.int32)
    tl = torch.empty(2, device=cuda_device, dtype=torch.bfloat16)
    al = torch.empty(32 * 1024, device=cuda_device, dtype=torch.bfloat16)
    hid = torch.empty(H, device=cuda_device, dtype=torch.bfloat16)
    nxt = torch.empty(33, device=cuda_device, dtype=torch.long)
    args = [dev_bf16(v, cuda_device) for v in (x, r, nw, text_head, audio)]
    _, h_ref = ops.add_rmsnorm(from_bf16_bits(x), from_bf16_bits(r), from_bf16_bits(nw), 1e-6)
    for (alen, delay), flags in itertools.product(((32, -1), (5, -1), (32, 3), (32, 32)), (0, 2)):
        a_len = torch.tensor([alen], device=cuda_device)
        d_len = torch.tensor([delay], device=cuda_device)
        nxt.fill_(-7)
        native.call("mt_heads_greedy", args[0].data_ptr(), args[1].data_ptr(), args[2].data_ptr(), 1e-6,
                    hid.data_ptr(), args[3].data_ptr(), args[4].data_ptr(), tl.data_ptr(), al.data_ptr(),
                    text_ids.data_ptr(), a_len.data_ptr(), d_len.data_ptr(), nxt.data_ptr(), best.data_ptr(),
                    ticket.data_ptr(), H, 2, 32, 1024, 0, 32, 99, 98, 1024, 1, flags,
                    torch.cuda.current_stream().cuda_stream)
        ids_ref, t_ref, a_ref = ops.heads_greedy(h_ref, from_bf16_bits(text_head), from_bf16_bits(audio),
                                                 np.array([7, 9]), alen, delay, 99, 98)
        assert np.mean(host_bits(hid) == bf16_bits(h_ref)) > 0.999
        close(host_bits(al), a_ref.reshape(-1))
        close(host_bits(tl), t_ref)
        got = nxt.cpu().numpy()
        # identical ids except on a near-tie (top-2 oracle gap within 2 bf16 ulps at |logit| < 8)
        a_ref = a_ref.reshape(32, 1024)
        top2 = np.sort(a_ref, axis=1)[:, -2:]
        for c in np.nonzero(got[1:] != ids_ref[1:])[0]:
            assert top2[c, 1] - top2[c, 0] <= 0.0625, (alen, delay, c)
        assert got[0] == ids_ref[0] or abs(float(t_ref[0] - t_ref[1])) <= 0.0625
        assert int(best.abs().sum()) == 0 and int(ticket.item()) == 0


# ------------------------------------------------------------------ packed tensor-core GEMV
def packed_linear(native, qw, sc, qz, n, k, mode, x, r, w, flags, device, ws=None, calls=1):
    """Pack once, then run mt_w4a16_linear_packed `calls` times; returns (y bits, summed bits, ws)."""
    nbytes, wbytes = native.w4a16_packed_size(n, k, qz is not None, mode & 4)
    packed = torch.empty(nbytes, dtype=torch.uint8, device=device)
    s = torch.cuda.current_stream().cuda_stream
    native.call("mt_w4a16_pack", qw.data_ptr(), sc.data_ptr(), native.ptr(qz), n, k, mode & 4,
                packed.data_ptr(), s)
    if ws is None:
        ws = torch.zeros(max(wbytes, 16), dtype=torch.uint8, device=device)
    n_out = n // 2 if mode & 4 else n
    outs = []
    for _ in range(calls):
        y = torch.empty((1, n_out), device=device, dtype=torch.bfloat16)
        summed = torch.empty_like(x)
        native.call("mt_w4a16_linear_packed", x.data_ptr(), r.data_ptr() if mode & 2 else None,
                    w.data_ptr() if mode & 1 else None, 1e-6, summed.data_ptr() if mode & 2 else None,
                    packed.data_ptr(), 1 if qz is not None else 0, y.data_ptr(), n, k, mode, ws.data_ptr(),
                    flags, s)
        outs.append((host_bits(y), host_bits(summed)))
    return outs, ws


@pytest.mark.parametrize("n,k,mode", [(6144, 4096, 1), (4096, 4096, 0), (24576, 4096, 7), (4096, 12288, 0),
                                      (12288, 4096, 0), (1536, 3072, 3), (2048, 1024, 4), (768, 6144, 0),
                                      (300, 1024, 4), (40, 512, 2 | 1), (26, 256, 4), (1000, 2048, 0)])
def test_packed_kernel_matches_oracle_and_register_kernel(cuda_device, n, k, mode):
    """Split-K tensor-core GEMV over the packed layout: oracle parity (fixed tolerance), agreement
    with the GPTQ-layout register kernel, PDL launch bitwise equal, repeat calls bitwise equal
    (the workspace tickets return to zero), ragged tiles and single-slice K."""
    from moss_tts._runtime import native
    rng = np.random.Generator(np.random.PCG64(n + 3 * k + mode))
    p = synthetic.quantized(rng, n, k, 32, mode != 0)
    qw, sc, qz = upload_w4(p, cuda_device)
    xb, rb = synthetic.activation(11 + n, (1, k)), synthetic.activation(12 + n, (1, k))
    nw = bf16_bits(from_bf16_bits(synthetic.activation(13, (k,), 0.02)) + 1.0)
    x, r, w = dev_bf16(xb, cuda_device), dev_bf16(rb, cuda_device), dev_bf16(nw, cuda_device)
    ws = torch.zeros(native.w4a16_packed_size(n, k, qz is not None, mode & 4)[1], dtype=torch.uint8,
                     device=cuda_device)
    ws[:1024 * 256].fill_(0x7F)  # partial-row slots hold stale data between calls; only tickets must be zero
    outs, ws = packed_linear(native, qw, sc, qz, n, k, mode, x, r, w, 0, cuda_device, ws=ws, calls=2)
    pdl, _ = packed_linear(native, qw, sc, qz, n, k, mode, x, r, w, 1, cuda_device, ws=ws)
    n_out = n // 2 if mode & 4 else n
    yreg = None
    if n % (8 if mode & 4 else 4) == 0:  # shapes the GPTQ-layout register kernel accepts
        yreg = torch.empty((1, n_out), device=cuda_device, dtype=torch.bfloat16)
        sreg = torch.empty_like(x)
        native.call("mt_w4a16_linear", x.data_ptr(), r.data_ptr() if mode & 2 else None,
                    w.data_ptr() if mode & 1 else None, 1e-6, sreg.data_ptr() if mode & 2 else None,
                    qw.data_ptr(), sc.data_ptr(), native.ptr(qz), yreg.data_ptr(), 1, n, k, 32, mode, 0,
                    torch.cuda.current_stream().cuda_stream)
    xin = from_bf16_bits(xb)
    if mode & 2:
        s_ref, h = ops.add_rmsnorm(xin, from_bf16_bits(rb), from_bf16_bits(nw), 1e-6)
        assert np.array_equal(outs[0][1], bf16_bits(s_ref))
    elif mode & 1:
        h = ops.rmsnorm(xin, from_bf16_bits(nw), 1e-6)
    else:
        h = xin
    ref = ops.linear(h, quant.dequantize_w4(p["qweight"], p["scales"], p["qzeros"]))
    if mode & 4:
        ref = ops.silu_mul(ref)
    close(outs[0][0], ref)
    # the two kernels sum in different orders; a one-ulp change of the bf16 gate can move
    # bf16(silu(gate)) * up by two ulps, so allow two
    if yreg is not None:
        a, b = from_bf16_bits(outs[0][0]), from_bf16_bits(host_bits(yreg))
        assert np.all(np.abs(a - b) <= 2.0 ** -6 * np.maximum(np.abs(a), np.abs(b)) + 2.0 ** -14)
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][0], pdl[0][0])
    # workspace: [1024 CTA boundaries][2][32] f32 partial rows, then [1024] i32 tickets
    assert int(ws[1024 * 256:].view(torch.int32).abs().sum()) == 0
    assert native.error_word() == 0


def test_packed_size_and_bad_arguments(cuda_device):
    from moss_tts._runtime import native
    assert native.w4a16_packed_size(4096, 4096, True, 0) == (256 * 16 * 2368, 1024 * (256 + 4))
    assert native.w4a16_packed_size(24576, 4096, False, 4) == (1536 * 16 * 2304, 1024 * (256 + 4))
    with pytest.raises(RuntimeError):
        native.w4a16_packed_size(64, 1000, True, 0)  # K not a multiple of 256
    with pytest.raises(RuntimeError):  # null workspace
        native.call("mt_w4a16_linear_packed", 16, None, None, 0.0, None, 16, 1, 16, 64, 1024, 0, None, 0, None)


def test_heads_tensor_parallel_shard_writes_only_its_codebooks(cuda_device):
    """A shard owning codebooks 8..15 and no text row: its ids there, zeros elsewhere."""
    from moss_tts._runtime import native
    rng = np.random.Generator(np.random.PCG64(321))
    H = 4096
    x, r = synthetic.activation(322, (H,)), synthetic.activation(323, (H,))
    nw = bf16_bits(from_bf16_bits(synthetic.activation(324, (H,), 0.02)) + 1.0)
    audio = synthetic._normal_bf16(rng, (8 * 1024, H))
    xs, rs, ws, au = (dev_bf16(v, cuda_device) for v in (x, r, nw, audio))
    best = torch.zeros(9, device=cuda_device, dtype=torch.int64)
    ticket = torch.zeros(1, device=cuda_device, dtype=torch.int32)
    al = torch.empty(8 * 1024, device=cuda_device, dtype=torch.bfloat16)
    nxt = torch.full((33,), -7, device=cuda_device, dtype=torch.long)
    a_len = torch.tensor([32], device=cuda_device)
    d_len = torch.tensor([-1], device=cuda_device)
    native.call("mt_heads_greedy", xs.data_ptr(), rs.data_ptr(), ws.data_ptr(), 1e-6, None, None, au.data_ptr(),
                None, al.data_ptr(), None, a_len.data_ptr(), d_len.data_ptr(), nxt.data_ptr(), best.data_ptr(),
                ticket.data_ptr(), H, 2, 8, 1024, 8, 32, 99, 98, 1024, 0, 0,
                torch.cuda.current_stream().cuda_stream)
    _, h_ref = ops.add_rmsnorm(from_bf16_bits(x), from_bf16_bits(r), from_bf16_bits(nw), 1e-6)
    logits = ops.linear(h_ref, from_bf16_bits(audio)).reshape(8, 1024)
    got = nxt.cpu().numpy()
    assert got[0] == 0 and np.all(got[1:9] == 0) and np.all(got[17:] == 0)
    top2 = np.sort(logits, axis=1)[:, -2:]
    want = np.argmax(logits, axis=1)
    for c in range(8):
        assert got[9 + c] == want[c] or top2[c, 1] - top2[c, 0] <= 0.0625
    assert int(best.abs().sum()) == 0 and int(ticket.item()) == 0


@pytest.mark.parametrize("n,k,mode,rows", [(6144, 4096, 1, 2), (24576, 4096, 7, 2), (4096, 12288, 0, 3),
                                           (4096, 4096, 3, 4), (300, 1024, 4, 2), (1000, 2048, 0, 5),
                                           (26, 256, 6 | 1, 2)])
def test_packed_rows_match_oracle_and_batch1(cuda_device, n, k, mode, rows):
    """mt_w4a16_linear_packed_rows: pairs of activation rows through the two-row kernel (one
    weight stream), an odd last row through the one-row kernel. Every row against the oracle
    (the fixed bar), against the batch-1 call on that row alone (same products, the per-group
    partial sums added in another order: two bf16 ulps), residual sums bit-exact; the PDL
    launch and a repeat call bitwise equal; the workspace tickets back to zero."""
    from moss_tts._runtime import native
    rng = np.random.Generator(np.random.PCG64(n + 5 * k + mode + rows))
    p = synthetic.quantized(rng, n, k, 32, mode != 0)
    qw, sc, qz = upload_w4(p, cuda_device)
    xb = synthetic.activation(21 + n, (rows, k))
    rb = synthetic.activation(22 + n, (rows, k))
    xb[rows - 1] = bf16_bits(from_bf16_bits(xb[rows - 1]) * 300.0)  # rows of very different scale
    nw = bf16_bits(from_bf16_bits(synthetic.activation(23, (k,), 0.02)) + 1.0)
    x, r, w = dev_bf16(xb, cuda_device), dev_bf16(rb, cuda_device), dev_bf16(nw, cuda_device)
    nbytes, wbytes = native.w4a16_packed_size(n, k, qz is not None, mode & 4)
    packed = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    native.call("mt_w4a16_pack", qw.data_ptr(), sc.data_ptr(), native.ptr(qz), n, k, mode & 4, packed.data_ptr(), s)
    ws = torch.zeros(wbytes, dtype=torch.uint8, device=cuda_device)
    n_out = n // 2 if mode & 4 else n
    zeros = 1 if qz is not None else 0

    def run(flags):
        y = torch.empty((rows, n_out), device=cuda_device, dtype=torch.bfloat16)
        summed = torch.empty_like(x)
        native.call("mt_w4a16_linear_packed_rows", x.data_ptr(), r.data_ptr() if mode & 2 else None,
                    w.data_ptr() if mode & 1 else None, 1e-6, summed.data_ptr() if mode & 2 else None,
                    packed.data_ptr(), zeros, y.data_ptr(), rows, n, k, mode, ws.data_ptr(), flags, s)
        return host_bits(y), host_bits(summed)

    y, summed = run(0)
    y2, _ = run(0)
    y3, _ = run(1)
    assert np.array_equal(y, y2) and np.array_equal(y, y3)
    wd = quant.dequantize_w4(p["qweight"], p["scales"], p["qzeros"])
    for i in range(rows):
        xin = from_bf16_bits(xb[i])
        if mode & 2:
            s_ref, h = ops.add_rmsnorm(xin, from_bf16_bits(rb[i]), from_bf16_bits(nw), 1e-6)
            assert np.array_equal(summed[i], bf16_bits(s_ref)), i
        elif mode & 1:
            h = ops.rmsnorm(xin, from_bf16_bits(nw), 1e-6)
        else:
            h = xin
        ref = ops.linear(h, wd)
        gu = None
        if mode & 4:
            gu = np.asarray(ref, np.float64)
            ref = ops.silu_mul(ref)
        scale = max(1.0, float(np.abs(ref).max()) / 8)  # the scaled row: the bar relative to its size
        if mode & 4:
            # y = bf16(bf16(silu(bf16 g)) * bf16 u): fp32 sums in another order can flip the bf16
            # g or u by one ulp, which moves y by |silu'(g) u| ulp(g) + |silu(g)| ulp(u) (plus
            # one ulp of y); with a large |u| that exceeds the fixed bar, so the bar adds it
            def ulp(v):
                return 2.0 ** (np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -100))) - 7)
            g, u = gu[: n_out], gu[n_out:]
            sg = 1.0 / (1.0 + np.exp(-g))
            flip = np.abs(sg * (1 + g * (1 - sg)) * u) * ulp(g) + np.abs(g * sg) * ulp(u) + ulp(ref)
            ref = np.asarray(ref, np.float64)
            err = np.abs(from_bf16_bits(y[i]).astype(np.float64) - ref)
            bar = ATOL * scale + RTOL * np.abs(ref) + flip
            print(f"row {i}: max abs err {err.max():.4g}, max err / bar {np.max(err / bar):.3g}")
            assert np.all(err <= bar), (i, err.max())
        else:
            close(y[i], ref, ATOL * scale)
        y1 = torch.empty((1, n_out), device=cuda_device, dtype=torch.bfloat16)
        native.call("mt_w4a16_linear_packed", x[i].data_ptr(), r[i].data_ptr() if mode & 2 else None,
                    w.data_ptr() if mode & 1 else None, 1e-6, None, packed.data_ptr(), zeros, y1.data_ptr(), n, k,
                    mode, ws.data_ptr(), 0, s)
        a, b = from_bf16_bits(y[i]), from_bf16_bits(host_bits(y1)[0])
        diff = np.abs(a.astype(np.float64) - b)
        if mode & 4:
            assert np.all(diff <= 2 * flip), i
        else:
            assert np.all(diff <= 2.0 ** -6 * np.maximum(np.abs(a), np.abs(b)) + 2.0 ** -14 * scale), i
    assert int(ws[1024 * 256:].view(torch.int32).abs().sum()) == 0
    assert native.error_word() == 0
