"""Batched causal prefill (``FastLLM.prefill``) on a B200.

* against the reference: the 2-layer model's 40-token prompt through the reference's
  ``MossTTSDelayModel`` (``tests/golden/prefill.npz``), last-row text logits over the full text
  head and 32 x 1024 audio logits;
* against the oracle's row-by-row causal pass on a 300-token prompt (three GEMM row tiles, the
  last partial): last-row logits, and every K/V cache row the prefill wrote;
* decode continues from the prefilled cache: the next decode step equals the one after the
  prompt was fed row by row through the decode step (ids except near-ties, hidden within bar).

All three projection modes run: resident bf16 copies from the bit-exact dequantization, the
same dequantized per call into a scratch, and the W4A16 tcgen05 GEMM.

Bars: the reference runs its prompt pass with bf16 matmul/attention outputs on the CPU, so the
logits are compared at 0.1 + 2e-2 |ref| with relative RMS <= 2% (the same bar pins the oracle
to that fixture); against the oracle, whose arithmetic this is up to fp32 summation order,
logits within 5e-2 + 2e-2 |ref| and cache rows within 2e-2 + 1e-2 |ref|.
"""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import model as omodel
from oracle.numerics import from_bf16_bits

from moss_tts._runtime import synthetic
from moss_tts._runtime.config import DecoderConfig, small_vocab
from moss_tts._runtime.engine import DecodeEngine
from moss_tts._runtime.llm import FastLLM
from moss_tts._runtime.weights import DecoderWeights

pytestmark = pytest.mark.gpu


def _host(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def _report(label, got, want, atol, rtol):
    want = np.asarray(want, np.float64).reshape(np.asarray(got).shape)
    err = np.abs(np.asarray(got, np.float64) - want)
    rms = np.sqrt(np.mean(err ** 2) / np.mean(want ** 2))
    print(f"{label}: max abs {err.max():.4g}, relative rms {rms:.3g}")
    return bool(np.all(err <= atol + rtol * np.abs(want))), rms


@pytest.fixture(scope="module")
def two_layer(cuda_device):
    dc = small_vocab(DecoderConfig(), vocab=2048, layers=2)
    host = synthetic.decoder_weights(dc, seed=7)
    return dc, host, DecoderWeights.from_host(dc, host, cuda_device)


@pytest.mark.parametrize("mode", ["bf16", "dequant", "w4"])
def test_prefill_matches_reference_model(two_layer, mode):
    dc, _, w = two_layer
    g = golden("prefill")
    llm = FastLLM(w, max_length=128, greedy=True)
    llm.prefill_mode = mode
    text, audio = llm.prefill(torch.from_numpy(g["ids"]))
    torch.cuda.synchronize()
    for label, got, want in (("prefill text logits", text, g["text"]), ("prefill audio logits", audio, g["audio"])):
        ok, rms = _report(label, _host(got), from_bf16_bits(want), 0.1, 2e-2)
        assert ok and rms <= 0.02, label
    assert int(llm.engine.status.item()) == 0


@pytest.mark.parametrize("mode", ["bf16", "dequant", "w4"])
def test_prefill_long_prompt_matches_oracle_and_decode_continues(two_layer, cuda_device, mode):
    dc, host, w = two_layer
    n = 300
    rng = np.random.Generator(np.random.PCG64(5))
    ids = np.full((1, n, 33), 1024, dtype=np.int64)
    ids[0, :, 0] = rng.integers(0, dc.vocab_size - 16, size=n)
    ids[0, :, 1:] = rng.integers(0, 1025, size=(n, 32))
    llm = FastLLM(w, max_length=384, greedy=True)
    llm.prefill_mode = mode
    text, audio = llm.prefill(torch.from_numpy(ids))
    text, audio = text.clone(), audio.clone()
    # a second prompt of this length replays the captured graph: the same bits
    again = llm.prefill(torch.from_numpy(ids))
    assert torch.equal(again[0], text) and torch.equal(again[1], audio)
    ref = omodel.Decoder(host, dc.as_dict(), max_length=384)
    rtext, raudio, _ = ref.prefill(ids[0])
    for label, got, want in (("long prefill text logits", text, rtext), ("long prefill audio logits", audio, raudio)):
        ok, _ = _report(label, _host(got), want, 5e-2, 2e-2)
        assert ok, label
    # every cache row the prefill wrote, both layers (layer 1's rows come from layer 0's outputs,
    # so they carry one layer of rounding differences: the multi-layer bar)
    kv = llm.engine.kv
    for layer, (atol, rtol) in enumerate(((2e-2, 1e-2), (5e-2, 2e-2))):
        for which, want in ((0, ref.k[layer]), (1, ref.v[layer])):
            ok, _ = _report(f"layer {layer} {'KV'[which]} rows 0..{n - 1}", _host(kv[layer, which, :, :n]),
                            want[:, :n], atol, rtol)
            assert ok
    # the decode step at position n from the prefilled cache vs the row-by-row path
    chain = DecodeEngine(w, max_length=384)
    for t in range(n):
        chain.step(torch.from_numpy(ids[0, t]), t, 1, -1)
    nxt = np.full(33, 7, dtype=np.int64)
    nxt[0] = dc.audio_assistant_gen_slot_token_id
    a = llm.step(torch.from_numpy(nxt).view(1, 1, 33), n, 1, -1).reshape(-1).cpu()
    b = chain.step(torch.from_numpy(nxt), n, 1, -1).reshape(-1).cpu()
    ok, _ = _report("decode after prefill vs row-by-row (hidden)", _host(llm.engine.hidden), _host(chain.hidden),
                    5e-2, 2e-2)
    assert ok
    differ = int((a != b).sum())
    print(f"decode after prefill: {differ} of 33 ids differ from the row-by-row path")
    assert differ <= 2
    assert int(llm.engine.status.item()) == 0


@pytest.mark.parametrize("start,n", [(0, 512), (100, 150), (0, 1), (37, 64)])
def test_prefill_attention_kernels_agree_with_oracle(cuda_device, start, n):
    """The tensor-core prefill attention (default) and the CUDA-core kernel (flags bit 1) against
    the oracle's causal attention (fp32 softmax, the reference's 1/sqrt(128) scale) on random
    q / cache rows: a cached prefix (start > 0), a partial last 64-row tile, a single row. The
    tensor-core kernel rounds the probabilities to bf16 before P V: within 2e-2 + 1e-2 |ref|."""
    from moss_tts._runtime import native
    nq, nkv, L = 32, 8, 640
    g = torch.Generator(device=cuda_device).manual_seed(start + n)
    q = torch.randn(n, nq, 128, device=cuda_device, generator=g).bfloat16()
    k = torch.randn(nkv, L, 128, device=cuda_device, generator=g).bfloat16()
    v = torch.randn(nkv, L, 128, device=cuda_device, generator=g).bfloat16()
    outs = []
    for flags in (0, 2):
        o = torch.full((n, nq * 128), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        native.call("mt_prefill_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), start, n, nq, nkv,
                    L, flags, torch.cuda.current_stream(cuda_device).cuda_stream)
        outs.append(_host(o))
    qh, kh, vh = _host(q), _host(k), _host(v)
    ref = np.zeros((n, nq, 128))
    for h in range(nq):
        kk, vv = kh[h // 4], vh[h // 4]
        for t in range(n):
            lg = kk[: start + t + 1] @ qh[t, h] * (1 / np.sqrt(128))
            p = np.exp(lg - lg.max())
            ref[t, h] = (p / p.sum()) @ vv[: start + t + 1]
    for name, got in zip(("tensor-core", "CUDA-core"), outs):
        ok, _ = _report(f"prefill attention {name} start {start} n {n}", got, ref.reshape(n, -1), 2e-2, 1e-2)
        assert ok, name
