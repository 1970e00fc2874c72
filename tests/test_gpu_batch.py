"""Batched decode on a B200: B sequences with ragged contexts in one step against the batch-1
engine run sequence by sequence on the same weights and caches.

Hidden states within max-abs 5e-2 / rel 2e-2; greedy ids identical except where the batch-1
engine's own top-two audio logits are a near-tie (a few bf16 ulps: the two paths sum in a
different order). Covers the tcgen05 GEMM path, the packed two-row GEMV (B = 2, and B = 3:
a pair plus one row), the GPTQ-layout GEMV (B <= 8 with both disabled), ragged positions, per-sequence delay masks, graph capture with the
device-side advance, and the batched greedy selection kernel against a host argmax.
"""
import numpy as np
import pytest
import torch

from oracle.numerics import from_bf16_bits

from moss_tts._runtime import native, synthetic
from moss_tts._runtime.batch_engine import BatchDecodeEngine
from moss_tts._runtime.config import DecoderConfig, small_vocab
from moss_tts._runtime.engine import DecodeEngine
from moss_tts._runtime.weights import DecoderWeights

pytestmark = pytest.mark.gpu
MAXLEN = 256


@pytest.fixture(scope="module")
def model(cuda_device):
    dc = small_vocab(DecoderConfig(), vocab=2048, layers=2)
    host = synthetic.decoder_weights(dc, seed=7)
    return dc, DecoderWeights.from_host(dc, host, cuda_device)


def host_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def near_tie_only(got, want, audio_logits, text_logits):
    bad = got != want
    if not bad.any():
        return 0
    if bad[0]:
        t = from_bf16_bits(host_bits(text_logits)).astype(np.float64)
        assert abs(t[0] - t[1]) <= 0.0625
    a = from_bf16_bits(host_bits(audio_logits)).astype(np.float64).reshape(32, -1)
    top2 = np.sort(a, axis=-1)[:, -2:]
    margins = (top2[:, 1] - top2[:, 0])[bad[1:]]
    assert np.all(margins <= 0.0625), margins
    return int(bad.sum())


@pytest.mark.parametrize("batch,gemm_min,packed", [(12, 2, True), (3, 2, True), (2, 5, True), (3, 5, True),
                                                   (3, 9, False)])
def test_batched_step_matches_batch1_engine(model, cuda_device, batch, gemm_min, packed):
    dc, w = model
    rng = np.random.Generator(np.random.PCG64(batch * 10 + gemm_min))
    pos = rng.integers(5, MAXLEN - 8, size=batch)
    eng = BatchDecodeEngine(w, batch, max_length=MAXLEN, gemm_min_batch=gemm_min, packed_gemv=packed)
    assert eng.rows_packed == (packed and batch < gemm_min)
    g = torch.Generator(device=cuda_device).manual_seed(batch)
    eng.kv.normal_(generator=g)
    singles = []
    for b in range(batch):
        e = DecodeEngine(w, max_length=MAXLEN)
        e.kv.copy_(eng.kv[:, :, b])
        singles.append(e)
    ids = np.zeros((batch, 33), dtype=np.int64)
    ids[:, 0] = dc.audio_assistant_gen_slot_token_id
    ids[:, 1:] = rng.integers(0, 1024, size=(batch, 32))
    alen = rng.integers(1, 33, size=batch)
    delay = np.where(rng.random(batch) < 0.5, -1, rng.integers(0, 33, size=batch))
    mismatched = 0
    for step in range(3):
        got = eng.step(torch.from_numpy(ids), torch.from_numpy(pos + step), torch.from_numpy(alen),
                       torch.from_numpy(delay)).cpu().numpy()
        nxt = np.zeros_like(ids)
        for b, e in enumerate(singles):
            want = e.step(torch.from_numpy(ids[b]), int(pos[b] + step), int(alen[b]), int(delay[b]))
            want = want.reshape(-1).cpu().numpy()
            h = from_bf16_bits(host_bits(eng.hidden[b])).astype(np.float64)
            ref = from_bf16_bits(host_bits(e.hidden)).astype(np.float64)
            assert np.all(np.abs(h - ref) <= 5e-2 + 2e-2 * np.abs(ref)), (step, b, np.abs(h - ref).max())
            mismatched += near_tie_only(got[b], want, e.audio_logits, e.text_logits)
            nxt[b] = want
        ids = nxt
    assert int(eng.status.item()) == 0 and native.error_word(clear=True) == 0
    assert mismatched <= 0.02 * 3 * batch * 33, mismatched


def test_batched_graph_advance_matches_eager(model, cuda_device):
    dc, w = model
    batch = 16
    rng = np.random.Generator(np.random.PCG64(5))
    pos = rng.integers(5, MAXLEN - 16, size=batch)
    a, b = BatchDecodeEngine(w, batch, max_length=MAXLEN), BatchDecodeEngine(w, batch, max_length=MAXLEN)
    g = torch.Generator(device=cuda_device).manual_seed(3)
    a.kv.normal_(generator=g)
    b.kv.copy_(a.kv)
    ids = np.zeros((batch, 33), dtype=np.int64)
    ids[:, 0] = dc.audio_assistant_gen_slot_token_id
    ids[:, 1:] = rng.integers(0, 1024, size=(batch, 32))
    alen, delay = np.ones(batch, dtype=np.int64), np.full(batch, -1, dtype=np.int64)
    for e in (a, b):
        e.set_inputs(torch.from_numpy(ids), torch.from_numpy(pos), torch.from_numpy(alen), torch.from_numpy(delay))
    b.capture(advance=True)
    for _ in range(6):
        a.run(advance=True)
        b.run(advance=True)
        assert torch.equal(a.ids, b.ids)
    assert torch.equal(a.position, b.position) and torch.equal(a.kv, b.kv)
    assert torch.equal(a.position.cpu(), torch.from_numpy(pos + 6))


def test_heads_select_matches_host_argmax(cuda_device):
    rng = np.random.Generator(np.random.PCG64(17))
    B, n_cb, V = 5, 8, 1024
    audio = torch.from_numpy(rng.standard_normal((B, n_cb * V)).astype(np.float32)).to(torch.bfloat16)
    audio[0, 7] = audio[0, 3] = 9.0  # first-index tie rule (sequence 0, codebook 0 = channel 8)
    text = torch.from_numpy(rng.standard_normal((B, 2)).astype(np.float32)).to(torch.bfloat16)
    text_ids = torch.tensor([151, 152], dtype=torch.long)
    alen = torch.tensor([33, 3, 33, 12, 1], dtype=torch.long)
    delay = torch.tensor([-1, -1, 0, 32, 5], dtype=torch.long)
    out = torch.full((B, 33), -7, dtype=torch.long, device=cuda_device)
    dev = [t.to(cuda_device) for t in (text, audio, text_ids, alen, delay)]
    native.call("mt_heads_select", dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), dev[3].data_ptr(),
                dev[4].data_ptr(), out.data_ptr(), B, 2, n_cb, V, 8, 32, 152, 153, 1024, 1, 0,
                torch.cuda.current_stream().cuda_stream)
    out = out.cpu().numpy()
    a = audio.float().numpy().reshape(B, n_cb, V)
    for b in range(B):
        tok = int(text_ids[int(np.argmax(text[b].float().numpy()))])
        if delay[b] >= 0:
            tok = 152
        if delay[b] == 32:
            tok = 153
        assert out[b, 0] == tok
        for ch in range(32):
            if not 8 <= ch < 16:
                assert out[b, 1 + ch] == 0  # another shard's codebook
                continue
            valid = ch < alen[b] and (delay[b] < 0 or ch >= delay[b])
            want = int(np.argmax(a[b, ch - 8])) if valid else 1024
            assert out[b, 1 + ch] == want, (b, ch)
    assert out[0, 1 + 8] == 3


def test_decode_advance_matches_reference_bookkeeping(cuda_device):
    """mt_decode_advance against first_audio_graph._advance's tensor arithmetic for a batch:
    ids fed back, positions and audio lengths + 1, delay counts started on the delay-slot text
    token and advanced once started."""
    B, n, slot = 6, 33, 153
    rng = np.random.Generator(np.random.PCG64(8))
    nxt = torch.from_numpy(rng.integers(0, 1000, size=(B, n))).long()
    nxt[[1, 3], 0] = slot
    ids = torch.from_numpy(rng.integers(0, 1000, size=(B, n))).long()
    pos = torch.tensor([5, 9, 100, 7, 0, 31])
    alen = torch.tensor([1, 2, 33, 4, 5, 6])
    delay = torch.tensor([-1, -1, 3, 0, 32, -1])
    control = torch.cat([ids.reshape(-1), pos, alen, delay]).to(cuda_device)
    native.call("mt_decode_advance", control.data_ptr(), nxt.to(cuda_device).data_ptr(), n, B, slot, 0,
                torch.cuda.current_stream().cuda_stream)
    got = control.cpu()
    d = torch.where((delay < 0) & (nxt[:, 0] == slot), torch.zeros_like(delay), delay)
    d = torch.where(d >= 0, d + 1, d)
    want = torch.cat([nxt.reshape(-1), pos + 1, alen + 1, d])
    assert torch.equal(got, want)
