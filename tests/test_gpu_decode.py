"""Full decode step on a B200 against the reference model and the oracle.

The model is the 2-layer, full-width (4096 hidden, 32/8 heads, 32 codebooks), 2048-vocab
random-init decoder of ``tests/golden/make_golden.py``; the fixture holds 64 teacher-forced
greedy steps of the reference's ``MossTTSDelayModel`` with ``FastLLM``'s head/mask logic.
Greedy ids must be identical except where the reference's own top-2 audio logits are a
near-tie (a few bf16 ulps); hidden states within max-abs 5e-2 / rel 2e-2.
"""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle.numerics import from_bf16_bits

from moss_tts._runtime import synthetic
from moss_tts._runtime.config import DecoderConfig, small_vocab
from moss_tts._runtime.engine import DecodeEngine
from moss_tts._runtime.weights import DecoderWeights

pytestmark = pytest.mark.gpu


def schedule(step):
    return min(step + 1, 32), (-1 if step < 30 else step - 30)


@pytest.fixture(scope="module")
def model(cuda_device):
    dc = small_vocab(DecoderConfig(), vocab=2048, layers=2)
    host = synthetic.decoder_weights(dc, seed=7)
    return dc, host, DecoderWeights.from_host(dc, host, cuda_device)


def host_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_teacher_forced_decode_matches_reference(model):
    dc, _, w = model
    g = golden("decode")
    eng = DecodeEngine(w, max_length=128)
    hs = list(g["hidden_steps"])
    mismatched = 0
    worst = 0.0
    for step in range(g["ids"].shape[0]):
        alen, delay = schedule(step)
        nxt = eng.step(torch.from_numpy(g["ids"][step]), step, alen, delay).reshape(-1).cpu().numpy()
        bad = nxt != g["next"][step]
        if bad.any():
            if bad[0]:  # text channel: the reference's two text logits must be a near-tie
                t = from_bf16_bits(g["text"][step])
                assert abs(float(t[0] - t[1])) <= 0.0625, step
            margins = g["audio_top2"][step][bad[1:]]
            assert np.all(margins <= 0.0625), (step, margins)
            mismatched += int(bad.sum())
        if step in hs:
            ref = from_bf16_bits(g["hidden"][hs.index(step)]).astype(np.float64)
            h = from_bf16_bits(host_bits(eng.hidden)).astype(np.float64)
            worst = max(worst, float(np.max(np.abs(h - ref) / (1 + np.abs(ref)))))
            assert np.all(np.abs(h - ref) <= 5e-2 + 2e-2 * np.abs(ref)), (step, np.abs(h - ref).max())
    print(f"reference model, 64 steps: worst |h - ref| / (1 + |ref|) = {worst:.4g}; "
          f"{mismatched} of {g['next'].size} ids differ, all on near-ties")
    assert int(eng.status.item()) == 0
    assert eng.health() == {"status": 0, "error_word": 0}
    assert mismatched <= 0.02 * g["next"].size, mismatched


def test_graph_replay_is_bitwise_eager(model):
    dc, _, w = model
    g = golden("decode")
    a, b = DecodeEngine(w, max_length=128), DecodeEngine(w, max_length=128)
    b.capture()
    for step in range(8):
        alen, delay = schedule(step)
        ids = torch.from_numpy(g["ids"][step])
        na = a.step(ids, step, alen, delay)
        nb = b.step(ids, step, alen, delay)
        assert torch.equal(na, nb)
        assert np.array_equal(host_bits(a.audio_logits), host_bits(b.audio_logits))
        assert np.array_equal(host_bits(a.hidden), host_bits(b.hidden))
    assert torch.equal(a.kv, b.kv)


def test_device_advance_graph_matches_host_loop(model):
    """The captured step+advance graph runs autonomously (ids fed back on the device)."""
    dc, _, w = model
    g = golden("decode")
    host, dev = DecodeEngine(w, max_length=128), DecodeEngine(w, max_length=128)
    dev.capture(advance=True)
    ids = torch.from_numpy(g["ids"][0])
    dev.set_inputs(ids, 0, 1, -1)
    alen, delay = 1, -1
    cur = ids
    for step in range(12):
        nxt = host.step(cur, step, alen, delay).reshape(-1)
        dev.run(advance=True)
        assert torch.equal(dev.ids.cpu(), nxt.cpu()), step
        # host-side replica of the delay bookkeeping (first_audio_graph.py:21-25)
        text = int(nxt[0])
        alen += 1
        if delay < 0 and text == dc.audio_assistant_delay_slot_token_id:
            delay = 0
        if delay >= 0:
            delay += 1
        cur = nxt.cpu()
    assert int(dev.position.item()) == 12


def test_pinned_host_roundtrip(model):
    dc, _, w = model
    g = golden("decode")
    eng = DecodeEngine(w, max_length=128)
    eng.capture()
    eng.set_inputs(torch.from_numpy(g["ids"][0]), 0, 1, -1)
    eng.run()
    out = eng.read_next_ids()
    assert out.device.type == "cpu" and out.is_pinned()
    assert out.shape == (1, 1, 33)


def test_bf16_preset_decode_matches_oracle(cuda_device):
    """The BF16 preset (bf16 projections, streamed bf16 GEMVs) of the same 2-layer full-width
    model against the oracle decoder: 16 greedy steps fed the oracle's own ids; hidden states
    within max-abs 5e-2 / rel 2e-2, ids identical except on near-ties of the oracle's top two."""
    from oracle import model as omodel
    dc = small_vocab(DecoderConfig(), vocab=2048, layers=2)
    host = synthetic.decoder_weights(dc, seed=9, preset="bf16")
    w = DecoderWeights.from_host(dc, host, cuda_device, preset="bf16")
    eng = DecodeEngine(w, max_length=64)
    dec = omodel.Decoder(host, dc.as_dict(), max_length=64)
    ids = np.zeros(1 + dc.n_vq, dtype=np.int64)
    ids[0] = dc.audio_assistant_gen_slot_token_id
    mismatched = 0
    for step in range(16):
        alen, delay = schedule(step)
        want, text, audio, h_ref = dec.step(ids, step, alen, delay)
        got = eng.step(torch.from_numpy(ids), step, alen, delay).reshape(-1).cpu().numpy()
        h = from_bf16_bits(host_bits(eng.hidden)).astype(np.float64).reshape(-1)
        ref = np.asarray(h_ref, dtype=np.float64).reshape(-1)
        assert np.all(np.abs(h - ref) <= 5e-2 + 2e-2 * np.abs(ref)), (step, np.abs(h - ref).max())
        bad = got != want
        if bad.any():
            assert not bad[0] or abs(float(text[0] - text[1])) <= 0.0625, step
            top2 = np.sort(np.asarray(audio, dtype=np.float64), axis=-1)[:, -2:]
            margins = (top2[:, 1] - top2[:, 0])[bad[1:]]
            assert np.all(margins <= 0.0625), (step, margins)
            mismatched += int(bad.sum())
        ids = want
    assert int(eng.status.item()) == 0
    assert mismatched <= 0.02 * 16 * (1 + dc.n_vq), mismatched
