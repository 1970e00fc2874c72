"""The device sampler (``mt_heads_sample``) and the 32-step first-audio graph on a B200.

* temperature 0 is ``mt_heads_select`` (greedy) exactly, masks included;
* every draw equals the oracle's replay of the same Philox draw (``oracle.sampling.device_pick``)
  unless the uniform lies within 1e-5 of a boundary of the kept cumulative probabilities (fp32
  softmax rounding); the draws' frequencies match the reference's ``sample_topk`` distribution
  (pinned to the reference's own draws on CPU) within 5 standard errors; every draw is in the
  distribution's support;
* ``FastLLM`` with sampling: the captured graph equals the eager step, draws are reproducible
  per (seed, position), and ``FirstAudioGraph`` replays 32 steps exactly as 32 eager steps
  with the device advance (greedy and sampled).
"""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import sampling
from oracle.numerics import from_bf16_bits

from moss_tts._runtime import native, synthetic
from moss_tts._runtime.config import DecoderConfig, small_vocab
from moss_tts._runtime.first_audio_graph import FirstAudioGraph
from moss_tts._runtime.llm import FastLLM
from moss_tts._runtime.weights import DecoderWeights

pytestmark = pytest.mark.gpu
AUDIO, TEXT = (1.7, 25, 0.8), (1.5, 2, 1.0)


def _bf16(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits, np.uint16).view(np.int16)).view(torch.bfloat16).to(dev)


def _sample(dev, text, audio, pos, alen, delay, seed, n_cb, vocab, temps=(TEXT, AUDIO), text_ids=None):
    B = pos.shape[0]
    out = torch.full((B, 1 + n_cb), -9, dtype=torch.long, device=dev)
    tids = text_ids if text_ids is not None else torch.tensor([7, 9], dtype=torch.long, device=dev)
    t, a = temps
    native.call("mt_heads_sample", text.data_ptr(), audio.data_ptr(), tids.data_ptr(), pos.data_ptr(), alen.data_ptr(),
                delay.data_ptr(), seed.data_ptr(), out.data_ptr(), B, 2, n_cb, vocab, 0, n_cb, 5, 6, 1024, 1,
                float(t[0]), int(t[1]), float(t[2]), float(a[0]), int(a[1]), float(a[2]), 0,
                torch.cuda.current_stream(dev).cuda_stream)
    return out.cpu().numpy()


def test_temperature_zero_is_greedy_selection(cuda_device):
    dev = cuda_device
    rng = np.random.Generator(np.random.PCG64(3))
    B, n_cb, V = 6, 32, 1024
    audio = torch.from_numpy(rng.standard_normal((B, n_cb * V)).astype(np.float32)).bfloat16().to(dev)
    audio[0, 5] = audio[0, 9] = 12.0  # first-index tie
    text = torch.from_numpy(rng.standard_normal((B, 2)).astype(np.float32)).bfloat16().to(dev)
    pos = torch.arange(B, dtype=torch.long, device=dev) + 40
    alen = torch.tensor([33, 3, 33, 12, 1, 33], dtype=torch.long, device=dev)
    delay = torch.tensor([-1, -1, 0, 32, 5, 31], dtype=torch.long, device=dev)
    seed = torch.arange(B, dtype=torch.long, device=dev)
    got = _sample(dev, text, audio, pos, alen, delay, seed, n_cb, V, temps=((0.0, 2, 1.0), (0.0, 25, 0.8)))
    want = torch.full((B, 33), -7, dtype=torch.long, device=dev)
    tids = torch.tensor([7, 9], dtype=torch.long, device=dev)
    native.call("mt_heads_select", text.data_ptr(), audio.data_ptr(), tids.data_ptr(), alen.data_ptr(),
                delay.data_ptr(), want.data_ptr(), B, 2, n_cb, V, 0, n_cb, 5, 6, 1024, 1, 0,
                torch.cuda.current_stream(dev).cuda_stream)
    assert np.array_equal(got, want.cpu().numpy())
    assert got[0, 1] == 5


def test_draws_replay_the_oracle_and_match_the_reference_distribution(cuda_device):
    dev = cuda_device
    g = golden("sampling")
    n_cb, V, B = 6, 1024, 4096
    audio_rows = g["audio_logits"]  # [6, 1024] bf16 bits: the reference fixture's rows
    text_rows = g["text_logits"][0]
    audio = _bf16(np.tile(audio_rows.reshape(1, -1), (B, 1)), dev)
    text = _bf16(np.tile(text_rows.reshape(1, -1), (B, 1)), dev)
    rng = np.random.Generator(np.random.PCG64(11))
    seeds = rng.integers(0, 2 ** 62, size=B, dtype=np.int64)
    positions = rng.integers(0, 2 ** 40, size=B, dtype=np.int64)
    pos = torch.from_numpy(positions).to(dev)
    seed = torch.from_numpy(seeds).to(dev)
    alen = torch.full((B,), 33, dtype=torch.long, device=dev)
    delay = torch.full((B,), -1, dtype=torch.long, device=dev)
    got = _sample(dev, text, audio, pos, alen, delay, seed, n_cb, V)
    assert np.array_equal(got, _sample(dev, text, audio, pos, alen, delay, seed, n_cb, V))  # reproducible
    rows = [(from_bf16_bits(text_rows), TEXT)] + [(from_bf16_bits(audio_rows[c]), AUDIO) for c in range(n_cb)]
    near, exact = 0, 0
    for ch, (logits, args) in enumerate(rows):
        idx, q = sampling.sample_distribution(logits, *args)
        picks = got[:, ch] if ch else np.where(got[:, 0] == 7, 0, 1)
        assert np.isin(picks, idx).all(), ch
        counts = np.array([(picks == i).sum() for i in idx])
        z = np.abs(counts / B - q) / np.sqrt(q * (1 - q) / B + 1e-12)
        assert z.max() <= 5, (ch, z.max())
        for b in range(0, B, 8):  # replay every eighth draw exactly
            want, dist = sampling.device_pick(logits, *args, int(seeds[b]), int(positions[b]), ch - 1)
            if dist < 1e-5:
                near += 1
            else:
                exact += 1
                assert picks[b] == want, (ch, b)
    print(f"sampler: {exact} draws replayed exactly, {near} within 1e-5 of a boundary")


def test_sampling_masks(cuda_device):
    dev = cuda_device
    rng = np.random.Generator(np.random.PCG64(5))
    B, n_cb, V = 4, 32, 1024
    audio = torch.from_numpy(rng.standard_normal((B, n_cb * V)).astype(np.float32) * 3).bfloat16().to(dev)
    text = torch.from_numpy(rng.standard_normal((B, 2)).astype(np.float32)).bfloat16().to(dev)
    pos = torch.tensor([3, 4, 5, 6], dtype=torch.long, device=dev)
    alen = torch.tensor([33, 4, 33, 33], dtype=torch.long, device=dev)
    delay = torch.tensor([-1, -1, 10, 32], dtype=torch.long, device=dev)
    seed = torch.tensor([1, 2, 3, 4], dtype=torch.long, device=dev)
    got = _sample(dev, text, audio, pos, alen, delay, seed, n_cb, V)
    assert (got[1, 1 + 4:] == 1024).all() and (got[1, 1:5] < 1024).all()
    assert (got[2, 1:11] == 1024).all() and (got[2, 11:] < 1024).all() and got[2, 0] == 5
    assert got[3, 0] == 6 and (got[3, 1:33] == 1024).all()
    assert got[0, 0] in (7, 9)


@pytest.fixture(scope="module")
def model(cuda_device):
    dc = small_vocab(DecoderConfig(), vocab=2048, layers=2)
    host = synthetic.decoder_weights(dc, seed=7)
    return dc, DecoderWeights.from_host(dc, host, cuda_device)


def test_fastllm_sampled_step_graph_and_reproducibility(model, cuda_device):
    dc, w = model
    llm = FastLLM(w, max_length=256, greedy=False)
    llm.engine.set_seed(1234)
    ids = torch.full((1, 1, 33), 7, dtype=torch.long)
    ids[0, 0, 0] = dc.audio_assistant_gen_slot_token_id
    eager = [llm.step(ids, 10 + i, 33, -1).cpu() for i in range(3)]
    llm.warmup()
    graphed = [llm.step(ids, 10 + i, 33, -1).cpu() for i in range(3)]
    assert all(torch.equal(a, b) for a, b in zip(eager, graphed))
    # the draws follow the engine's own logits: every id in the sampler's support
    llm.step(ids, 40, 33, -1)
    audio = llm.engine.audio_logits.view(32, -1).float().cpu().numpy()
    nxt = llm.next_ids.view(-1).cpu().numpy()
    for c in range(32):
        idx, _ = sampling.sample_distribution(audio[c], *AUDIO)
        assert nxt[1 + c] in idx, c
    llm.engine.set_seed(99)
    other = llm.step(ids, 10, 33, -1).cpu()
    assert not torch.equal(other, eager[0])  # another seed, other draws (33 channels)
    assert int(llm.engine.status.item()) == 0


@pytest.mark.parametrize("greedy", [True, False])
def test_first_audio_graph_matches_eager_steps(model, cuda_device, greedy):
    dc, w = model
    llm = FastLLM(w, max_length=256, greedy=greedy)
    llm.engine.set_seed(77)
    llm.warmup()
    fa = FirstAudioGraph(llm, 128)
    fa.warmup()
    first = torch.full((1, 1, 33), dc.audio_pad_code, dtype=torch.long, device=cuda_device)
    first[0, 0, 0] = dc.audio_start_token_id
    g = torch.Generator(device=cuda_device).manual_seed(5)
    llm.engine.kv.normal_(generator=g)
    kv0 = llm.engine.kv.clone()
    hist, status = fa.run(first, 20)
    hist, status = hist.cpu().clone(), status.cpu().clone()
    # the same 32 steps eagerly, from the same cache
    llm.engine.kv.copy_(kv0)
    e = llm.engine
    e.ids.copy_(first.view(-1))
    e.position.fill_(20)
    e.audio_length.fill_(1)
    e.delay_length.fill_(-1)
    rows = []
    for _ in range(32):
        llm._decode()
        rows.append(e.next_ids.cpu().clone())
        e.launch_advance()
    assert torch.equal(hist, torch.stack(rows))
    st = status.tolist()
    assert st[0] == int(rows[-1][0]) and st[1] == 33 and st[3] == 52 and st[2] == int(e.delay_length.item())
    # audio channel c is masked to the pad code while audio_length <= c (step s has length s + 1)
    for s in range(32):
        assert (hist[s, 2 + s:] == dc.audio_pad_code).all(), s
    with pytest.raises(ValueError):
        fa.run(first, 100)
