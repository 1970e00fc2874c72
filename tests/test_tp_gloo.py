"""Tensor-parallel host logic on CPU: two ``gloo`` ranks, no GPU.

* ``shard_weights`` gives each rank the right q/k/v heads and gate/up rows (column-parallel)
  and the right o_proj / down input columns (row-parallel): every rank's column-parallel
  output equals its slice of the unsharded projection, and the row-parallel partials summed
  with ``TensorParallel.all_reduce`` equal the unsharded projection (oracle arithmetic,
  fp32 reduction order aside).
* Failure detection happens on the host: a rank that dies before a collective makes the
  surviving rank's collective fail within the process-group timeout instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ops, quant
from oracle.numerics import from_bf16_bits

from moss_tts._runtime import synthetic
from moss_tts._runtime.config import DecoderConfig
from moss_tts._runtime.engine import TensorParallel, shard_weights
from moss_tts._runtime.weights import DecoderWeights

CFG = DecoderConfig(hidden_size=1024, intermediate_size=1024, num_layers=1, num_heads=8, num_kv_heads=4,
                    head_dim=128, vocab_size=64, n_vq=4, audio_vocab_size=64, pad_token_id=48,
                    im_start_token_id=49, im_end_token_id=50, audio_user_slot_token_id=51,
                    audio_assistant_gen_slot_token_id=52, audio_assistant_delay_slot_token_id=53,
                    audio_start_token_id=54, audio_end_token_id=55, audio_pad_code=64)


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def init(rank, world, port, seconds):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=seconds))


def dense(p) -> np.ndarray:
    """Dequantized fp32 weights of a (CPU) Projection."""
    qz = None if p.qzeros is None else p.qzeros.numpy()
    sc = p.scales.contiguous().view(torch.int16).numpy().view(np.uint16)
    return quant.dequantize_w4(p.qweight.numpy(), sc, qz)


def shard_worker(rank, world, port, out_dir):
    init(rank, world, port, 60)
    host = synthetic.decoder_weights(CFG, seed=5)
    full = DecoderWeights.from_host(CFG, host, "cpu")
    mine = shard_weights(full, rank, world)
    tp = TensorParallel(rank, world)
    lf, lm = full.layers[0], mine.layers[0]
    d, nq, nkv, inter = CFG.head_dim, CFG.num_heads // world, CFG.num_kv_heads // world, CFG.intermediate_size
    x = from_bf16_bits(synthetic.activation(3, (1, CFG.hidden_size)))
    report = {}
    # column-parallel q|k|v: this rank's heads of the unsharded output, in q, k, v order
    y_full = ops.linear(x, dense(lf.qkv))
    y_mine = ops.linear(x, dense(lm.qkv))
    q0, k0, v0 = rank * nq * d, CFG.num_heads * d + rank * nkv * d, (CFG.num_heads + CFG.num_kv_heads) * d + rank * nkv * d
    want = np.concatenate([y_full[:, q0:q0 + nq * d], y_full[:, k0:k0 + nkv * d], y_full[:, v0:v0 + nkv * d]], 1)
    report["qkv_exact"] = bool(np.array_equal(y_mine, want))
    # row-parallel o_proj: partial over this rank's attention columns, summed over ranks
    a = from_bf16_bits(synthetic.activation(4, (1, CFG.num_heads * d)))
    part = torch.from_numpy(ops.linear(a[:, rank * nq * d:(rank + 1) * nq * d], dense(lm.out)).astype(np.float32))
    tp.all_reduce(part)
    ref = ops.linear(a, dense(lf.out))
    report["o_err"] = float(np.abs(part.numpy() - ref).max())
    report["o_scale"] = float(np.abs(ref).max())
    # MLP: column-parallel gate/up (+ SiLU), row-parallel down, one all-reduce
    h = from_bf16_bits(synthetic.activation(6, (1, CFG.hidden_size)))
    mid = ops.silu_mul(ops.linear(h, dense(lm.gate_up)))
    part = torch.from_numpy(ops.linear(mid, dense(lm.down)).astype(np.float32))
    tp.all_reduce(part)
    ref = ops.linear(ops.silu_mul(ops.linear(h, dense(lf.gate_up))), dense(lf.down))
    report["mlp_err"] = float(np.abs(part.numpy() - ref).max())
    report["mlp_scale"] = float(np.abs(ref).max())
    # audio heads: this rank's codebooks
    cb = CFG.n_vq // world
    v = CFG.audio_vocab_size
    report["heads_exact"] = bool(torch.equal(mine.head_audio, full.head_audio[rank * cb * v:(rank + 1) * cb * v]))
    report["meta"] = mine.meta.get("tp_rank") == rank and mine.meta.get("tp_world") == world
    dist.barrier()
    dist.destroy_process_group()
    torch.save(report, os.path.join(out_dir, f"rank{rank}.pt"))


def test_shard_weights_and_all_reduce_match_unsharded(tmp_path):
    port = free_port()
    mp.start_processes(shard_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for rank in range(2):
        r = torch.load(tmp_path / f"rank{rank}.pt")
        assert r["qkv_exact"] and r["heads_exact"] and r["meta"], r
        # bf16 partials summed in fp32 against one bf16-rounded dot product: a few bf16 ulps
        assert r["o_err"] <= 2e-2 * r["o_scale"] + 1e-3, r
        assert r["mlp_err"] <= 2e-2 * r["mlp_scale"] + 1e-3, r


def failure_worker(rank, world, port, out_dir):
    init(rank, world, port, 5)
    if rank == 1:
        os._exit(3)  # a rank that dies between steps, before the next collective
    status = "hung"
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        status = "completed"
    except Exception as exc:  # the surviving rank learns of the failure on the host
        status = "detected: " + type(exc).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_dead_rank_is_detected_by_the_survivor(tmp_path):
    port = free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=failure_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not exit")
    assert procs[1].exitcode == 3
    assert (tmp_path / "rank0.txt").read_text().startswith("detected"), (tmp_path / "rank0.txt").read_text()
