"""Worker for tests/test_gpu_tp.py, launched with torchrun on 2+ GPUs (one rank per GPU).

Every rank builds the same 2-layer full-width decoder (small vocabulary), shards it with
``shard_weights`` and runs captured decode steps through NCCL tensor parallelism; rank 0
also runs the unsharded model on its own GPU and writes the comparison to argv[1].
"""
import datetime
import json
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(REPO), str(REPO / "moss-tts-optimized_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from moss_tts._runtime import native, synthetic  # noqa: E402
from moss_tts._runtime.config import DecoderConfig, small_vocab  # noqa: E402
from moss_tts._runtime.batch_engine import BatchDecodeEngine  # noqa: E402
from moss_tts._runtime.engine import DecodeEngine, TensorParallel, shard_weights  # noqa: E402
from moss_tts._runtime.weights import DecoderWeights  # noqa: E402


def main(out_path: str) -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = small_vocab(DecoderConfig(), vocab=2048, layers=2)
    host = synthetic.decoder_weights(cfg, seed=7)
    full = DecoderWeights.from_host(cfg, host, dev)
    tp = TensorParallel(rank, world, dist.group.WORLD)
    dist.all_reduce(torch.ones(1, device=dev))  # communicator up before capture
    eng = DecodeEngine(shard_weights(full, rank, world), max_length=128, tp=tp)
    eng.capture()
    ref = DecodeEngine(full, max_length=128) if rank == 0 else None
    # every rank enters the first step together (rank 0 built the reference engine meanwhile)
    torch.cuda.synchronize(dev)
    dist.barrier()
    native.error_word(clear=True)
    ids = torch.full((33,), 7, dtype=torch.long)
    ids[0] = 5
    report = {"steps": []}
    for step in range(6):
        got = eng.step(ids, step, step + 1, -1).reshape(-1).cpu()
        if rank == 0:
            want = ref.step(ids, step, step + 1, -1).reshape(-1).cpu()
            h_tp, h_1 = eng.hidden.float().cpu(), ref.hidden.float().cpu()
            report["steps"].append({
                "ids_equal": int((got == want).sum()), "ids": int(got.numel()),
                "hidden_max_abs": float((h_tp - h_1).abs().max()),
                "hidden_scale": float(h_1.abs().max()),
                # rank 0 holds codebooks 0 .. n_vq / world - 1: the first rows of the full heads
                "audio_logits_max_abs": float((eng.audio_logits.float().cpu()
                                               - ref.audio_logits.float().cpu()[:eng.audio_logits.numel()]).abs().max()),
            })
            ids = want
        obj = [ids]
        dist.broadcast_object_list(obj, src=0)
        ids = obj[0]
    report["status"] = int(eng.status.item())
    # a peer-exchange poll that gave up (error word 2) would have computed with stale rows
    word = torch.tensor([native.error_word(clear=True)], device=dev, dtype=torch.int32)
    dist.all_reduce(word, op=dist.ReduceOp.MAX)
    report["error_word"] = int(word.item())
    eng.graph = None  # graphs holding NCCL work go before the process group
    # batched decode (tcgen05 GEMM projections, ragged contexts) through the same all-reduces
    B, nkv = 16, cfg.num_kv_heads // world
    beng = BatchDecodeEngine(shard_weights(full, rank, world), B, max_length=128, tp=tp)
    bref = BatchDecodeEngine(full, B, max_length=128) if rank == 0 else None
    g = torch.Generator(device=dev).manual_seed(11)
    kv = torch.randn((2, 2, B, cfg.num_kv_heads, 128, 128), generator=g, device=dev).to(torch.bfloat16)
    beng.kv.copy_(kv[:, :, :, rank * nkv:(rank + 1) * nkv])
    if rank == 0:
        bref.kv.copy_(kv)
    pos = torch.arange(B) * 6 + 9
    bids = torch.full((B, 33), 7, dtype=torch.long)
    bids[:, 0] = 5
    one, neg = torch.ones(B, dtype=torch.long), torch.full((B,), -1, dtype=torch.long)
    report["batched"] = []
    for step in range(2):
        got = beng.step(bids, pos + step, one, neg).cpu()
        if rank == 0:
            want = bref.step(bids, pos + step, one, neg).cpu()
            h_tp, h_1 = beng.hidden.float().cpu(), bref.hidden.float().cpu()
            report["batched"].append({"ids_equal": int((got == want).sum()), "ids": int(got.numel()),
                                      "hidden_max_abs": float((h_tp - h_1).abs().max()),
                                      "hidden_scale": float(h_1.abs().max())})
            bids = want
        obj = [bids]
        dist.broadcast_object_list(obj, src=0)
        bids = obj[0]
    report["status"] |= int(beng.status.item())
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        Path(out_path).write_text(json.dumps(report))


if __name__ == "__main__":
    main(sys.argv[1])
