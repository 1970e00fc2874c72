#!/usr/bin/env python
"""Batch-1 decode benchmark of the MOSS-TTS 8B backbone (W4A16 G32) on B200.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Workload: the full 36-layer Qwen3-8B-shaped decoder with random-init
W4A16 G32 projections, 32 x 1024-row audio heads and the reference decode step's 2-row
audio-phase text head (``FastLLM._decode``); a 512-token prompt is stood in for by
filling the first 512 KV-cache rows with seeded N(0, 1) values, then W + K greedy
decode steps run at positions 512, 513, ... One step = one pass of the whole decode
hot path. N > 1 runs tensor parallelism over N GPUs (NCCL all-reduce after o_proj and
down); total work per step is fixed, so scaling is "strong".

Reported: ``value`` = steps/s with inputs resident in HBM (CUDA graph with device-side
feedback of the ids, CUDA events, max over ranks); ``e2e`` = the same through
``FastLLM.step_host`` with the step's int64 control block copied from pinned host memory
and the next ids copied back every step; ``roofline`` for the dominant kernel (the W4A16
gate/up GEMV); ``cpu_baseline`` = the CPU oracle on a bounded sample (rank 0, N = 1).
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (str(REPO), str(REPO / "moss-tts-optimized_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "batch-1 decode steps/s (8B W4A16 G32)"
UNIT = "steps/s"
PROMPT = 512


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=36, help=argparse.SUPPRESS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-bf16", action="store_true", help="skip the BF16-preset step timing")
    ap.add_argument("--no-prefill", action="store_true", help="skip the 512-token prefill timing")
    ap.add_argument("--batch-sweep", default=None, metavar="B,B,...",
                    help="config 4: batched decode of B sequences with ragged contexts (uniform in "
                         "[256, 4096], seeded) for each listed B; prints one JSON line per B")
    ap.add_argument("--profile-gemm", type=int, default=0, metavar="B",
                    help="only launch the tcgen05 W4A16 GEMM on the fused gate/up shape with B rows "
                         "(4 launches on random weights, for an ncu capture); prints its mean launch time")
    ap.add_argument("--config0", action="store_true",
                    help="config 0 alone: the 12288 x 4096 W4A16 G32 GEMV (zero points), 8 rotating weight sets "
                         "(233 MB > L2, every launch L2-cold), CUDA events; prints one JSON line with its roofline")
    ap.add_argument("--config0-sets", type=int, default=8, help=argparse.SUPPRESS)
    ap.add_argument("--profile-attention", default=None, metavar="B,CTX",
                    help="decode attention alone: B sequences at CTX cached tokens, one layer (GB/s line)")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="per-kernel device time of one 512-token prefill (CUPTI through torch.profiler)")
    ap.add_argument("--profile-kernel", action="store_true",
                    help="only launch the dominant kernel (packed add+norm+gate/up+SiLU GEMV), once per "
                         "layer per step, for an ncu capture; prints its mean launch time")
    return ap.parse_args()


class ClockSampler:
    """Polls NVML (read-only) for SM clock and throttle reasons during the timed region."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [v.strip() for v in visible.split(",") if v.strip()]
        if ids and all(v.isdigit() for v in ids) and index < len(ids):
            index = int(ids[index])
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no clocks rather than guess
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.reasons |= {n for bit, n in self.REASONS.items() if r & bit}
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nv is not None:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.nv is not None:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def gate_up_bytes(k: int, n: int) -> int:
    """Algorithmic bytes of one fused add+norm+gate/up+SiLU launch (batch 1)."""
    codes, scales, zeros = n * k // 2, n * (k // 32) * 2, n * (k // 64)
    act = 4 * k * 2  # x, residual, norm weight read; summed written
    return codes + scales + zeros + act + (n // 2) * 2


# ---------------------------------------------------------------------------- CPU leg
def workload_config(layers: int, world: int, max_length: int) -> dict:
    """The config-3 workload both arms time (identical dict in the GPU line and the reference line)."""
    return {"workload": "config3: 36-layer 8B-shaped decoder, W4A16 G32 (zero points), batch-1 greedy "
                        "decode, prompt 512 (synthetic KV), positions 512+",
            "layers": layers, "hidden": 4096, "intermediate": 12288,
            "heads": "32x1024 audio rows + 2-row audio-phase text head (FastLLM._decode)",
            "parallelism": f"tp{world}", "max_length": max_length,
            "l2": "inputs larger than L2: ~4.4 GB of weights streamed per step"}


def max_length_for(args) -> int:
    return max(1024, ((PROMPT + args.warmup + args.steps + 1 + 127) // 128) * 128)


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def cpu_oracle_run(layers: int, steps: int, warmup: int, threads: int):
    """Decode steps of the numpy oracle -- the reference's decode step restated on the CPU --
    over the whole config-3 model: ``layers`` distinct random-init W4A16 G32 layers (zero
    points), dequantized once to fp32 up front (the reference's CPU path keeps dequantized
    weights), the 32 x 1024 audio heads and the 2-row text head, a synthetic 512-token KV
    prefix; ``warmup`` untimed then ``steps`` timed steps at positions 512, 513, ...
    Returns (steps/s, seconds of set-up)."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import model as omodel
    from moss_tts._runtime import synthetic
    from moss_tts._runtime.config import DecoderConfig, small_vocab

    t0 = time.perf_counter()
    with threadpool_limits(limits=threads):
        cfg = small_vocab(DecoderConfig(), vocab=2048, layers=layers)
        host = synthetic.decoder_weights(cfg, seed=11)
        dec = omodel.Decoder(host, cfg.as_dict(), max_length=PROMPT + warmup + steps + 8, threads=threads)
        del host
        rng = np.random.Generator(np.random.PCG64(12))
        kv = rng.standard_normal((layers, 8, PROMPT, 128), dtype=np.float32)
        dec.fill_cache(kv, kv)
        del kv
        setup = time.perf_counter() - t0
        ids = np.full(33, 17, dtype=np.int64)
        ids[0] = cfg.audio_assistant_gen_slot_token_id
        pos = PROMPT
        for _ in range(warmup):
            ids = dec.step(ids, pos, 1, -1)[0]
            pos += 1
        t1 = time.perf_counter()
        for _ in range(steps):
            ids = dec.step(ids, pos, 1, -1)[0]
            pos += 1
        elapsed = time.perf_counter() - t1
    return steps / elapsed, setup


def cpu_sample_text(layers: int, steps: int, threads: int) -> str:
    return (f"numpy oracle (the reference's decode step restated), all {layers} layers distinct, dequantized "
            f"fp32 weights cached, 32x1024 audio heads + 2-row text head, {steps} timed steps at ctx "
            f"{PROMPT}+, {threads} BLAS threads")


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU algorithm for the decode step (the numpy port; the
    reference's own CUDA/Triton kernels are SM90-only and its package is not installable on the
    GPU box) on all host threads, over the same config-3 workload, K timed steps after W warm-up
    steps. Under torchrun only rank 0 runs it; the other ranks exit without work."""
    if rank != 0:
        return
    threads = cpu_threads()
    value, setup = cpu_oracle_run(args.layers, args.steps, args.warmup, threads)
    sample = cpu_sample_text(args.layers, args.steps, threads)
    line = {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 / value, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": workload_config(args.layers, world, max_length_for(args)),
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample, "setup_s": round(setup, 1)},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- GPU leg
def packed_gate_up(native, lw, x, r, summed, mid, workspace, flags, stream_ptr):
    """One launch of the decode step's dominant kernel: add + RMSNorm + gate/up + SiLU over the
    packed W4 tiles (what DecodeEngine runs)."""
    p = lw.gate_up
    native.call("mt_w4a16_linear_packed", x.data_ptr(), r.data_ptr(), lw.post_norm.data_ptr(), 1e-6,
                summed.data_ptr(), p.packed_tiles(True).data_ptr(), 1 if p.qzeros is not None else 0,
                mid.data_ptr(), p.n, p.k, 7, workspace.data_ptr(), flags, stream_ptr)


def profile_kernel(args):
    """Eager launches of the dominant kernel over each layer's weights (no graph, so every
    launch is visible to a profiler); inputs larger than L2 once there are 3+ layers."""
    import torch

    from moss_tts._runtime import native
    from moss_tts._runtime.config import DecoderConfig
    from moss_tts._runtime.weights import DecoderWeights

    dev = torch.device("cuda", 0)
    cfg = DecoderConfig().with_(num_layers=args.layers)
    with torch.inference_mode():
        w = DecoderWeights.random(cfg, dev, seed=0, preset="gptq", full_text_head=False)
        for lw in w.layers:
            lw.gate_up.packed_tiles(True)
        x = torch.randn(cfg.hidden_size, device=dev).bfloat16()
        r = torch.randn(cfg.hidden_size, device=dev).bfloat16()
        summed = torch.empty_like(x)
        mid = torch.empty(cfg.intermediate_size, device=dev, dtype=torch.bfloat16)
        ws = torch.zeros(native.w4a16_packed_size(2 * cfg.intermediate_size, cfg.hidden_size, True, 4)[1],
                         device=dev, dtype=torch.uint8)
        s = torch.cuda.current_stream(dev)
        for _ in range(args.warmup):
            for lw in w.layers:
                packed_gate_up(native, lw, x, r, summed, mid, ws, native.FLAG_PDL, s.cuda_stream)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(args.steps):
            for lw in w.layers:
                packed_gate_up(native, lw, x, r, summed, mid, ws, native.FLAG_PDL, s.cuda_stream)
        e1.record(s)
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1000 / (args.steps * len(w.layers))
    print(json.dumps({"kernel": "mt_w4a16_linear_packed gate/up (N=%d K=%d)" % (2 * cfg.intermediate_size,
                                                                            cfg.hidden_size),
                      "launches": args.steps * len(w.layers), "eager_launch_us": round(us, 3),
                      "bytes_per_launch": gate_up_bytes(cfg.hidden_size, 2 * cfg.intermediate_size)}), flush=True)


def bf16_step_rate(args, cfg, dev, rank, world, group, max_length):
    """Device-resident steps/s of the same decode step with the BF16 preset (config 3 is timed in
    both formats): random bf16 weights drawn on the device, the same graph replay and timing."""
    import torch
    import torch.distributed as dist

    from moss_tts._runtime.engine import DecodeEngine, TensorParallel, shard_weights
    from moss_tts._runtime.weights import DecoderWeights

    with torch.inference_mode():
        full = DecoderWeights.random(cfg, dev, seed=1, preset="bf16", full_text_head=False)
        w = shard_weights(full, rank, world)
        del full
        torch.cuda.empty_cache()
        eng = DecodeEngine(w, max_length=max_length, tp=TensorParallel(rank, world, group))
        ids0 = torch.full((33,), 17, dtype=torch.long)
        ids0[0] = cfg.audio_assistant_gen_slot_token_id
        eng.set_inputs(ids0, PROMPT, 1, -1)
        eng.capture(advance=True)
        stream = torch.cuda.current_stream(dev)
        for _ in range(args.warmup):
            eng.run(advance=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            eng.run(advance=True)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = float(ms.item())
        step_bytes = w.layer_bytes() + w.head_audio.numel() * 2 + 2 * cfg.hidden_size * 2 \
            + 147456 // world * (PROMPT + args.warmup + args.steps // 2) * args.layers // 36
        status = int(eng.status.item())
        eng.graph = eng.graph_advance = None
        del eng, w
        torch.cuda.empty_cache()
    return args.steps / (ms / 1000.0), ms / args.steps, step_bytes, status


def config0(args):
    """Config 0 on its own: y[1, 12288] = x[1, 4096] . W^T, W4A16 G32 with per-group zero points
    (codes U[0, 15], zeros U[6, 9], scales |N(0, 0.02)| / 7 + 1e-4), the packed tensor-core GEMV
    (mt_w4a16_linear_packed) and, beside it, the GPTQ-layout register GEMV (mt_w4a16_linear).
    ``--config0-sets`` independent weight sets (default 8: 233 MB, more than the 126 MB L2) are
    used in rotation, so every launch reads its weights from HBM. Algorithmic bytes per launch:
    codes + scales + zero points + x + y = 29,130,752 (the survey's config-0 figure)."""
    import torch

    from moss_tts._runtime import native
    from moss_tts._runtime.weights import Projection

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, k, sets = 12288, 4096, max(1, args.config0_sets)
    g = torch.Generator(device=dev).manual_seed(0)
    projs = []
    for _ in range(sets):
        qw = torch.randint(0, 256, (n, k // 2), generator=g, device=dev, dtype=torch.uint8)
        sc = (torch.randn((n, k // 32), generator=g, device=dev).abs() * 0.02 / 7 + 1e-4).to(torch.bfloat16)
        z = torch.randint(6, 10, (n, k // 32), generator=g, device=dev, dtype=torch.uint8)
        p = Projection(n, k, qw, sc, (z[:, 0::2] | (z[:, 1::2] << 4)).contiguous())
        p.packed_tiles(False)
        projs.append(p)
    x = torch.randn(k, generator=g, device=dev).to(torch.bfloat16)
    y = torch.empty(n, device=dev, dtype=torch.bfloat16)
    ws = torch.zeros(native.w4a16_packed_size(n, k, True, 0)[1], device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream(dev)
    algo = n * k // 2 + n * (k // 32) * 2 + n * (k // 64) + k * 2 + n * 2
    peak, peak_kind = measured_peaks()

    def packed(p):
        native.call("mt_w4a16_linear_packed", x.data_ptr(), None, None, 0.0, None, p.packed_tiles(False).data_ptr(), 1,
                    y.data_ptr(), n, k, 0, ws.data_ptr(), native.FLAG_PDL, stream.cuda_stream)

    def gptq(p):
        native.call("mt_w4a16_linear", x.data_ptr(), None, None, 0.0, None, p.qweight.data_ptr(), p.scales.data_ptr(),
                    p.qzeros.data_ptr(), y.data_ptr(), 1, n, k, 32, 0, native.FLAG_PDL, stream.cuda_stream)

    results = {}
    for name, fn in (("packed", packed), ("gptq_layout", gptq)):
        for _ in range(max(3, args.warmup)):
            for p in projs:
                fn(p)
        torch.cuda.synchronize(dev)
        reps = max(1, args.steps)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(0) as clocks:
            e0.record(stream)
            for _ in range(reps):
                for p in projs:
                    fn(p)
            e1.record(stream)
            torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1000 / (reps * sets)
        results[name] = {"launch_us": round(us, 3), "achieved_gbs": round(algo / (us * 1e-6) / 1e9, 1),
                         "frac": round(algo / (us * 1e-6) / 1e9 / peak, 4), "clocks": clocks.summary()}
    best = results["packed"]
    print(json.dumps({
        "metric": "config0 W4A16 G32 GEMV HBM GB/s (12288 x 4096, batch 1)", "value": best["achieved_gbs"],
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config0: one W4A16 G32 linear 12288 x 4096 with zero points, batch 1",
                   "weight_sets": sets, "l2": f"{sets} rotating weight sets ({sets * algo / 1e6:.0f} MB > L2)"},
        "roofline": {"bound": "hbm", "kernel": "mt_w4a16_linear_packed (mode 0, N=12288 K=4096)",
                     "achieved": best["achieved_gbs"], "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": best["frac"], "bytes_per_launch": algo, "launch_us": best["launch_us"],
                     "traffic": None},
        "kernels": results}), flush=True)


def profile_gemm(rows: int):
    """The batched projection alone: the tcgen05 GEMM on gate/up (N = 24576, K = 4096, fused
    pair) with `rows` activation rows, random codes / scales / zero points, in both weight
    layouts (GPTQ: mt_w4a16_gemm; packed: mt_w4a16_gemm_packed, what the batched engine runs).
    Three weight sets are rotated (175 MB per layout, more than the 126 MB L2), so every launch
    streams its weights from HBM; CUDA events over 6 launches after 3."""
    import torch

    from moss_tts._runtime import native

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    n, k, sets = 24576, 4096, 3
    peak, peak_kind = measured_peaks()
    qw = [torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=g) for _ in range(sets)]
    sc = [(torch.rand(n, k // 32, device=dev, generator=g) * 0.01 + 1e-4).to(torch.bfloat16) for _ in range(sets)]
    qz = [torch.randint(0, 256, (n, k // 64), dtype=torch.uint8, device=dev, generator=g) for _ in range(sets)]
    s = torch.cuda.current_stream(dev).cuda_stream
    pk_bytes = native.w4a16_gemm_pack_size(n, k, native.LINEAR_PAIRED)
    pk = [torch.empty(pk_bytes, dtype=torch.uint8, device=dev) for _ in range(sets)]
    for i in range(sets):
        native.call("mt_w4a16_gemm_pack", qw[i].data_ptr(), sc[i].data_ptr(), qz[i].data_ptr(), n, k,
                    native.LINEAR_PAIRED, pk[i].data_ptr(), s)
    x = torch.randn(rows, k, device=dev, generator=g).to(torch.bfloat16)
    y = torch.empty(rows, n // 2, device=dev, dtype=torch.bfloat16)
    ws = torch.zeros(native.w4a16_gemm_workspace(rows, n, k, native.LINEAR_PAIRED), dtype=torch.uint8, device=dev)
    weight_bytes = n * k // 2 + n * k // 32 * 2 + n * k // 64  # codes, scales, zero points
    flops = 2.0 * rows * n * k
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for layout in ("gptq", "packed"):
        for i in range(9):
            if i == 3:
                e0.record()
            j = i % sets
            if layout == "gptq":
                native.call("mt_w4a16_gemm", x.data_ptr(), qw[j].data_ptr(), sc[j].data_ptr(), qz[j].data_ptr(),
                            y.data_ptr(), rows, n, k, native.LINEAR_PAIRED, ws.data_ptr(), 0, s)
            else:
                native.call("mt_w4a16_gemm_packed", x.data_ptr(), pk[j].data_ptr(), y.data_ptr(), rows, n, k,
                            native.LINEAR_PAIRED, ws.data_ptr(), 0, s)
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1000 / 6
        print(json.dumps({"kernel": f"tcgen05 gate/up GEMM ({layout} layout)", "rows": rows, "launch_us": round(us, 2),
                          "weight_gbs": round(weight_bytes / us / 1e3, 1),
                          "frac_hbm": round(weight_bytes / us / 1e3 / peak, 4), "tflops": round(flops / us / 1e6, 1),
                          "peak_gbs": peak, "peak_kind": peak_kind, "error_word": native.error_word(clear=True)}),
              flush=True)


def batch_sweep(args, rank, world, local):
    """Config 4: W4A16 decode of B independent sequences per step, each with its own context
    length drawn uniformly from [256, 4096] (seeded), for every B of --batch-sweep. One step
    advances every sequence by one token; the metric is tokens/s = B x steps/s (device-resident
    inputs, CUDA graph with device-side advance, CUDA events, max over ranks). B = 1 runs the
    batch-1 engine; larger B the batched engine (two-row packed GEMV below 5 sequences, tcgen05
    GEMM projections from 5)."""
    import torch
    import torch.distributed as dist

    from moss_tts._runtime.batch_engine import BatchDecodeEngine
    from moss_tts._runtime.config import DecoderConfig
    from moss_tts._runtime.engine import DecodeEngine, TensorParallel, shard_weights
    from moss_tts._runtime import native
    from moss_tts._runtime.weights import DecoderWeights

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        group = dist.group.WORLD
        dist.all_reduce(torch.ones(1, device=dev))
    cfg = DecoderConfig().with_(num_layers=args.layers)
    peak, peak_kind = measured_peaks()
    batches = [int(b) for b in args.batch_sweep.split(",") if b]
    max_length = ((4096 + args.warmup + args.steps + 1 + 127) // 128) * 128
    with torch.inference_mode():
        full = DecoderWeights.random(cfg, dev, seed=0, preset="gptq", full_text_head=False)
        weights = shard_weights(full, rank, world)
        del full
        torch.cuda.empty_cache()
        tp = TensorParallel(rank, world, group)
        weight_bytes = weights.layer_bytes() + weights.head_audio.numel() * 2 + 2 * cfg.hidden_size * 2
        kv_row = 2 * (cfg.num_kv_heads // world) * cfg.head_dim * 2 * args.layers  # bytes per token, all layers
        for B in batches:
            rng = torch.Generator().manual_seed(1000 + B)
            ctx = torch.randint(256, 4097, (B,), generator=rng)
            if B == 1:
                eng = DecodeEngine(weights, max_length=max_length, tp=tp)
                kv = eng.kv.unsqueeze(2)
            else:
                eng = BatchDecodeEngine(weights, B, max_length=max_length, tp=tp)
                kv = eng.kv
            g = torch.Generator(device=dev).manual_seed(100 + rank)
            kv.normal_(generator=g)  # synthetic prompts: every cached row is N(0, 1)
            ids = torch.full((B, 33), 17, dtype=torch.long)
            ids[:, 0] = cfg.audio_assistant_gen_slot_token_id
            if B == 1:
                eng.set_inputs(ids[0], int(ctx[0]), 1, -1)
            else:
                eng.set_inputs(ids, ctx, torch.ones(B, dtype=torch.long), torch.full((B,), -1, dtype=torch.long))
            eng.capture(advance=True)
            for _ in range(args.warmup):
                eng.run(advance=True)
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize(dev)
            stream = torch.cuda.current_stream(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(local) as clocks:
                e0.record(stream)
                for _ in range(args.steps):
                    eng.run(advance=True)
                e1.record(stream)
                torch.cuda.synchronize(dev)
            ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
            if world > 1:
                dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            ms = float(ms.item()) / args.steps
            status = int(eng.status.item()) | native.error_word(clear=True)
            # bytes one step must read per GPU: weights once + every sequence's KV rows (mid-run context)
            mean_ctx = float(ctx.double().mean()) + args.warmup + args.steps / 2
            step_bytes = weight_bytes + int(kv_row * mean_ctx * B)
            if rank == 0:
                print(json.dumps({
                    "metric": "batched decode tokens/s (8B W4A16 G32, ragged contexts)", "value": round(B * 1000.0 / ms, 2),
                    "unit": "tokens/s", "batch": B, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": round(ms, 4), "steps_per_s": round(1000.0 / ms, 2), "dtype": "bf16",
                    "data": "synthetic", "scaling": "strong",
                    "config": {"workload": "config4: 36-layer 8B-shaped decoder, W4A16 G32, batched greedy decode, "
                                           "per-sequence context uniform in [256, 4096] (seeded)",
                               "parallelism": f"tp{world}", "projections": "packed GEMV" if B == 1 else
                               ("tcgen05 GEMM" if getattr(eng, "gemm", False) else
                                "packed two-row GEMV" if getattr(eng, "rows_packed", False) else "GPTQ-layout GEMV"),
                               "mean_context": round(mean_ctx, 1)},
                    "step_bytes_per_gpu": step_bytes,
                    "hbm_roofline_frac": round(step_bytes / (ms * 1e-3) / 1e9 / peak, 4), "peak_gbs": peak,
                    "peak_kind": peak_kind, "clocks": clocks.summary(), "status": status}), flush=True)
            eng.graph = eng.graph_advance = None
            del eng, kv
            torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def profile_attention(batch: int, ctx: int):
    """The fused decode attention (``mt_attention_decode``: QK-norm, RoPE, KV-row write, cluster
    split-K attention) alone for one layer: ``batch`` sequences at position ``ctx - 1`` (``ctx``
    cached tokens each, the last one written by the call), 32 query / 8 KV heads of 128, random
    cache. Algorithmic bytes per launch: the K and V rows read (batch x 8 x ctx x 512 B) plus the
    q|k|v rows and outputs; with more than 126 MB of cache every launch reads it from HBM.
    Eight timed launches after three warm-up ones, CUDA events."""
    import torch

    from moss_tts._runtime import native
    from moss_tts._runtime.engine import rope_tables

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    nq, nkv, d = 32, 8, 128
    max_len = (ctx + 127) // 128 * 128
    g = torch.Generator(device=dev).manual_seed(0)
    k = torch.randn(batch, nkv, max_len, d, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(batch, nkv, max_len, d, device=dev, generator=g).to(torch.bfloat16)
    qkv = torch.randn(batch, (nq + 2 * nkv) * d, device=dev, generator=g).to(torch.bfloat16)
    qn = torch.ones(d, device=dev, dtype=torch.bfloat16)
    cos, sin = (t.to(dev) for t in rope_tables(max_len, d, 1e6))
    pos = torch.full((batch,), ctx - 1, dtype=torch.long, device=dev)
    out = torch.empty(batch, nq * d, device=dev, dtype=torch.bfloat16)
    splits = max_len // 32
    partial = torch.empty(batch * nkv * splits * (nq // nkv) * d, device=dev, dtype=torch.float32)
    lse = torch.empty(batch * nkv * splits * (nq // nkv), device=dev, dtype=torch.float32)
    tickets = torch.zeros(batch * nkv, device=dev, dtype=torch.int32)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    s = torch.cuda.current_stream(dev).cuda_stream

    def launch():
        native.call("mt_attention_decode", qkv.data_ptr(), qn.data_ptr(), qn.data_ptr(), cos.data_ptr(),
                    sin.data_ptr(), pos.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), partial.data_ptr(),
                    lse.data_ptr(), tickets.data_ptr(), batch, nq, nkv, max_len, 1, 1e-6, status.data_ptr(), 0, s)

    for _ in range(3):
        launch()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(8):
        launch()
    e1.record()
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1000 / 8
    nbytes = batch * nkv * ctx * d * 2 * 2 + batch * ((nq + 2 * nkv) * d + nq * d) * 2
    peak, kind = measured_peaks()
    gbs = nbytes / (us * 1e-6) / 1e9
    print(json.dumps({"kernel": "mt_attention_decode (cluster)", "batch": batch, "ctx": ctx,
                      "bytes_per_launch": nbytes, "launch_us": round(us, 3), "achieved_gbs": round(gbs, 1),
                      "peak_gbs": peak, "peak_kind": kind, "frac": round(gbs / peak, 4),
                      "status": int(status.item()), "error_word": native.error_word(clear=True)}), flush=True)


def profile_prefill(args):
    """Per-kernel device time of one 512-token ``FastLLM.prefill`` of the config-3 model (full
    text head), each projection mode after two warm-up prompts, from CUPTI kernel records
    (torch.profiler): where the prompt pass spends its time. Not a bench line."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from moss_tts._runtime.config import DecoderConfig
    from moss_tts._runtime.llm import FastLLM
    from moss_tts._runtime.weights import DecoderWeights

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = DecoderConfig().with_(num_layers=args.layers)
    with torch.inference_mode():
        w = DecoderWeights.random(cfg, dev, seed=0, preset="gptq", full_text_head=True)
        llm = FastLLM(w, max_length=1024, greedy=True)
        g = torch.Generator().manual_seed(3)
        ids = torch.full((1, PROMPT, 33), 1024, dtype=torch.long)
        ids[0, :, 0] = torch.randint(0, cfg.vocab_size, (PROMPT,), generator=g)
        ids[0, :, 1:] = torch.randint(0, 1025, (PROMPT, 32), generator=g)
        ids = ids.to(dev)
        for mode in ("bf16", "dequant", "w4"):
            llm.prefill_mode = mode
            for _ in range(2):
                llm.prefill(ids)
            torch.cuda.synchronize(dev)
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                llm.prefill(ids)
                torch.cuda.synchronize(dev)
            rows = {}
            for e in prof.key_averages():
                t = getattr(e, "device_time_total", None) or getattr(e, "cuda_time_total", 0)
                if t > 0 and e.count > 0 and not e.key.startswith("cuda"):
                    rows[e.key] = (e.count, t)
            total = sum(t for _, t in rows.values())
            print(f"== prefill mode {mode}: {total / 1000:.3f} ms of kernel time, {PROMPT} tokens, {args.layers} layers")
            for name, (n, t) in sorted(rows.items(), key=lambda kv: -kv[1][1])[:12]:
                print(f"{t / 1000:9.3f} ms {100 * t / total:5.1f}% {n:5d} x {t / n:8.2f} us  {name[:90]}")
            llm.prefill_graphs.clear()


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.profile_kernel:
        profile_kernel(args)
        return
    if args.batch_sweep:
        batch_sweep(args, rank, world, local)
        return
    if args.profile_gemm:
        profile_gemm(args.profile_gemm)
        return
    if args.config0:
        config0(args)
        return
    if args.profile_prefill:
        profile_prefill(args)
        return
    if args.profile_attention:
        b, ctx = (int(v) for v in args.profile_attention.split(","))
        profile_attention(b, ctx)
        return
    import torch
    import torch.distributed as dist

    from moss_tts._runtime.config import DecoderConfig
    from moss_tts._runtime.engine import TensorParallel, shard_weights
    from moss_tts._runtime.llm import FastLLM
    from moss_tts._runtime import native
    from moss_tts._runtime.weights import DecoderWeights

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        group = dist.group.WORLD
        dist.all_reduce(torch.ones(1, device=dev))  # NCCL communicator up before graph capture
    cfg = DecoderConfig().with_(num_layers=args.layers)
    max_length = max_length_for(args)
    with torch.inference_mode():
        full = DecoderWeights.random(cfg, dev, seed=0, preset="gptq")
        weights = shard_weights(full, rank, world)
        del full
        torch.cuda.empty_cache()
        tp = TensorParallel(rank, world, group)
        llm = FastLLM(weights, max_length=max_length, greedy=True, tp=tp)
        eng = llm.engine
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        eng.kv[:, :, :, :PROMPT].copy_(torch.randn(eng.kv[:, :, :, :PROMPT].shape, generator=g, device=dev))
        ids0 = torch.full((33,), 17, dtype=torch.long)
        ids0[0] = cfg.audio_assistant_gen_slot_token_id
        eng.set_inputs(ids0, PROMPT, 1, -1)
        eng.capture(advance=True)
        llm.warmup()  # the public-API graph (FastLLM.step / step_host)
        stream = torch.cuda.current_stream(dev)

        # ---------------- device-resident throughput: W warm-up + K timed graph replays
        eng.set_inputs(ids0, PROMPT, 1, -1)
        for _ in range(args.warmup):
            eng.run(advance=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            e0.record(stream)
            for _ in range(args.steps):
                eng.run(advance=True)
            e1.record(stream)
            torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = float(ms.item())
        value = args.steps / (ms / 1000.0)
        status = int(eng.status.item())

        # ---------------- end to end through the public API with host buffers
        host_ids = ids0.clone().pin_memory()
        pos, alen, delay = PROMPT, 1, -1
        for _ in range(args.warmup):
            out = llm.step_host(host_ids, pos, alen, delay)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for s in range(args.steps):
            out = llm.step_host(host_ids, PROMPT + s, alen, delay)
            host_ids.copy_(out.reshape(-1))
            alen += 1
        f1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = torch.tensor([f0.elapsed_time(f1)], device=dev)
        if world > 1:
            dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        e2e_value = args.steps / (float(e2e_ms.item()) / 1000.0)

        # ---------------- dominant kernel: fused add+norm+gate/up+SiLU W4A16 GEMV on the packed
        # tiles, one launch per layer (each layer's 58 MB of weights: cold in L2), CUDA events
        lw0 = weights.layers[0].gate_up
        x = torch.randn(cfg.hidden_size, device=dev).bfloat16()
        r = torch.randn(cfg.hidden_size, device=dev).bfloat16()
        summed = torch.empty_like(x)
        mid = torch.empty(lw0.n // 2, device=dev, dtype=torch.bfloat16)
        # captured in a CUDA graph (as inside the decode step) so host launch overhead is not timed
        side = torch.cuda.Stream(dev)

        def gate_up(lw):
            packed_gate_up(native, lw, x, r, summed, mid, eng.w4_workspace, native.FLAG_PDL, side.cuda_stream)
        with torch.cuda.stream(side):
            for lw in weights.layers:
                gate_up(lw)
        torch.cuda.synchronize(dev)
        kgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(kgraph, stream=side):
            for lw in weights.layers:
                gate_up(lw)
        kgraph.replay()
        torch.cuda.synchronize(dev)
        reps = 5
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(stream)
        for _ in range(reps):
            kgraph.replay()
        k1.record(stream)
        torch.cuda.synchronize(dev)
        kernel_us = k0.elapsed_time(k1) * 1000 / (reps * len(weights.layers))
        del kgraph

        # ---------------- the 32 steps after audio_start as one graph (FirstAudioGraph)
        first_audio = None
        if world == 1:
            from moss_tts._runtime.first_audio_graph import FirstAudioGraph
            fa = FirstAudioGraph(llm, 1024)
            fa.warmup()
            start_row = torch.full((1, 1, 33), cfg.audio_pad_code, dtype=torch.long, device=dev)
            start_row[0, 0, 0] = cfg.audio_start_token_id
            for _ in range(2):
                fa.run(start_row, PROMPT)
            torch.cuda.synchronize(dev)
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            for _ in range(5):
                fa.run(start_row, PROMPT)
            a1.record(stream)
            torch.cuda.synchronize(dev)
            fms = a0.elapsed_time(a1) / 5
            first_audio = {"ms_per_32_steps": round(fms, 3), "ms_per_step": round(fms / 32, 4),
                           "positions": f"{PROMPT}..{PROMPT + 31}", "sampling": "greedy",
                           "reference_published_ms": 60.39,
                           "reference_note": "H200 NVL, G32 W4A8, first 32 decode steps after audio start "
                                             "(docs/benchmark.json:86)"}
            fa.graph = None
            del fa

        # ---------------- prefill of the 512-token prompt (FastLLM.prefill, one GPU)
        prefill = None
        if world == 1 and not args.no_prefill:
            g2 = torch.Generator().manual_seed(3)
            pids = torch.full((1, PROMPT, 33), 1024, dtype=torch.long)
            pids[0, :, 0] = torch.randint(0, cfg.vocab_size, (PROMPT,), generator=g2)
            pids[0, :, 1:] = torch.randint(0, 1025, (PROMPT, 32), generator=g2)
            pids = pids.to(dev)
            preps, pms = 5, {}
            for mode in ("bf16", "dequant", "w4"):
                llm.prefill_mode = mode
                for _ in range(2):
                    llm.prefill(pids)
                torch.cuda.synchronize(dev)
                p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                p0.record(stream)
                for _ in range(preps):
                    llm.prefill(pids)
                p1.record(stream)
                torch.cuda.synchronize(dev)
                pms[mode] = p0.elapsed_time(p1) / preps
                llm.prefill_graphs.clear()
            llm.prefill_mode = "auto"
            prefill = {"prompt_tokens": PROMPT, "ms": round(pms["bf16"], 3),
                       "tokens_per_s": round(PROMPT / pms["bf16"] * 1000, 1), "reps": preps,
                       "path": "resident bf16 weights (bit-exact W4 dequantization, once) + bf16 GEMM (cuBLAS), "
                               "prefill QK-norm/RoPE/KV and causal attention kernels",
                       "dequant_per_call_ms": round(pms["dequant"], 3), "w4_gemm_ms": round(pms["w4"], 3),
                       "reference_published_ms": 6.83,
                       "reference_note": "H200 NVL, BF16 prefill of the G32 preset (docs/benchmark.json:85)"}
    # the BF16 preset (config 3 is timed in both formats), after releasing the W4A16 engine's graphs
    bf16 = None
    if not args.no_bf16:
        llm.graph = None
        eng.graph = eng.graph_advance = None
        torch.cuda.synchronize(dev)
        b_val, b_ms, b_bytes, b_status = bf16_step_rate(args, cfg, dev, rank, world, group, max_length)
        pk, _ = measured_peaks()
        bf16 = {"value": round(b_val, 3), "unit": UNIT, "ms_per_step": round(b_ms, 4), "status": b_status,
                "step_bytes_per_gpu": b_bytes, "hbm_roofline_frac": round(b_bytes / (b_ms * 1e-3) / 1e9 / pk, 4)}
    peak, peak_kind = measured_peaks()
    gu_bytes = gate_up_bytes(lw0.k, lw0.n)
    achieved = gu_bytes / (kernel_us * 1e-6) / 1e9
    traffic = None
    tf = REPO / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(f"gate_up_tp{world}")
    step_bytes = weights.layer_bytes() + weights.head_audio.numel() * 2 + 2 * cfg.hidden_size * 2 \
        + 147456 // world * (PROMPT + args.warmup + args.steps // 2) * args.layers // 36
    if world > 1:
        dist.barrier()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads()
        cpu_steps = 3
        v, setup = cpu_oracle_run(args.layers, cpu_steps, 1, threads)
        cpu = {"value": round(v, 4), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": cpu_sample_text(args.layers, cpu_steps, threads), "setup_s": round(setup, 1)}
    # embedding, per layer q/k/v, attention (+ o_proj when folded), o_proj, gate/up, down; heads; advance
    per_layer = 4 if getattr(eng, "fused_oproj", False) else 5
    launches = 3 + per_layer * args.layers
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(args.layers, world, max_length),
        "step_bytes_per_gpu": step_bytes,
        "hbm_roofline_frac": round(step_bytes / (ms / args.steps * 1e-3) / 1e9 / peak, 4),
        "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": 36 * 8,
                "d2h_bytes_per_step": 33 * 8},
        "roofline": {"bound": "hbm", "kernel": "mt_w4a16_linear_packed (add+RMSNorm+gate/up+SiLU, N=%d K=%d)" % (lw0.n, lw0.k),
                     "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "bytes_per_launch": gu_bytes,
                     "launch_us": round(kernel_us, 3)},
        "cpu_baseline": cpu,
        "bf16": bf16,
        "prefill": prefill,
        "first_audio": first_audio,
        "clocks": clocks.summary(),
        "gpu_launches": launches * args.steps,
        "status": status,
        "reference_published": {"value": 530.0, "unit": UNIT, "hardware": "H200 NVL",
                                "note": "reference G32 W4A8 first 32 decode steps (docs/benchmark.json:86)"},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    # graphs holding NCCL work are released before the process group goes away
    eng.graph = eng.graph_advance = llm.graph = None
    del llm, eng
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
