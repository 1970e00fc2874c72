"""Batch-1 decode engine: static device buffers, the per-step kernel sequence, CUDA graphs.

On one GPU with W4 weights a decode step is three launches: ``mt_embedding_sum``, the whole
layer stack as one persistent kernel (``mt_decode_layers``: one CTA per SM streaming every
layer's packed weights without a break, grid barriers between the sublayers) and
``mt_heads_greedy``. Otherwise (tensor parallelism, the BF16 preset, ``persistent=False``)
one decode step (reference ``FastLLM._decode`` + ``hidden``, ``src/moss_tts/_runtime/llm.py:227-287``,
fused-residual order) is 2 + 5 * layers launches, all PDL-chained and capturable:

    embedding_sum(ids)                                         -> emb
    per layer:  W4A16 [add +] RMSNorm + QKV projection         -> qkv  (residual stream updated)
                fused QK-norm/RoPE/KV-write + split-K attention -> attn
                W4A16 o_proj                                   -> proj  [TP: all-reduce]
                W4A16 add + RMSNorm + gate/up + SiLU*up         -> mid   (residual stream updated)
                W4A16 down                                     -> mlp   [TP: all-reduce]
    heads: add + final RMSNorm, text/audio logits, greedy ids, delay masks -> next_ids

The step's inputs live in one int64 control block ``[ids(1 + n_vq), position, audio_length,
delay_length]`` so a host request is a single host-to-device copy; the step's result is
``next_ids`` (one device-to-host copy). Tensor parallelism (``TensorParallel``) shards heads,
KV heads, intermediate columns and codebooks; partial o_proj/down outputs are summed with
NCCL all-reduce, and each rank writes only its own codebooks' ids (zeros elsewhere), summed
by one int64 all-reduce.
"""
import ctypes
import os

import torch

from . import native
from .weights import DecoderWeights, Projection

CONTROL_IDS = 33


def rope_tables(max_length: int, head_dim: int = 128, theta: float = 1e6):
    """bf16 cos/sin tables built exactly as transformers' default rotary embedding does on
    the CPU (fp32 inverse frequencies, fp32 ``freqs = inv_freq * position``, fp32 cos/sin,
    bf16 cast); evaluated once on the host instead of per step on the device."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float) / head_dim))
    pos = torch.arange(max_length, dtype=torch.float32)
    freqs = (inv[None, :, None].float() @ pos[None, None, :].float()).transpose(1, 2)[0]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


class TensorParallel:
    """Rank/world of a tensor-parallel group plus the all-reduce used between sublayers."""

    def __init__(self, rank: int = 0, world: int = 1, group=None):
        self.rank, self.world, self.group = rank, world, group

    def all_reduce(self, t: torch.Tensor) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, group=self.group)


class PeerExchange:
    """Peer-memory exchange of the row-parallel projections' partial rows (``mt_tp_exchange``).

    One symmetric allocation per rank (``torch.distributed._symmetric_memory``, mapped on every
    rank of the group) of 8-byte cells ``[slots][world][width / 2]``, each {bf16 pair, uint32
    flag}. The producer GEMV writes its rows into every rank's cells with this step's flag;
    the consumer GEMV polls its own cells for the flag and sums the ranks' rows.
    """

    def __init__(self, tp: TensorParallel, slots: int, width: int, device):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.world, self.rank, self.slots, self.width = tp.world, tp.rank, slots, width
        self.buf = symm_mem.empty(slots * tp.world * width * 4, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, tp.group or dist.group.WORLD)
        self.ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.epoch = torch.zeros(1, device=device, dtype=torch.long)  # steps started on this rank
        torch.cuda.synchronize(device)
        dist.barrier(group=tp.group)

    def desc(self, in_slot: int = -1, out_slot: int = -1) -> "native.TpExchange":
        d = native.TpExchange()
        for r, p in enumerate(self.ptrs):
            d.recv[r] = p
        d.epoch = self.epoch.data_ptr()
        d.world, d.rank, d.in_slot, d.out_slot, d.slot_elems = self.world, self.rank, in_slot, out_slot, self.width
        return d


def shard_weights(w: DecoderWeights, rank: int, world: int) -> DecoderWeights:
    """Megatron-style shard of the decoder for tensor-parallel rank ``rank`` of ``world``:
    q/k/v heads and gate/up rows column-parallel, o_proj/down columns row-parallel,
    audio codebooks split across ranks, norms and embeddings replicated."""
    if world == 1:
        return w
    cfg = w.cfg
    if cfg.num_kv_heads % world or cfg.n_vq % world or cfg.intermediate_size % (64 * world):
        raise ValueError("world size must divide the KV heads, codebooks and intermediate size")
    d, nq, nkv, i = cfg.head_dim, cfg.num_heads // world, cfg.num_kv_heads // world, cfg.intermediate_size
    from .weights import LayerWeights

    def cat_rows(parts):
        def c(attr):
            ts = [getattr(p, attr) for p in parts]
            return None if ts[0] is None else torch.cat(ts, 0).contiguous()
        return Projection(sum(p.n for p in parts), parts[0].k, c("qweight"), c("scales"), c("qzeros"), c("weight"))

    layers = []
    for lw in w.layers:
        q0, k0, v0 = rank * nq * d, cfg.num_heads * d + rank * nkv * d, (cfg.num_heads + cfg.num_kv_heads) * d + rank * nkv * d
        qkv = cat_rows([lw.qkv.rows(q0, q0 + nq * d), lw.qkv.rows(k0, k0 + nkv * d), lw.qkv.rows(v0, v0 + nkv * d)])
        il = i // world
        gu = cat_rows([lw.gate_up.rows(rank * il, (rank + 1) * il), lw.gate_up.rows(i + rank * il, i + (rank + 1) * il)])
        layers.append(LayerWeights(lw.input_norm, lw.post_norm, lw.q_norm, lw.k_norm, qkv,
                                   lw.out.cols(rank * nq * d, (rank + 1) * nq * d), gu,
                                   lw.down.cols(rank * il, (rank + 1) * il)))
    cb = cfg.n_vq // world
    v = cfg.audio_vocab_size
    head_audio = w.head_audio[rank * cb * v:(rank + 1) * cb * v].contiguous()
    out = DecoderWeights(cfg, layers, w.final_norm, w.embed_text, w.embed_audio, w.head_text_rows,
                         head_audio, w.head_text, w.preset, dict(w.meta))
    out.meta.update(tp_rank=rank, tp_world=world)
    return out


class DecodeEngine:
    """Static-buffer decode step for one sequence over (a shard of) ``DecoderWeights``."""

    def __init__(self, weights: DecoderWeights, max_length: int = 1024, *, splits: int | None = None,
                 pdl: bool = True, tp: TensorParallel | None = None, persistent: bool | None = None):
        cfg = weights.cfg
        cfg.validate()
        self.w, self.cfg, self.max_length = weights, cfg, max_length
        self.tp = tp or TensorParallel()
        world = self.tp.world
        dev = weights.device
        self.device = dev
        h, d = cfg.hidden_size, cfg.head_dim
        self.nq, self.nkv = cfg.num_heads // world, cfg.num_kv_heads // world
        self.n_cb = cfg.n_vq // world
        self.cb_offset = self.tp.rank * self.n_cb
        self.flags = native.FLAG_PDL if pdl else 0
        bf = dict(device=dev, dtype=torch.bfloat16)
        # control block: ids | position | audio_length | delay_length
        self.control = torch.zeros(CONTROL_IDS + 3, device=dev, dtype=torch.long)
        self.ids = self.control[:CONTROL_IDS]
        self.position = self.control[CONTROL_IDS:CONTROL_IDS + 1]
        self.audio_length = self.control[CONTROL_IDS + 1:CONTROL_IDS + 2]
        self.delay_length = self.control[CONTROL_IDS + 2:CONTROL_IDS + 3]
        self.emb = torch.zeros(h, **bf)
        self.res = [torch.zeros(h, **bf), torch.zeros(h, **bf)]
        self.qkv = torch.zeros((self.nq + 2 * self.nkv) * d, **bf)
        self.attn = torch.zeros(self.nq * d, **bf)
        self.proj = torch.zeros(h, **bf)
        self.mid = torch.zeros(weights.layers[0].gate_up.n // 2, **bf)
        self.mlp = torch.zeros(h, **bf)
        self.hidden = torch.zeros(h, **bf)
        n_layers = len(weights.layers)
        self.kv = torch.zeros((n_layers, 2, self.nkv, max_length, d), **bf)
        self.cos, self.sin = (t.to(dev) for t in rope_tables(max_length, d, cfg.rope_theta))
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.splits = splits or max(1, min(64, (sms + self.nkv - 1) // self.nkv))
        rep = self.nq // self.nkv
        self.partial = torch.empty(self.nkv * self.splits * rep * d, device=dev, dtype=torch.float32)
        self.lse = torch.empty(self.nkv * self.splits * rep, device=dev, dtype=torch.float32)
        self.tickets = torch.zeros(self.nkv + 1, device=dev, dtype=torch.int32)
        self.best = torch.zeros(1 + self.n_cb, device=dev, dtype=torch.int64)
        self.text_ids = torch.tensor([cfg.audio_assistant_gen_slot_token_id,
                                      cfg.audio_assistant_delay_slot_token_id], device=dev, dtype=torch.long)
        self.text_logits = torch.zeros(2, **bf)
        self.audio_logits = torch.zeros(self.n_cb * cfg.audio_vocab_size, **bf)
        self.next_ids = torch.zeros(CONTROL_IDS, device=dev, dtype=torch.long)
        self.status = torch.zeros(1, device=dev, dtype=torch.int32)
        # Non-greedy decoding: (text T, top-k, top-p, audio T, top-k, top-p) of the device sampler
        # (mt_heads_sample) run after the heads, or None for the heads kernel's greedy ids. The
        # seed (drawn from torch's default generator, so torch.manual_seed fixes it) keys the
        # sampler's counter-based generator together with the position.
        self.sampling = None
        self.seed = torch.randint(0, 2 ** 62, (1,), dtype=torch.int64).to(dev)
        self.graph = None
        self.graph_advance = None
        self._host_control = torch.zeros(CONTROL_IDS + 3, dtype=torch.long, pin_memory=True)
        self._host_next = torch.zeros(CONTROL_IDS, dtype=torch.long, pin_memory=True)
        self._scalars = torch.zeros(3, dtype=torch.long, pin_memory=True)
        self._staged = None
        # batch-1 W4 projections run on the packed layout; one workspace serves them all
        ws = 0
        for lw in weights.layers:
            for p, paired in ((lw.qkv, False), (lw.out, False), (lw.gate_up, True), (lw.down, False)):
                if self._packed_ok(p, paired):
                    p.packed_tiles(paired)
                    ws = max(ws, native.w4a16_packed_size(p.n, p.k, p.qzeros is not None,
                                                          native.LINEAR_PAIRED if paired else 0)[1])
        self.w4_workspace = torch.zeros(max(ws, 16), device=dev, dtype=torch.uint8)
        # Tensor parallelism: the row-parallel partials travel through peer memory (o_proj and
        # every down but the last; that one feeds the heads through an NCCL all-reduce).
        self.exchange = None
        if world > 1 and os.environ.get("MT_TP_EXCHANGE", "p2p") != "nccl" and weights.layers[0].out.quantized \
                and all(self._packed_ok(p, False) for lw in weights.layers for p in (lw.out, lw.down)):
            self.exchange = PeerExchange(self.tp, 2 * len(weights.layers), h, dev)
        # Single GPU, W4 weights: the whole layer stack can run as one persistent launch
        # (mt_decode_layers); None follows MT_PERSISTENT (default: the per-sublayer launch chain)
        if persistent is None:
            persistent = os.environ.get("MT_PERSISTENT", "0") == "1"
        self.persistent = persistent and world == 1 and all(
            self._packed_ok(p, paired) for lw in weights.layers
            for p, paired in ((lw.qkv, False), (lw.out, False), (lw.gate_up, True), (lw.down, False)))
        if self.persistent:
            self._build_layer_table()
        # One GPU, packed W4 o_proj, MT_FUSED_OPROJ=1: the attention kernel also runs the o_proj
        # (split over the KV heads, mt_attention_oproj_decode), one launch fewer per layer. Off by
        # default: measured slower (594 against 669 steps/s), since the o_proj weights then stream
        # into the 64 attention SMs only, while the separate GEMV prefetches them on all 148.
        rep_ = self.nq // self.nkv
        self.fused_oproj = (world == 1 and os.environ.get("MT_FUSED_OPROJ", "0") == "1"
                            and os.environ.get("MT_ATTN_TC", "1") != "0" and rep_ in (2, 4)
                            and h % 128 == 0 and all(self._packed_ok(lw.out, False) for lw in weights.layers))
        if self.fused_oproj:
            self.oproj_ws = torch.zeros(self.nkv * h * 4 + 64, device=dev, dtype=torch.uint8)

    # ------------------------------------------------------------------ kernels
    def _build_layer_table(self) -> None:
        """Device table of ``mt_decode_layer`` entries (packed projections, norms, caches) and the
        zero-filled workspace of the persistent layer-stack kernel."""
        w, n = self.w, len(self.w.layers)
        table = (native.DecodeLayer * n)()
        for i, lw in enumerate(w.layers):
            e = table[i]
            e.qkv, e.out = lw.qkv.packed_tiles(False).data_ptr(), lw.out.packed_tiles(False).data_ptr()
            e.gate_up, e.down = lw.gate_up.packed_tiles(True).data_ptr(), lw.down.packed_tiles(False).data_ptr()
            e.input_norm, e.post_norm = lw.input_norm.data_ptr(), lw.post_norm.data_ptr()
            e.q_norm, e.k_norm = lw.q_norm.data_ptr(), lw.k_norm.data_ptr()
            e.k_cache, e.v_cache = self.kv[i, 0].data_ptr(), self.kv[i, 1].data_ptr()
        self.layer_table = torch.frombuffer(bytearray(bytes(table)), dtype=torch.uint8).to(self.device)
        self.has_zeros = 1 if w.layers[0].qkv.qzeros is not None else 0
        if any((p.qzeros is not None) != bool(self.has_zeros)
               for lw in w.layers for p in (lw.qkv, lw.out, lw.gate_up, lw.down)):
            raise ValueError("all projections must share one zero-point format")
        nbytes = native.decode_layers_workspace(n, self.cfg.intermediate_size)
        self.layers_workspace = torch.zeros(nbytes, device=self.device, dtype=torch.uint8)
        self.residual = torch.zeros(self.cfg.hidden_size, device=self.device, dtype=torch.bfloat16)

    def reset_workspace(self) -> None:
        """Zero the persistent kernel's workspace (needed only after a call reported a timeout)."""
        if self.persistent:
            self.layers_workspace.zero_()

    @staticmethod
    def _packed_ok(p: Projection, paired: bool) -> bool:
        return p.quantized and p.k % 256 == 0 and 256 <= p.k <= 16384 and (not paired or p.n % 2 == 0)

    def _linear(self, p: Projection, x, y, *, residual=None, norm=None, summed=None, paired=False, tp=None):
        mode = (native.LINEAR_NORM if norm is not None else 0) | (native.LINEAR_ADD if residual is not None else 0)
        mode |= native.LINEAR_PAIRED if paired else 0
        eps = float(self.cfg.rms_norm_eps)
        s = torch.cuda.current_stream(self.device).cuda_stream
        if tp is not None:
            native.call("mt_w4a16_linear_packed_tp", x.data_ptr(), native.ptr(residual), native.ptr(norm), eps,
                        native.ptr(summed), p.packed_tiles(paired).data_ptr(), 1 if p.qzeros is not None else 0,
                        y.data_ptr(), p.n, p.k, mode, self.w4_workspace.data_ptr(), ctypes.byref(tp),
                        self.flags, s)
        elif self._packed_ok(p, paired):
            native.call("mt_w4a16_linear_packed", x.data_ptr(), native.ptr(residual), native.ptr(norm), eps,
                        native.ptr(summed), p.packed_tiles(paired).data_ptr(), 1 if p.qzeros is not None else 0,
                        y.data_ptr(), p.n, p.k, mode, self.w4_workspace.data_ptr(), self.flags, s)
        elif p.quantized:
            native.call("mt_w4a16_linear", x.data_ptr(), native.ptr(residual), native.ptr(norm), eps,
                        native.ptr(summed), p.qweight.data_ptr(), p.scales.data_ptr(), native.ptr(p.qzeros),
                        y.data_ptr(), 1, p.n, p.k, 32, mode, self.flags, s)
        else:
            native.call("mt_bf16_linear", x.data_ptr(), native.ptr(residual), native.ptr(norm), eps,
                        native.ptr(summed), p.weight.data_ptr(), y.data_ptr(), 1, p.n, p.k, mode,
                        self.flags, s)

    def launch_step(self) -> None:
        """Enqueue one decode step on the current stream (no host synchronisation)."""
        cfg, w = self.cfg, self.w
        s = torch.cuda.current_stream(self.device).cuda_stream
        native.call("mt_embedding_sum", self.ids.data_ptr(), w.embed_text.data_ptr(), w.embed_audio.data_ptr(),
                    self.emb.data_ptr(), 1, cfg.hidden_size, w.embed_text.shape[0], w.embed_audio.shape[1],
                    cfg.n_vq, self.status.data_ptr(), self.flags, s)
        eps = float(cfg.rms_norm_eps)
        if self.persistent:
            native.call("mt_decode_layers", self.layer_table.data_ptr(), len(w.layers), cfg.intermediate_size,
                        self.has_zeros, self.emb.data_ptr(), self.position.data_ptr(), self.cos.data_ptr(),
                        self.sin.data_ptr(), self.max_length, eps, self.residual.data_ptr(), self.mlp.data_ptr(),
                        self.layers_workspace.data_ptr(), self.status.data_ptr(), self.flags, s)
            self._launch_heads(self.residual, s)
            return
        res = self.emb
        nxt = 0
        ex, last = self.exchange, len(w.layers) - 1
        if ex is not None:
            ex.epoch.add_(1)  # one step: every exchange slot is expected once more
        for i, lw in enumerate(w.layers):
            if i == 0:
                self._linear(lw.qkv, self.emb, self.qkv, norm=lw.input_norm)
            else:
                out = self.res[nxt]
                tp_in = ex.desc(in_slot=2 * (i - 1) + 1) if ex is not None else None
                self._linear(lw.qkv, self.mlp, self.qkv, residual=res, norm=lw.input_norm, summed=out, tp=tp_in)
                res, nxt = out, 1 - nxt
            k, v = self.kv[i, 0], self.kv[i, 1]
            if self.fused_oproj:
                native.call("mt_attention_oproj_decode", self.qkv.data_ptr(), lw.q_norm.data_ptr(),
                            lw.k_norm.data_ptr(), self.cos.data_ptr(), self.sin.data_ptr(), self.position.data_ptr(),
                            k.data_ptr(), v.data_ptr(), self.attn.data_ptr(), lw.out.packed_tiles(False).data_ptr(),
                            1 if lw.out.qzeros is not None else 0, self.proj.data_ptr(), cfg.hidden_size,
                            self.oproj_ws.data_ptr(), self.nq, self.nkv, self.max_length, eps,
                            self.status.data_ptr(), self.flags, s)
            else:
                native.call("mt_attention_decode", self.qkv.data_ptr(), lw.q_norm.data_ptr(), lw.k_norm.data_ptr(),
                            self.cos.data_ptr(), self.sin.data_ptr(), self.position.data_ptr(), k.data_ptr(),
                            v.data_ptr(), self.attn.data_ptr(), self.partial.data_ptr(), self.lse.data_ptr(),
                            self.tickets.data_ptr(), 1, self.nq, self.nkv, self.max_length, self.splits, eps,
                            self.status.data_ptr(), self.flags, s)
            if self.fused_oproj:  # the projection is already in self.proj
                pass
            elif ex is not None:
                self._linear(lw.out, self.attn, self.proj, tp=ex.desc(out_slot=2 * i))
            else:
                self._linear(lw.out, self.attn, self.proj)
                self.tp.all_reduce(self.proj)
            out = self.res[nxt]
            tp_in = ex.desc(in_slot=2 * i) if ex is not None else None
            self._linear(lw.gate_up, self.proj, self.mid, residual=res, norm=lw.post_norm, summed=out, paired=True,
                         tp=tp_in)
            res, nxt = out, 1 - nxt
            if ex is not None and i < last:
                self._linear(lw.down, self.mid, self.mlp, tp=ex.desc(out_slot=2 * i + 1))
            else:
                self._linear(lw.down, self.mid, self.mlp)
                self.tp.all_reduce(self.mlp)
        self._launch_heads(res, s)
        if self.tp.world > 1:
            self.tp.all_reduce(self.next_ids)

    def _launch_heads(self, res, s) -> None:
        cfg, w, eps = self.cfg, self.w, float(self.cfg.rms_norm_eps)
        native.call("mt_heads_greedy", self.mlp.data_ptr(), res.data_ptr(), w.final_norm.data_ptr(), eps,
                    self.hidden.data_ptr(), w.head_text_rows.data_ptr(), w.head_audio.data_ptr(),
                    self.text_logits.data_ptr(), self.audio_logits.data_ptr(), self.text_ids.data_ptr(),
                    self.audio_length.data_ptr(), self.delay_length.data_ptr(), self.next_ids.data_ptr(),
                    self.best.data_ptr(), self.tickets[self.nkv:].data_ptr(), cfg.hidden_size, 2, self.n_cb,
                    cfg.audio_vocab_size, self.cb_offset, cfg.n_vq, cfg.audio_assistant_delay_slot_token_id,
                    cfg.audio_end_token_id, cfg.audio_pad_code, 1 if self.tp.rank == 0 else 0, self.flags, s)
        if self.sampling is not None:
            tt, tk, tp_, at, ak, ap = self.sampling
            native.call("mt_heads_sample", self.text_logits.data_ptr(), self.audio_logits.data_ptr(),
                        self.text_ids.data_ptr(), self.position.data_ptr(), self.audio_length.data_ptr(),
                        self.delay_length.data_ptr(), self.seed.data_ptr(), self.next_ids.data_ptr(), 1, 2,
                        self.n_cb, cfg.audio_vocab_size, self.cb_offset, cfg.n_vq,
                        cfg.audio_assistant_delay_slot_token_id, cfg.audio_end_token_id, cfg.audio_pad_code,
                        1 if self.tp.rank == 0 else 0, float(tt), int(tk), float(tp_), float(at), int(ak), float(ap),
                        self.flags, s)

    def set_seed(self, seed: int) -> None:
        """Seed of the device sampler (any integer; reduced to 64 bits)."""
        self.seed.fill_(int(seed) & (2 ** 63 - 1))

    def launch_advance(self) -> None:
        """Device-side state advance after a step (feed next_ids back, position += 1, delay
        bookkeeping as ``first_audio_graph._advance``, ``first_audio_graph.py:14-27``), one launch."""
        native.call("mt_decode_advance", self.control.data_ptr(), self.next_ids.data_ptr(), CONTROL_IDS, 1,
                    self.cfg.audio_assistant_delay_slot_token_id, self.flags,
                    torch.cuda.current_stream(self.device).cuda_stream)

    # ------------------------------------------------------------------ graphs
    def capture(self, advance: bool = False) -> None:
        """Warm up on a side stream, then capture the step (optionally + advance) as a graph."""
        saved = self.control.clone()
        kv = None
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for _ in range(2):
                self.launch_step()
                if advance:
                    self.launch_advance()
                self.control.copy_(saved)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.launch_step()
            if advance:
                self.launch_advance()
        self.control.copy_(saved)
        del kv
        if advance:
            self.graph_advance = graph
        else:
            self.graph = graph

    def run(self, advance: bool = False) -> None:
        g = self.graph_advance if advance else self.graph
        if g is not None:
            g.replay()
        else:
            self.launch_step()
            if advance:
                self.launch_advance()

    def set_inputs(self, ids, position: int, audio_length: int, delay_length: int) -> None:
        """Stage one request: a single host-to-device copy of the int64 control block."""
        if not 0 <= position < self.max_length:
            raise ValueError("KV capacity exceeded")
        ids = torch.as_tensor(ids, dtype=torch.long).reshape(-1)
        if ids.numel() != CONTROL_IDS:
            raise ValueError("ids must hold 1 + 32 token ids")
        if ids.is_cuda:
            self.ids.copy_(ids)
            self._scalars.copy_(torch.tensor([position, audio_length, delay_length]), non_blocking=True)
            self.control[CONTROL_IDS:].copy_(self._scalars, non_blocking=True)
            return
        if self._staged is not None:
            self._staged.synchronize()  # the previous copy out of the staging block is done
        self._host_control[:CONTROL_IDS].copy_(ids)
        self._host_control[CONTROL_IDS] = position
        self._host_control[CONTROL_IDS + 1] = audio_length
        self._host_control[CONTROL_IDS + 2] = delay_length
        self.control.copy_(self._host_control, non_blocking=True)
        self._staged = torch.cuda.Event()
        self._staged.record(torch.cuda.current_stream(self.device))

    def health(self, clear: bool = True) -> dict:
        """The device-side failure flags of the steps run so far (synchronises the device).

        ``status``: 1 = a position or an id was out of range (clamped), 3 = a bounded copy wait
        in the attention expired. ``error_word`` (the library's, shared by every call in this
        process): 1 = a bounded pipeline wait expired, 2 = a tensor-parallel exchange poll gave up
        on a dead or late peer, so that step used stale rows. ``clear`` resets both."""
        torch.cuda.synchronize(self.device)
        status = int(self.status.item())
        word = native.error_word(clear=clear)
        if clear:
            self.status.zero_()
        return {"status": status, "error_word": word}

    def read_next_ids(self) -> torch.Tensor:
        """Device-to-host copy of the step result into pinned memory (synchronises)."""
        self._host_next.copy_(self.next_ids, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._host_next.view(1, 1, CONTROL_IDS)

    def step(self, ids, position: int, audio_length: int, delay_length: int) -> torch.Tensor:
        """Run one decode step and return the next ids ``[1, 1, 33]`` (device tensor)."""
        self.set_inputs(ids, position, audio_length, delay_length)
        self.run()
        return self.next_ids.view(1, 1, CONTROL_IDS).clone()

    def reset_cache(self) -> None:
        self.kv.zero_()
