"""Batched decode engine: `batch` independent sequences with ragged contexts in one step.

The reference decodes one request at a time (``FastLLM``, ``src/moss_tts/_runtime/llm.py:227-287``);
this engine runs the same step for B sequences at once, each with its own position, audio
length and delay length (ragged static KV caches). Per step, all PDL-chained and capturable:

    embedding_sum(ids [B, 33])                                     -> emb [B, H]
    per layer:  [add +] RMSNorm + QKV projection                   -> qkv [B, 6144]
                QK-norm/RoPE/KV-write + cluster attention over each sequence's own context
                o_proj                                             -> proj  [TP: all-reduce]
                add + RMSNorm + gate/up + SiLU*up                  -> mid
                down                                               -> mlp   [TP: all-reduce]
    heads: add + final RMSNorm, text/audio logits (plain bf16 GEMMs, as the reference's
           F.linear heads), greedy ids + delay masks per sequence  -> next_ids [B, 33]

Projections: below ``gemm_min_batch`` (default 5) sequences run the packed tensor-core GEMV
with its fused norm prologue (``mt_w4a16_linear_packed_rows``: two activation rows share one
pass over the weights, so B = 2 costs about one batch-1 step); from ``gemm_min_batch`` rows
the W4A16 projections run on the tcgen05 GEMM over its load-time packed layout
(``mt_w4a16_gemm_pack`` / ``mt_w4a16_gemm_packed``) after a separate RMSNorm. Shapes the
packed layout does not take (K not a multiple of 256), or ``packed_gemv=False``, use the
GPTQ-layout GEMV (``mt_w4a16_linear``, up to 8 rows). Inputs live in one int64 control block ``[ids B*33 |
positions B | audio_length B | delay_length B]`` (one host-to-device copy per step); the
result is ``next_ids``.
"""
import torch

from . import native
from .engine import CONTROL_IDS, TensorParallel, rope_tables
from .weights import DecoderWeights, Projection


class BatchDecodeEngine:
    """Static-buffer decode step for ``batch`` sequences over (a shard of) W4A16 ``DecoderWeights``."""

    def __init__(self, weights: DecoderWeights, batch: int, max_length: int = 4096, *, pdl: bool = True,
                 tp: TensorParallel | None = None, gemm_min_batch: int = 5, packed_gemv: bool = True):
        cfg = weights.cfg
        cfg.validate()
        if batch < 1 or batch > 128:
            raise ValueError("batch must be 1..128")
        if not all(p.quantized for lw in weights.layers for p in (lw.qkv, lw.out, lw.gate_up, lw.down)):
            raise ValueError("the batched engine runs W4A16 projections")
        self.w, self.cfg, self.batch, self.max_length = weights, cfg, batch, max_length
        self.tp = tp or TensorParallel()
        world = self.tp.world
        dev = weights.device
        self.device = dev
        self.gemm = batch >= gemm_min_batch
        if not self.gemm and batch > 8:
            raise ValueError("more than 8 rows need the tcgen05 GEMM (gemm_min_batch <= batch)")
        layers = weights.layers
        self.rows_packed = packed_gemv and not self.gemm and all(
            p.k % 256 == 0 and 256 <= p.k <= 16384 and (not paired or p.n % 2 == 0)
            for lw in layers for p, paired in ((lw.qkv, False), (lw.out, False), (lw.gate_up, True), (lw.down, False)))
        h, d, B = cfg.hidden_size, cfg.head_dim, batch
        self.nq, self.nkv = cfg.num_heads // world, cfg.num_kv_heads // world
        self.n_cb = cfg.n_vq // world
        self.cb_offset = self.tp.rank * self.n_cb
        self.flags = native.FLAG_PDL if pdl else 0
        bf = dict(device=dev, dtype=torch.bfloat16)
        self.control = torch.zeros(B * (CONTROL_IDS + 3), device=dev, dtype=torch.long)
        self.ids = self.control[:B * CONTROL_IDS].view(B, CONTROL_IDS)
        self.position = self.control[B * CONTROL_IDS:B * (CONTROL_IDS + 1)]
        self.audio_length = self.control[B * (CONTROL_IDS + 1):B * (CONTROL_IDS + 2)]
        self.delay_length = self.control[B * (CONTROL_IDS + 2):]
        self.emb = torch.zeros(B, h, **bf)
        self.res = [torch.zeros(B, h, **bf), torch.zeros(B, h, **bf)]
        self.normed = torch.zeros(B, h, **bf)
        self.qkv = torch.zeros(B, (self.nq + 2 * self.nkv) * d, **bf)
        self.attn = torch.zeros(B, self.nq * d, **bf)
        self.proj = torch.zeros(B, h, **bf)
        self.mid = torch.zeros(B, weights.layers[0].gate_up.n // 2, **bf)
        self.mlp = torch.zeros(B, h, **bf)
        self.hidden = torch.zeros(B, h, **bf)
        n_layers = len(weights.layers)
        self.kv = torch.zeros((n_layers, 2, B, self.nkv, max_length, d), **bf)
        self.cos, self.sin = (t.to(dev) for t in rope_tables(max_length, d, cfg.rope_theta))
        rep = self.nq // self.nkv
        self.partial = torch.empty(B * self.nkv * rep * d, device=dev, dtype=torch.float32)
        self.lse = torch.empty(B * self.nkv * rep, device=dev, dtype=torch.float32)
        self.tickets = torch.zeros(B * self.nkv, device=dev, dtype=torch.int32)
        self.text_ids = torch.tensor([cfg.audio_assistant_gen_slot_token_id,
                                      cfg.audio_assistant_delay_slot_token_id], device=dev, dtype=torch.long)
        self.text_logits = torch.zeros(B, 2, **bf)
        self.audio_logits = torch.zeros(B, self.n_cb * cfg.audio_vocab_size, **bf)
        self.next_ids = torch.zeros(B, CONTROL_IDS, device=dev, dtype=torch.long)
        self.status = torch.zeros(1, device=dev, dtype=torch.int32)
        ws = 256
        self.packed = {}  # id(projection) -> packed layout of the tcgen05 GEMM (repacked once)
        if self.gemm:
            s = torch.cuda.current_stream(dev).cuda_stream
            for lw in weights.layers:
                for p, paired in ((lw.qkv, False), (lw.out, False), (lw.gate_up, True), (lw.down, False)):
                    mode = native.LINEAR_PAIRED if paired else 0
                    ws = max(ws, native.w4a16_gemm_workspace(B, p.n, p.k, mode))
                    t = torch.empty(native.w4a16_gemm_pack_size(p.n, p.k, mode), device=dev, dtype=torch.uint8)
                    native.call("mt_w4a16_gemm_pack", p.qweight.data_ptr(), p.scales.data_ptr(), native.ptr(p.qzeros),
                                p.n, p.k, mode, t.data_ptr(), s)
                    self.packed[id(p)] = t
        if self.rows_packed:  # the packed GEMV's tiles (shared with a batch-1 engine on the same weights)
            for lw in layers:
                for p, paired in ((lw.qkv, False), (lw.out, False), (lw.gate_up, True), (lw.down, False)):
                    p.packed_tiles(paired)
                    ws = max(ws, native.w4a16_packed_size(p.n, p.k, p.qzeros is not None,
                                                          native.LINEAR_PAIRED if paired else 0)[1])
        self.gemm_workspace = torch.zeros(ws, device=dev, dtype=torch.uint8)
        self.graph = None
        self.graph_advance = None
        self._host_control = torch.zeros(B * (CONTROL_IDS + 3), dtype=torch.long, pin_memory=True)
        self._host_next = torch.zeros(B, CONTROL_IDS, dtype=torch.long, pin_memory=True)
        self._staged = None

    # ------------------------------------------------------------------ kernels
    def _linear(self, p: Projection, x, y, *, residual=None, norm=None, summed=None, paired=False):
        eps = float(self.cfg.rms_norm_eps)
        s = torch.cuda.current_stream(self.device).cuda_stream
        B = self.batch
        if self.gemm:
            if norm is not None:
                native.call("mt_rmsnorm", x.data_ptr(), native.ptr(residual), norm.data_ptr(), native.ptr(summed),
                            self.normed.data_ptr(), B, x.shape[-1], eps, self.flags, s)
                x = self.normed
            native.call("mt_w4a16_gemm_packed", x.data_ptr(), self.packed[id(p)].data_ptr(), y.data_ptr(), B, p.n,
                        p.k, native.LINEAR_PAIRED if paired else 0, self.gemm_workspace.data_ptr(), self.flags, s)
            return
        mode = (native.LINEAR_NORM if norm is not None else 0) | (native.LINEAR_ADD if residual is not None else 0)
        mode |= native.LINEAR_PAIRED if paired else 0
        if self.rows_packed:
            native.call("mt_w4a16_linear_packed_rows", x.data_ptr(), native.ptr(residual), native.ptr(norm), eps,
                        native.ptr(summed), p.packed_tiles(paired).data_ptr(), 1 if p.qzeros is not None else 0,
                        y.data_ptr(), B, p.n, p.k, mode, self.gemm_workspace.data_ptr(), self.flags, s)
            return
        native.call("mt_w4a16_linear", x.data_ptr(), native.ptr(residual), native.ptr(norm), eps, native.ptr(summed),
                    p.qweight.data_ptr(), p.scales.data_ptr(), native.ptr(p.qzeros), y.data_ptr(), B, p.n, p.k, 32,
                    mode, self.flags, s)

    def launch_step(self) -> None:
        """Enqueue one batched decode step on the current stream (no host synchronisation)."""
        cfg, w, B = self.cfg, self.w, self.batch
        s = torch.cuda.current_stream(self.device).cuda_stream
        eps = float(cfg.rms_norm_eps)
        native.call("mt_embedding_sum", self.ids.data_ptr(), w.embed_text.data_ptr(), w.embed_audio.data_ptr(),
                    self.emb.data_ptr(), B, cfg.hidden_size, w.embed_text.shape[0], w.embed_audio.shape[1],
                    cfg.n_vq, self.status.data_ptr(), self.flags, s)
        res, nxt = self.emb, 0
        for i, lw in enumerate(w.layers):
            if i == 0:
                self._linear(lw.qkv, self.emb, self.qkv, norm=lw.input_norm)
            else:
                out = self.res[nxt]
                self._linear(lw.qkv, self.mlp, self.qkv, residual=res, norm=lw.input_norm, summed=out)
                res, nxt = out, 1 - nxt
            native.call("mt_attention_decode", self.qkv.data_ptr(), lw.q_norm.data_ptr(), lw.k_norm.data_ptr(),
                        self.cos.data_ptr(), self.sin.data_ptr(), self.position.data_ptr(),
                        self.kv[i, 0].data_ptr(), self.kv[i, 1].data_ptr(), self.attn.data_ptr(),
                        self.partial.data_ptr(), self.lse.data_ptr(), self.tickets.data_ptr(), B, self.nq, self.nkv,
                        self.max_length, 1, eps, self.status.data_ptr(), self.flags, s)
            self._linear(lw.out, self.attn, self.proj)
            self.tp.all_reduce(self.proj)
            out = self.res[nxt]
            self._linear(lw.gate_up, self.proj, self.mid, residual=res, norm=lw.post_norm, summed=out, paired=True)
            res, nxt = out, 1 - nxt
            self._linear(lw.down, self.mid, self.mlp)
            self.tp.all_reduce(self.mlp)
        native.call("mt_rmsnorm", self.mlp.data_ptr(), res.data_ptr(), w.final_norm.data_ptr(), None,
                    self.hidden.data_ptr(), B, cfg.hidden_size, eps, self.flags, s)
        # the heads are plain bf16 GEMMs (the reference's F.linear, llm.py:271-274)
        torch.matmul(self.hidden, w.head_audio.t(), out=self.audio_logits)
        torch.matmul(self.hidden, w.head_text_rows.t(), out=self.text_logits)
        native.call("mt_heads_select", self.text_logits.data_ptr(), self.audio_logits.data_ptr(),
                    self.text_ids.data_ptr(), self.audio_length.data_ptr(), self.delay_length.data_ptr(),
                    self.next_ids.data_ptr(), B, 2, self.n_cb, cfg.audio_vocab_size, self.cb_offset, cfg.n_vq,
                    cfg.audio_assistant_delay_slot_token_id, cfg.audio_end_token_id, cfg.audio_pad_code,
                    1 if self.tp.rank == 0 else 0, 0, s)
        if self.tp.world > 1:
            self.tp.all_reduce(self.next_ids)

    def launch_advance(self) -> None:
        """Device-side advance of every sequence (ids fed back, position += 1, delay bookkeeping
        as ``first_audio_graph._advance``, ``first_audio_graph.py:14-27``), one launch."""
        native.call("mt_decode_advance", self.control.data_ptr(), self.next_ids.data_ptr(), CONTROL_IDS, self.batch,
                    self.cfg.audio_assistant_delay_slot_token_id, self.flags,
                    torch.cuda.current_stream(self.device).cuda_stream)

    # ------------------------------------------------------------------ graphs and I/O
    def capture(self, advance: bool = False) -> None:
        saved = self.control.clone()
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

    def set_inputs(self, ids, positions, audio_length, delay_length) -> None:
        """Stage one step for every sequence: ids [B, 33], positions / audio_length /
        delay_length [B]; a single host-to-device copy of the control block."""
        B = self.batch
        ids = torch.as_tensor(ids, dtype=torch.long).reshape(B, CONTROL_IDS)
        cols = [torch.as_tensor(v, dtype=torch.long).reshape(-1).expand(B) for v in (positions, audio_length,
                                                                                  delay_length)]
        if int(cols[0].min()) < 0 or int(cols[0].max()) >= self.max_length:
            raise ValueError("KV capacity exceeded")
        if self._staged is not None:
            self._staged.synchronize()
        hc = self._host_control
        hc[:B * CONTROL_IDS].copy_(ids.reshape(-1))
        for j, col in enumerate(cols):
            hc[B * (CONTROL_IDS + j):B * (CONTROL_IDS + j + 1)].copy_(col)
        self.control.copy_(hc, non_blocking=True)
        self._staged = torch.cuda.Event()
        self._staged.record(torch.cuda.current_stream(self.device))

    def read_next_ids(self) -> torch.Tensor:
        self._host_next.copy_(self.next_ids, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._host_next

    def step(self, ids, positions, audio_length, delay_length) -> torch.Tensor:
        """One decode step of every sequence; returns next ids [B, 33] (device tensor)."""
        self.set_inputs(ids, positions, audio_length, delay_length)
        self.run()
        return self.next_ids.clone()
