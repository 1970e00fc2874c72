/*
 * moss_tts_b200.h -- C ABI of the MOSS-TTS batch-1 decode kernels for NVIDIA B200 (sm_100a).
 *
 * Library: libmoss_tts_b200.so (moss-tts-optimized_b200/moss_tts/_runtime/). No torch
 * types cross this boundary: tensors are plain device pointers, sizes are ints, the
 * stream is a cudaStream_t passed as void*. Conventions, following the reference's
 * native launcher (src/moss_tts/_runtime/attention_native.cu:91-97):
 *   - every function returns an int cudaError_t (0 = success); invalid arguments
 *     (null pointers, unsupported sizes, misaligned buffers) return
 *     cudaErrorInvalidValue (1) before anything is launched;
 *   - nothing allocates, nothing synchronizes: all work is enqueued on `stream`,
 *     so every call is CUDA-graph capturable; the caller owns all memory;
 *   - bf16 tensors are row-major __nv_bfloat16; int64 ids/positions are device
 *     arrays, read on the device (no host round-trip inside a decode step);
 *   - `flags` bit 0 (MT_FLAG_PDL) launches with programmatic dependent launch so
 *     a kernel's prologue (weight prefetch) overlaps its predecessor's tail.
 *
 * Weight format of the int4 projections (G = 32):
 *   qweight uint8 [N, K/2]  codes, element k in nibble (k & 1) of byte k/2 (the
 *                           reference's export packing, calibration.py:190-191;
 *                           equivalently int32 [N, K/8], element 8i+j in nibble j)
 *   scales  bf16  [N, K/G]
 *   qzeros  uint8 [N, K/(2G)] one 4-bit zero point per group, even group in the
 *                           low nibble; NULL means z = 8 (the reference's signed
 *                           codes with bit 3 flipped: q = code + 8)
 *   W[n][k] = bf16((q - z) * scale)
 */
#ifndef MOSS_TTS_B200_H
#define MOSS_TTS_B200_H

#ifdef __cplusplus
extern "C" {
#endif

#define MT_FLAG_PDL 1
#define MT_FLAG_REGISTER_PIPELINE 2 /* alternative kernels: split-K attention, register-pipelined heads
                                      and bf16 GEMV */
#define MT_LINEAR_NORM 1   /* RMSNorm prologue over each activation row            */
#define MT_LINEAR_ADD 2    /* bf16 residual add before the norm (requires NORM)    */
#define MT_LINEAR_PAIRED 4 /* rows [0,N/2) gate, [N/2,N) up; y = bf16(silu(g)) * u */

/* ABI revision of this header (1). */
int mt_abi_version(void);

/*
 * Diagnostic: copies the library's error word for the current device into *value (1 after a
 * kernel abandoned a bounded wait on its own asynchronous copies, then drained them and
 * returned early; 2 after a tensor-parallel exchange gave up waiting for a peer; 0 otherwise)
 * and clears it when `clear` is non-zero. This one call is synchronous. No counterpart in the
 * reference (its kernels never wait).
 */
int mt_read_error_word(int* value, int clear);

/*
 * Bit-exact dequantization: out bf16 [n, k] = bf16((q - z) * s).
 * Replaces calibrated_backend.unpack_signed + calibrated_quant.dequantize
 * (src/moss_tts/_runtime/calibrated_backend.py:8-13, calibrated_quant.py:41-42).
 */
int mt_dequant_w4(const void* qweight, const void* scales, const void* qzeros, void* out,
                  int n, int k, int group, void* stream);

/*
 * Static G32 scales of a weight matrix w [n, k] (dtype 0 = bf16, 1 = fp32, 2 = fp16):
 * out bf16 [n, k / 32] = bf16(max(absmax of the group, 1e-8) / 7). Offline calibration.
 * Replaces calibrated_quant.static_scales (src/moss_tts/_runtime/calibrated_quant.py:36-38).
 */
int mt_static_scales(const void* w, int dtype, void* out, int n, int k, void* stream);

/*
 * One block of the GPTQ column loop: columns [start, start + cols) (cols <= 128) of the
 * permuted weights for n rows. w fp32 [n, cols] (the block, updated in place), errors fp32
 * [n, cols] (out: (w - bf16(code * s)) / hinv[c][c] per column), codes int8 [n, k] (written at
 * the original column perm[start + c]), scales bf16 [n, k / group], hinv fp32 [k, k] (upper
 * Cholesky factor of the damped, permuted inverse Hessian), perm int64 [k]. Per column:
 * code = clamp(rint(w / s), -7, 7), then w[:, j] -= err * hinv[c][j] for j >= c, each
 * operation rounded on its own. The caller applies errors @ hinv[block, after] to the
 * columns after the block.
 * Replaces the per-column Triton _column launches of calibrated_quant.gptq
 * (src/moss_tts/_runtime/calibrated_quant.py:15-33, 65-84).
 */
int mt_gptq_block(void* w, void* errors, void* codes, const void* scales, const void* hinv, const void* perm,
                  int start, int cols, int n, int k, int group, void* stream);

/*
 * W4A16 G32 decode GEMV, batch 1..8: y[b, :] = bf16(x'[b, :] . W^T) with fp32 accumulation,
 * where x' = x, or RMSNorm(x) (mode NORM), or RMSNorm(bf16(x + residual)) (mode NORM|ADD,
 * also storing bf16(x + residual) into `summed` when non-NULL). With mode PAIRED, y has
 * N/2 columns: bf16(bf16(silu(bf16 gate)) * bf16 up).
 * Replaces int4_dp4a (src/moss_tts/_runtime/int4_dp4a.py:56-74), dp4a_packing.linear /
 * project (dp4a_packing.py:94-125; paired SiLU at :85-89) and the fused norm projection
 * dp4a_norm_projection.linear (dp4a_norm_projection.py:99-117), as W4A16 instead of W4A8.
 * Requires k % 128 == 0, n % 4 == 0 (n % 8 when PAIRED), x/residual/summed/norm_w 8-byte
 * and qweight 16-byte aligned. Reads the GPTQ layout directly (register-pipelined kernel);
 * the decode engine's batch-1 path is mt_w4a16_linear_packed over the packed layout.
 */
int mt_w4a16_linear(const void* x, const void* residual, const void* norm_w, float eps,
                    void* summed, const void* qweight, const void* scales, const void* qzeros,
                    void* y, int batch, int n, int k, int group, int mode, int flags,
                    void* stream);

/*
 * Packed W4 layout for the batch-1 tensor-core GEMV (mt_w4a16_linear_packed): sizes of the
 * packed weights and of the per-call workspace for an [n, k] projection with `mode`
 * (PAIRED changes the row order). Requires k % 256 == 0, 256 <= k <= 16384, n even when
 * PAIRED. Pure host arithmetic.
 */
int mt_w4a16_packed_size(int n, int k, int has_zeros, int mode, long long* packed_bytes,
                         long long* workspace_bytes);

/*
 * Load-time repack of GPTQ W4 weights (qweight/scales/qzeros as above; qzeros NULL for
 * symmetric weights) into the packed layout: tiles of 16 weight rows (8 gate + 8 up rows
 * when PAIRED) x 256 input columns, each 2368 bytes (2304 without zero points) laid out in
 * the order the tensor-core lanes read them. Counterpart of the reference's load-time
 * repack install_packing / pack_interleaved (src/moss_tts/_runtime/dp4a_packing.py:15-20,
 * 128-160). `packed` must hold mt_w4a16_packed_size bytes, 16-byte aligned.
 */
int mt_w4a16_pack(const void* qweight, const void* scales, const void* qzeros, int n, int k,
                  int mode, void* packed, void* stream);

/*
 * Batch-1 W4A16 GEMV over packed weights, same math and modes as mt_w4a16_linear (replaces
 * the same reference projections): bulk-copy streaming of the packed tiles, codes as exact
 * fp16 operands of mma.sync m16n8k16, split-K over the SMs. `workspace` holds
 * mt_w4a16_packed_size's workspace bytes, zero-filled by the caller once before first
 * use; every call leaves it zeroed again. Calls that share a workspace must be ordered on
 * one stream. All pointers 16-byte aligned.
 */
int mt_w4a16_linear_packed(const void* x, const void* residual, const void* norm_w, float eps,
                           void* summed, const void* packed, int has_zeros, void* y, int n, int k,
                           int mode, void* workspace, int flags, void* stream);

/*
 * The same projection for `rows` (1..64) activation rows: x, residual and summed [rows, k],
 * y [rows, n (n / 2 when PAIRED)], row-major; the RMSNorm is per row. Two rows share one
 * pass over the weights (the activation rows ride in separate columns of the same mma), so
 * a pair costs about one batch-1 call; an odd last row runs the batch-1 kernel. Used for
 * the batched decode step of 2-4 sequences; replaces the same reference projections.
 */
int mt_w4a16_linear_packed_rows(const void* x, const void* residual, const void* norm_w, float eps,
                                void* summed, const void* packed, int has_zeros, void* y, int rows,
                                int n, int k, int mode, void* workspace, int flags, void* stream);

/*
 * Tensor-parallel exchange over peer memory (NVLink), replacing the NCCL all-reduce after a
 * row-parallel projection for mt_w4a16_linear_packed_tp. Every rank owns a receive area of
 * [slots][world][slot_elems / 2] 64-bit cells (flag << 32 | bf16 pair), mapped on every rank
 * (the caller's symmetric allocation); `recv` lists the areas by rank. Each cell is written
 * and read as one 64-bit element, which is single-copy atomic, so a reader that sees this
 * step's flag sees this step's data: no fences, counters or atomics.
 *   out_slot >= 0: the producer writes its output rows into recv[r][out_slot][rank] of every
 *                  rank r (flag = low 32 bits of *epoch) -- plain stores, no TMA multicast;
 *   in_slot >= 0:  the consumer polls its recv[rank][in_slot][r] cells until every flag equals
 *                  *epoch, and uses x = bf16(sum over ranks r in order) in place of `x`.
 * The poll of one call is bounded by a 1 s deadline for the whole kernel: a cell still stale
 * then (a dead or late peer) sets error word 2 (mt_read_error_word), the kernel finishes with
 * what it read, and later calls give up at once while the word is 2.
 * `epoch` is the caller's device step counter, incremented once per step on every rank before
 * the step's first exchange. No reference counterpart: the reference is single-GPU; this is
 * the all-reduce after o_proj and down of a Megatron-style tensor-parallel decoder.
 */
#define MT_TP_MAX_RANKS 8
typedef struct mt_tp_exchange {
  void* recv[MT_TP_MAX_RANKS];
  const long long* epoch;
  int world, rank;
  int in_slot, out_slot, slot_elems;
} mt_tp_exchange;

/* mt_w4a16_linear_packed with the peer-memory exchange `tp` (see mt_tp_exchange). */
int mt_w4a16_linear_packed_tp(const void* x, const void* residual, const void* norm_w, float eps,
                              void* summed, const void* packed, int has_zeros, void* y, int n, int k,
                              int mode, void* workspace, const mt_tp_exchange* tp, int flags,
                              void* stream);

/*
 * The decode step's whole layer stack in one persistent launch (batch 1, single GPU). Runs,
 * for every layer, RMSNorm + q|k|v, QK-norm + RoPE + K/V cache write + attention over rows
 * 0..position, o_proj, add + RMSNorm + gate/up + SiLU·up and down -- the body of the
 * reference's FastLLM.hidden (src/moss_tts/_runtime/llm.py:227-260; with the gptq preset
 * qkv_cluster_model.Hidden, qkv_cluster_model.py:50-72) -- as one kernel with one CTA per SM
 * whose producer warps stream every layer's packed weights without a break.
 * `layers` is a DEVICE array of n_layers mt_decode_layer entries (16-byte aligned): packed
 * projections from mt_w4a16_pack (q|k|v [6144, 4096] and o [4096, 4096] and down
 * [4096, inter] with mode 0, gate/up [2 inter, 4096] with MT_LINEAR_PAIRED), bf16 norm
 * weights, and the layer's caches k/v bf16 [8, max_len, 128]. The shapes are those of the
 * MOSS-TTS 8B backbone: hidden 4096, 32 query and 8 KV heads of 128; inter % 256 == 0.
 * x = the layer-0 input (embedding sum) bf16 [4096]; positions int64 [1]; cos/sin bf16
 * [max_len, 128]. Outputs: residual bf16 [4096] (the residual stream before the last MLP
 * add) and mlp_out bf16 [4096] (the last down projection) -- the x / residual inputs of
 * mt_heads_greedy. `workspace` (mt_decode_layers_workspace bytes, 256-byte aligned) is
 * zero-filled by the caller once; every successful call leaves its counters zero again. A
 * call whose bounded waits expire (status below) leaves it dirty: zero it before reuse.
 * mt_read_error_word reports 1 (a copy wait expired) or 3 (a grid barrier expired). Calls
 * sharing a workspace must be ordered on one stream. A position outside [0, max_len) sets
 * *status = 1 (status may be NULL).
 */
typedef struct mt_decode_layer {
  const void* qkv;
  const void* out;
  const void* gate_up;
  const void* down;
  const void* input_norm;
  const void* post_norm;
  const void* q_norm;
  const void* k_norm;
  void* k_cache;
  void* v_cache;
} mt_decode_layer;

int mt_decode_layers_workspace(int n_layers, int inter, long long* bytes);
int mt_decode_layers(const void* layers, int n_layers, int inter, int has_zeros, const void* x,
                     const void* positions, const void* cos_tab, const void* sin_tab, int max_len,
                     float eps, void* residual, void* mlp_out, void* workspace, void* status, int flags,
                     void* stream);

/*
 * Batched W4A16 G32 projection on the tcgen05 tensor cores (batch 1..128, meant for the
 * batched decode sweep at 16 and up, where the CUDA-core GEMVs fall behind the weight
 * stream): y[b, :] = bf16(x[b, :] . W^T) with W = bf16((q - z) * s) dequantised exactly as
 * calibrated_quant.dequantize (src/moss_tts/_runtime/calibrated_quant.py:41-42) and fp32
 * accumulation — the projection of dp4a_packing.linear (dp4a_packing.py:94-125) at batch > 8.
 * mode 0, or MT_LINEAR_PAIRED (y = bf16(silu(bf16 gate)) * bf16 up, n/2 columns). GPTQ
 * layout as mt_w4a16_linear; requires n % 128 == 0, k % 256 == 0, 16-byte aligned x and
 * qweight. `workspace` (mt_w4a16_gemm_workspace bytes, 256-byte aligned) is zero-filled once
 * and left with its tickets zero; calls of any shapes may share one workspace of the largest
 * size when they are ordered on one stream.
 */
int mt_w4a16_gemm_workspace(int batch, int n, int k, int mode, long long* bytes);
int mt_w4a16_gemm(const void* x, const void* qweight, const void* scales, const void* qzeros, void* y,
                  int batch, int n, int k, int mode, void* workspace, int flags, void* stream);

/*
 * Packed layout of the batched projection: mt_w4a16_gemm_pack repacks a GPTQ-layout
 * projection once at load time (as the reference's install_packing,
 * src/moss_tts/_runtime/dp4a_packing.py:128-160) into one contiguous 18,944-byte block per
 * 128-row tile and 256-column chunk (mt_w4a16_gemm_pack_size bytes); mt_w4a16_gemm_packed is
 * mt_w4a16_gemm over it (one bulk copy per chunk instead of row pieces), same results and
 * workspace. Requires n % 128 == 0, k % 256 == 0, 16-byte aligned x / packed.
 */
int mt_w4a16_gemm_pack_size(int n, int k, int mode, long long* bytes);
int mt_w4a16_gemm_pack(const void* qweight, const void* scales, const void* qzeros, int n, int k, int mode,
                       void* packed, void* stream);
int mt_w4a16_gemm_packed(const void* x, const void* packed, void* y, int batch, int n, int k, int mode,
                         void* workspace, int flags, void* stream);

/*
 * bf16-weight decode GEMV with the same modes as mt_w4a16_linear (w bf16 [n, k]).
 * Replaces linear_decode (src/moss_tts/_runtime/kernels.py:93-108) and the paired gate/up
 * SiLU GEMV fp8_silu_decode (src/moss_tts/_runtime/fused_mlp.py:7-30). Batch 1 with
 * k <= 12288 streams the rows through shared memory (one CTA per SM); other batches, and
 * MT_FLAG_REGISTER_PIPELINE, use the register-pipelined kernel.
 */
int mt_bf16_linear(const void* x, const void* residual, const void* norm_w, float eps,
                   void* summed, const void* w, void* y, int batch, int n, int k, int mode,
                   int flags, void* stream);

/*
 * rmsnorm (residual == NULL) or add_rmsnorm, rows of width n:
 * replaces kernels.rmsnorm / kernels.add_rmsnorm (src/moss_tts/_runtime/kernels.py:62, :85).
 */
int mt_rmsnorm(const void* x, const void* residual, const void* weight, void* summed, void* y,
               int rows, int n, float eps, int flags, void* stream);

/* y[rows, n] = bf16(bf16(silu(x[:, :n])) * x[:, n:]); replaces kernels.silu_mul (kernels.py:132). */
int mt_silu_mul(const void* x, void* y, int rows, int n, int flags, void* stream);

/*
 * Text + n_vq audio embedding sum with per-add bf16 rounding; ids int64 [tokens, 1 + n_vq].
 * Replaces kernels.embedding_sum (src/moss_tts/_runtime/kernels.py:21). Out-of-range ids
 * read row 0 and set *status = 2 (status may be NULL).
 */
int mt_embedding_sum(const void* ids, const void* text, const void* audio, void* out, int tokens,
                     int h, int vocab, int audio_vocab, int n_vq, void* status, int flags,
                     void* stream);

/*
 * QK head RMSNorm + rotate-half RoPE + K/V cache-row write for `batch` sequences:
 * qkv bf16 [batch, (nq + 2 nkv) * 128], rope tables bf16 [max_len, 128], positions int64
 * [batch], q_out bf16 [batch, nq, 128], caches bf16 [batch, nkv, max_len, 128].
 * Replaces the _qk_rope_cache launch of qk_rope_decode (src/moss_tts/_runtime/kernels.py:142-170,
 * :222). A position outside [0, max_len) sets *status = 1 and writes nothing.
 */
int mt_qk_rope_kv(const void* qkv, const void* q_norm, const void* k_norm, const void* cos_tab,
                  const void* sin_tab, const void* positions, void* q_out, void* k_cache,
                  void* v_cache, int batch, int nq, int nkv, int max_len, float eps, void* status,
                  int flags, void* stream);

/*
 * Fused decode attention: QK-norm + RoPE + cache write (as mt_qk_rope_kv), split-K GQA
 * attention over rows 0..positions[b] with `splits` splits of ceil(len / splits) tokens,
 * and the log-sum-exp merge, out bf16 [batch, nq * 128].
 * Replaces qk_rope_decode (src/moss_tts/_runtime/kernels.py:211-251), which launches
 * _qk_rope_cache, launch_attention_ordered (attention_native.cu:91-97) and the split
 * reduction (kernels.py:198-208).
 * Scratch (caller-allocated): partial fp32 [batch * nkv * splits * (nq/nkv) * 128],
 * lse fp32 [batch * nkv * splits * (nq/nkv)], tickets uint32 [batch * nkv] (zero before the
 * first call; every call leaves them zero). nq / nkv must be 1, 2 or 4.
 */
int mt_attention_decode(const void* qkv, const void* q_norm, const void* k_norm,
                        const void* cos_tab, const void* sin_tab, const void* positions,
                        void* k_cache, void* v_cache, void* out, void* partial, void* lse,
                        void* tickets, int batch, int nq, int nkv, int max_len, int splits,
                        float eps, void* status, int flags, void* stream);

/*
 * mt_attention_decode of one sequence with the attention output projection folded into the
 * kernel's tail: out = attention (as mt_attention_decode), proj = bf16(W_o . out), W_o
 * [n_out, nq*128] in the packed layout of mt_w4a16_pack (wo_zeros != 0: blocks carry zero
 * points). Replaces the attention + o_proj pair of the reference's decode layer
 * (src/moss_tts/_runtime/llm.py:246-252: attention, then the quantized o_proj of
 * dp4a_packing.project). Each KV head's 8-CTA cluster multiplies its head group's columns of
 * W_o (blocks fetched into shared memory before the dependency wait); the KV heads'
 * partials are summed in KV-head order by the last CTA of each row block (deterministic).
 * workspace: nkv*n_out*4 + 64 bytes, zero-filled once; calls leave it reusable. Requires
 * nq/nkv = 2 or 4, n_out % 128 == 0, 16-byte aligned wo_packed and workspace.
 */
int mt_attention_oproj_decode(const void* qkv, const void* q_norm, const void* k_norm, const void* cos_tab,
                              const void* sin_tab, const void* positions, void* k_cache, void* v_cache,
                              void* out, const void* wo_packed, int wo_zeros, void* proj, int n_out,
                              void* workspace, int nq, int nkv, int max_len, float eps, void* status,
                              int flags, void* stream);

/*
 * mt_attention_decode for callers that cannot allocate device memory: real-time audio
 * callbacks that must not block on an allocator, and plugin or FFI hosts that own no device
 * allocator of their own. No counterpart in the reference.
 * The split-K scratch is a fixed array inside this library (about 1.04 MiB per GPU that
 * loads it, held until exit): batch*nkv*splits*(nq/nkv)*128 <= 262144 and
 * batch*nkv <= 1024, otherwise cudaErrorMemoryAllocation (2) is returned and nothing is
 * launched. The first call on a device resolves the array's device address, so make it
 * before any stream capture. All calls on a device share the array: calls whose work
 * overlaps on the GPU race and must be serialised by the caller. Never allocates.
 */
int mt_attention_decode_noalloc(const void* qkv, const void* q_norm, const void* k_norm,
                                const void* cos_tab, const void* sin_tab, const void* positions,
                                void* k_cache, void* v_cache, void* out, int batch, int nq, int nkv,
                                int max_len, int splits, float eps, void* status, int flags,
                                void* stream);

/*
 * Prompt prefill, the non-projection parts of the reference's batched prompt pass
 * (FastLLM.prefill / _prefill_forward, src/moss_tts/_runtime/llm.py:204-226, 303-318; the
 * fused prefill_qkv.project, prefill_qkv.py:7-69). Prompt row t of n sits at position
 * start + t; the cache is one sequence's bf16 [nkv, max_len, 128] (start + n <= max_len).
 * mt_prefill_qk_rope_kv: qkv bf16 [n, (nq + 2 nkv) * 128] -> head RMSNorm + rotate-half RoPE,
 * q_out bf16 [n, nq, 128], K/V rows written into the cache.
 * mt_prefill_attention: causal GQA attention of q bf16 [n, nq, 128] over cache rows
 * 0..start + t for row t, out bf16 [n, nq * 128] (fp32 softmax, scale 1/sqrt(128)).
 */
int mt_prefill_qk_rope_kv(const void* qkv, const void* q_norm, const void* k_norm, const void* cos_tab,
                          const void* sin_tab, int start, void* q_out, void* k_cache, void* v_cache, int n,
                          int nq, int nkv, int max_len, float eps, int flags, void* stream);
int mt_prefill_attention(const void* q, const void* k_cache, const void* v_cache, void* out, int start, int n,
                         int nq, int nkv, int max_len, int flags, void* stream);

/*
 * Output heads of one decode step with greedy selection: final add_rmsnorm of
 * (x + residual), logits of the n_text text-head rows and n_cb audio codebooks of `vocab`
 * rows each, argmax with the first-index tie rule, delay-pattern masks, next token ids
 * int64 [1 + n_vq] (entries of this shard's codebooks, plus the text token when
 * text_owner != 0). hidden_size 4096 runs the bulk-copy streaming kernel; flags bit 1 selects
 * the register-pipelined one. Replaces the head half of FastLLM._decode with greedy sampling
 * (src/moss_tts/_runtime/llm.py:268-287). Scratch: best uint64 [1 + n_cb] and ticket
 * uint32 [1], zero before the first call and left zero by every call.
 */
int mt_heads_greedy(const void* x, const void* residual, const void* norm_w, float eps,
                    void* hidden, const void* text_head, const void* audio_heads,
                    void* text_logits, void* audio_logits, const void* text_ids,
                    const void* audio_length, const void* delay_length, void* next_ids,
                    void* best, void* ticket, int hidden_size, int n_text, int n_cb, int vocab,
                    int cb_offset, int n_vq, int delay_slot_id, int audio_end_id, int pad_code,
                    int text_owner, int flags, void* stream);

/*
 * Greedy selection of `batch` decode steps from precomputed head logits (text bf16
 * [batch, n_text], audio bf16 [batch, n_cb * vocab]): argmax per codebook with the
 * first-index tie rule, the text token through text_ids, the delay-pattern masks with each
 * sequence's audio_length / delay_length (int64 [batch]). Writes next_ids int64
 * [batch, 1 + n_vq]: this shard's codebooks, zeros for the others, the text token when
 * text_owner != 0 (else zero). Replaces the sampling half of FastLLM._decode with greedy=True
 * (src/moss_tts/_runtime/llm.py:276-287) for the batched decode step, whose logits come from
 * one plain bf16 GEMM per head as the reference's F.linear (llm.py:271-274).
 */
/*
 * Device-side advance after a decode step of `batch` sequences: control int64
 * [ids batch*n_ids | positions batch | audio_length batch | delay_length batch] takes
 * next_ids [batch, n_ids] as its ids; positions and audio lengths advance by one; a sequence
 * whose next text token is delay_slot_id starts its delay count (0), and a started count
 * advances by one. Replaces first_audio_graph._advance (src/moss_tts/_runtime/
 * first_audio_graph.py:14-27) as one launch.
 */
int mt_decode_advance(void* control, const void* next_ids, int n_ids, int batch, int delay_slot_id, int flags,
                      void* stream);

int mt_heads_select(const void* text_logits, const void* audio_logits, const void* text_ids,
                    const void* audio_length, const void* delay_length, void* next_ids, int batch,
                    int n_text, int n_cb, int vocab, int cb_offset, int n_vq, int delay_slot_id,
                    int audio_end_id, int pad_code, int text_owner, int flags, void* stream);

/*
 * Sampled next ids for `batch` sequences from their head logits: the non-greedy half of
 * FastLLM._decode (src/moss_tts/_runtime/llm.py:280-287) with the reference sampler
 * sample_topk (llm.py:10-19) per channel -- x = float(logit) / temperature, the top_k largest
 * (ties in ascending index order), softmax over them, entries whose cumulative probability
 * before them exceeds top_p dropped, one draw in proportion to the rest -- then the delay
 * masks. Text: (text_temperature, text_top_k, text_top_p) over n_text logits, the index mapped
 * through text_ids; audio: (audio_*) over each codebook's `vocab` logits (vocab <= 1024). A
 * temperature <= 0 selects the argmax (first index on ties). The uniform of each draw is
 * Philox4x32-10 keyed by seed[b] (uint64) with counter (channel, position[b]): reproducible
 * per (seed, position, channel). position, audio_length, delay_length int64 [batch];
 * next_ids int64 [batch, 1 + n_vq] as mt_heads_select writes it. top_k in 1..64.
 */
int mt_heads_sample(const void* text_logits, const void* audio_logits, const void* text_ids,
                    const void* position, const void* audio_length, const void* delay_length,
                    const void* seed, void* next_ids, int batch, int n_text, int n_cb, int vocab,
                    int cb_offset, int n_vq, int delay_slot_id, int audio_end_id, int pad_code,
                    int text_owner, float text_temperature, int text_top_k, float text_top_p,
                    float audio_temperature, int audio_top_k, float audio_top_p, int flags,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOSS_TTS_B200_H */
