// Output heads of one decode step, streamed through shared memory (sm_100a).
//
// Same contract as heads_greedy (bf16_gemv.cu), restructured for bandwidth: the 32 x 1024
// audio rows and the two audio-phase text rows (268 MB of bf16 per step) are split into
// balanced contiguous row ranges, one CTA per SM; a producer warp streams RS-row stages
// with cp.async.bulk into an NS-deep ring (full/empty mbarriers, bounded waits), issuing
// the first stages before griddepcontrol.wait. Consumer thread t owns hidden elements
// 8t .. 8t+7 (the final add + RMSNorm is computed once per CTA into registers), so
// shared memory carries only weight bytes. Per-warp row partials are kept in shared
// memory and reduced once at the end; each CTA folds its rows into per-codebook argmax
// keys (order-preserving bf16 logit bits, ~index: torch.argmax's first-index tie rule)
// with shared atomics and publishes them with one global atomicMax per codebook it
// touched; the last CTA applies the delay-pattern masks (src/moss_tts/_runtime/llm.py:280-286).
#include "stream_pipeline.cuh"

namespace mt {

__device__ int g_heads_error;  // set when a bounded wait expired (read through mt_read_error_word)

using namespace pipe;

struct HeadsStreamArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* hidden;
  const __nv_bfloat16* text_head;
  const __nv_bfloat16* audio_heads;
  __nv_bfloat16* text_logits;
  __nv_bfloat16* audio_logits;
  const int64_t* text_ids;
  const int64_t* audio_length;
  const int64_t* delay_length;
  int64_t* next_ids;
  unsigned long long* best;
  unsigned* ticket;
  int H, n_text, n_cb, V, cb_offset, n_vq;
  int delay_slot_id, audio_end_id, pad_code, text_owner;
  float eps;
};

constexpr int kMaxLocalKeys = 8;

__device__ __forceinline__ unsigned long long head_key(float v, int idx) {
  return ((unsigned long long)ordered_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

template <int RS, int NS>
__global__ void __launch_bounds__(544, 1) heads_stream(HeadsStreamArgs a, int max_rows) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[NS];
  __shared__ __align__(8) uint64_t empty[NS];
  __shared__ float ssum[32];
  __shared__ unsigned long long keys[kMaxLocalKeys];
  __shared__ int failed;
  __shared__ unsigned last;

  const int H = a.H, consumers = H >> 3, cwarps = consumers >> 5;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool producer = tid >= consumers;
  const size_t row_bytes = (size_t)H * 2, stage_bytes = (size_t)RS * row_bytes;
  const int n_audio = a.n_cb * a.V, n_text = a.text_owner ? a.n_text : 0;
  const int units = (n_audio + n_text) >> 1;
  const int u0 = (int)((long)blockIdx.x * units / gridDim.x), u1 = (int)((long)(blockIdx.x + 1) * units / gridDim.x);
  const int r0 = 2 * u0, nrows = 2 * (u1 - u0);
  const int stages = (nrows + RS - 1) / RS;
  const int cb_first = r0 < n_audio ? r0 / a.V : 0;
  float* partial = reinterpret_cast<float*>(smem + (size_t)NS * stage_bytes);  // [cwarps][max_rows]

  auto issue = [&](int st) {
    const int slot = st % NS;
    const int rows = min(RS, nrows - st * RS);
    const int g0 = r0 + st * RS, g1 = g0 + rows;
    uint8_t* dst = smem + (size_t)slot * stage_bytes;
    mbar_expect_tx(&full[slot], (unsigned)(rows * row_bytes));
    const int a1 = min(g1, n_audio);
    if (g0 < a1)
      bulk_copy(dst, reinterpret_cast<const uint8_t*>(a.audio_heads) + (size_t)g0 * row_bytes,
                (unsigned)((a1 - g0) * row_bytes), &full[slot]);
    const int t0 = max(g0, n_audio);
    if (t0 < g1)
      bulk_copy(dst + (size_t)(t0 - g0) * row_bytes,
                reinterpret_cast<const uint8_t*>(a.text_head) + (size_t)(t0 - n_audio) * row_bytes,
                (unsigned)((g1 - t0) * row_bytes), &full[slot]);
  };

  if (tid == consumers) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], cwarps);
    }
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int st = 0; st < NS && st < stages; ++st) issue(st);
  }
  if (tid < kMaxLocalKeys) keys[tid] = 0ull;
  __syncthreads();

  if (producer) {
    pdl_trigger();
    if (lane == 0) {
      int st = NS;
      for (; st < stages; ++st) {
        const int slot = st % NS;
        if (!mbar_wait_bounded(&empty[slot], (unsigned)(((st / NS) - 1) & 1))) break;
        issue(st);
      }
      if (st < stages) {
        atomicExch(&g_heads_error, 1);
        for (int d = st - NS; d < st; ++d)
          if (d >= 0) mbar_wait_bounded(&full[d % NS], (unsigned)((d / NS) & 1));
      }
    }
    return;
  }

  pdl_wait();
  pdl_trigger();

  // Final residual add + RMSNorm (llm.py:259; kernels.py:69-90) for elements 8t .. 8t+7.
  float xv[8];
  {
    const uint4 xr = reinterpret_cast<const uint4*>(a.x)[tid];
    const uint4 rr = reinterpret_cast<const uint4*>(a.residual)[tid];
    const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w}, rw[4] = {rr.x, rr.y, rr.z, rr.w};
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xv[2 * i] = round_bf16(bf16_lo(xw[i]) + bf16_lo(rw[i]));
      xv[2 * i + 1] = round_bf16(bf16_hi(xw[i]) + bf16_hi(rw[i]));
      ss += xv[2 * i] * xv[2 * i] + xv[2 * i + 1] * xv[2 * i + 1];
    }
    ss = warp_sum(ss);
    if (lane == 0) ssum[warp] = ss;
    named_sync(1, consumers);
    float tot = 0.f;
    for (int w = 0; w < cwarps; ++w) tot += ssum[w];
    const float inv = 1.0f / sqrtf(tot / (float)H + a.eps);
    const uint4 wr = reinterpret_cast<const uint4*>(a.norm_w)[tid];
    const uint32_t ww[4] = {wr.x, wr.y, wr.z, wr.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xv[2 * i] = round_bf16(round_bf16(xv[2 * i] * inv) * bf16_lo(ww[i]));
      xv[2 * i + 1] = round_bf16(round_bf16(xv[2 * i + 1] * inv) * bf16_hi(ww[i]));
      __nv_bfloat162 pr = __floats2bfloat162_rn(xv[2 * i], xv[2 * i + 1]);
      o[i] = *reinterpret_cast<uint32_t*>(&pr);
    }
    if (a.hidden && blockIdx.x == 0) reinterpret_cast<uint4*>(a.hidden)[tid] = make_uint4(o[0], o[1], o[2], o[3]);
  }

  bool ok = true;
  for (int st = 0; st < stages; ++st) {
    const int slot = st % NS;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[slot], (unsigned)((st / NS) & 1)))) { ok = false; break; }
    const int rows = min(RS, nrows - st * RS);
    const uint8_t* base = smem + (size_t)slot * stage_bytes + (size_t)tid * 16;
    float acc[RS];
#pragma unroll
    for (int i = 0; i < RS; ++i) {
      float2 d = make_float2(0.f, 0.f);
      if (i < rows) {
        const uint4 w = *reinterpret_cast<const uint4*>(base + (size_t)i * row_bytes);
        d = __ffma2_rn(make_float2(bf16_lo(w.x), bf16_hi(w.x)), make_float2(xv[0], xv[1]), d);
        d = __ffma2_rn(make_float2(bf16_lo(w.y), bf16_hi(w.y)), make_float2(xv[2], xv[3]), d);
        d = __ffma2_rn(make_float2(bf16_lo(w.z), bf16_hi(w.z)), make_float2(xv[4], xv[5]), d);
        d = __ffma2_rn(make_float2(bf16_lo(w.w), bf16_hi(w.w)), make_float2(xv[6], xv[7]), d);
      }
      acc[i] = d.x + d.y;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    const float tot = butterfly<RS>(acc, lane);
    constexpr int dup = 32 / RS;
    if ((lane & (dup - 1)) == 0) {
      const int i = row_of<RS>(lane);
      if (i < rows) partial[(size_t)warp * max_rows + st * RS + i] = tot;
    }
  }
  if (!ok && lane == 0) failed = 1;
  named_sync(1, consumers);
  if (failed) {
    if (tid == 0) atomicExch(&g_heads_error, 1);
    return;
  }
  for (int i = tid; i < nrows; i += consumers) {
    float sum = 0.f;
    for (int w = 0; w < cwarps; ++w) sum += partial[(size_t)w * max_rows + i];
    const __nv_bfloat16 lb = to_bf16(sum);
    const float lv = __bfloat162float(lb);
    const int r = r0 + i;
    if (r < n_audio) {
      a.audio_logits[r] = lb;
      const int cb = r / a.V;
      atomicMax(&keys[1 + cb - cb_first], head_key(lv, r - cb * a.V));
    } else {
      a.text_logits[r - n_audio] = lb;
      atomicMax(&keys[0], head_key(lv, r - n_audio));
    }
  }
  named_sync(1, consumers);
  if (tid < kMaxLocalKeys && keys[tid] != 0ull) {
    const int slot = tid == 0 ? 0 : 1 + cb_first + tid - 1;
    atomicMax(a.best + slot, keys[tid]);
  }
  // The last CTA to finish turns the argmax keys into next-step token ids.
  __threadfence();
  named_sync(1, consumers);
  if (tid == 0) last = (atomicAdd(a.ticket, 1u) == gridDim.x - 1) ? 1u : 0u;
  named_sync(1, consumers);
  if (!last) return;
  __threadfence();
  const int64_t delay = *a.delay_length, alen = *a.audio_length;
  if (!a.text_owner && tid == 0) a.next_ids[0] = 0;
  for (int ch = tid; ch < a.n_vq; ch += consumers)
    if (ch < a.cb_offset || ch >= a.cb_offset + a.n_cb) a.next_ids[1 + ch] = 0;
  if (tid == 0 && a.text_owner) {  // llm.py:280-283
    const unsigned long long k = __ldcg(a.best);
    const int idx = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    int64_t tok = a.text_ids[(idx >= 0 && idx < a.n_text) ? idx : 0];
    if (delay >= 0) tok = a.delay_slot_id;
    if (delay == 32) tok = a.audio_end_id;
    a.next_ids[0] = tok;
    a.best[0] = 0ull;
  }
  for (int c = tid; c < a.n_cb; c += consumers) {  // llm.py:284-286
    const unsigned long long k = __ldcg(a.best + 1 + c);
    const int idx = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    const int ch = a.cb_offset + c;
    const bool valid = ch < alen && (delay < 0 || ch >= delay);
    a.next_ids[1 + ch] = valid ? (int64_t)idx : (int64_t)a.pad_code;
    a.best[1 + c] = 0ull;
  }
  if (tid == 0) *a.ticket = 0u;
}

bool heads_stream_supported(int hidden_size, int n_text, int n_cb, int vocab, int text_owner) {
  if (hidden_size != 4096 || vocab % 2) return false;
  if (text_owner && n_text % 2) return false;
  const int rows = n_cb * vocab + (text_owner ? n_text : 0);
  if (rows < 2) return false;
  int blocks = sm_count();
  if (blocks > rows / 2) blocks = rows / 2;
  const int max_rows = 2 * ((rows / 2 + blocks - 1) / blocks);
  // every CTA must span at most kMaxLocalKeys - 1 codebooks
  return (max_rows + vocab - 1) / vocab + 1 <= kMaxLocalKeys - 1;
}

cudaError_t heads_stream_launch(const HeadsStreamArgs& a, int flags, cudaStream_t s) {
  constexpr int RS = 8, NS = 3;
  const int rows = a.n_cb * a.V + (a.text_owner ? a.n_text : 0);
  int blocks = sm_count();
  if (blocks > rows / 2) blocks = rows / 2;
  const int max_rows = 2 * ((rows / 2 + blocks - 1) / blocks);
  const int cwarps = a.H / 8 / 32;
  const size_t smem = (size_t)NS * RS * a.H * 2 + (size_t)cwarps * max_rows * sizeof(float);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  return launch(heads_stream<RS, NS>, dim3(blocks), dim3(a.H / 8 + 32), smem, s, flags, a, max_rows);
}

// The argument block of mt_heads_greedy (bf16_gemv.cu); field order and types match it.
struct HeadsArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* hidden;
  const __nv_bfloat16* text_head;
  const __nv_bfloat16* audio_heads;
  __nv_bfloat16* text_logits;
  __nv_bfloat16* audio_logits;
  const int64_t* text_ids;
  const int64_t* audio_length;
  const int64_t* delay_length;
  int64_t* next_ids;
  unsigned long long* best;
  unsigned* ticket;
  int H, n_text, n_cb, V, cb_offset, n_vq;
  int delay_slot_id, audio_end_id, pad_code;
  int text_owner;
  float eps;
};

cudaError_t heads_stream_dispatch(const HeadsArgs& h, int flags, cudaStream_t s) {
  HeadsStreamArgs a;
  a.x = h.x; a.residual = h.residual; a.norm_w = h.norm_w; a.hidden = h.hidden;
  a.text_head = h.text_head; a.audio_heads = h.audio_heads; a.text_logits = h.text_logits;
  a.audio_logits = h.audio_logits; a.text_ids = h.text_ids; a.audio_length = h.audio_length;
  a.delay_length = h.delay_length; a.next_ids = h.next_ids; a.best = h.best; a.ticket = h.ticket;
  a.H = h.H; a.n_text = h.n_text; a.n_cb = h.n_cb; a.V = h.V; a.cb_offset = h.cb_offset; a.n_vq = h.n_vq;
  a.delay_slot_id = h.delay_slot_id; a.audio_end_id = h.audio_end_id; a.pad_code = h.pad_code;
  a.text_owner = h.text_owner; a.eps = h.eps;
  return heads_stream_launch(a, flags, s);
}

cudaError_t heads_error_word(int* value, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_heads_error, sizeof(int));
  if (e != cudaSuccess) return e;
  *value |= v;
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_heads_error, &zero, sizeof(int));
  }
  return e;
}

}  // namespace mt
