// bf16-weight GEMV kernels for B200 (sm_100a): the bf16-preset projections and the
// fused output heads of the decode step.
//
// Layout: weights bf16 [N, K] row-major. One warp owns R rows; lane l of chunk c
// reads 16 bytes (8 weights) at element 8 * (32c + l), so a warp-wide load pulls
// 512 contiguous bytes of a row. The activation is staged once per CTA in shared
// memory as fp32, split into two float4 planes [2][K/8] so the 32 lanes read
// consecutive 16-byte words. fp32 accumulation with packed FFMA2, shuffle reduce.
//
// The heads kernel computes the MOSS-TTS output logits of one decode step
// (src/moss_tts/_runtime/llm.py:268-287): final residual add + RMSNorm prologue,
// the two audio-phase text-head rows and the 32 x 1024 audio-codebook rows, then
// greedy selection fused as a 64-bit atomicMax over (ordered bf16 logit, ~index)
// keys (torch.argmax's first-index tie rule), and the delay-pattern masks applied
// by the last CTA to finish, which writes the next [1 + 32] token ids.
#include "common.cuh"

namespace mt {

struct Bf16Args {
  const __nv_bfloat16* x;         // [B, K]
  const __nv_bfloat16* residual;  // [B, K] (ADD)
  const __nv_bfloat16* norm_w;    // [K] (NORM)
  __nv_bfloat16* summed;          // [B, K] (ADD, optional)
  const __nv_bfloat16* w;         // [N, K]
  __nv_bfloat16* y;               // [B, N] or [B, N/2] (PAIRED)
  int batch, n, k;
  float eps;
};

// x planes: xs[(b * 2 + h) * E + e] holds elements 8e + 4h .. 8e + 4h + 3, E = K / 8.
template <int B, bool NORM, bool ADD>
__device__ __forceinline__ void stage_bf16(const __nv_bfloat16* x, const __nv_bfloat16* residual,
                                           const __nv_bfloat16* norm_w, __nv_bfloat16* summed,
                                           int batch, int K, float eps, float4* xs, float* red,
                                           bool writer, __nv_bfloat16* normed = nullptr) {
  const int E = K >> 3, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = blockDim.x >> 5;
  for (int b = 0; b < B; ++b) {
    const bool live = b < batch;
    float ss = 0.f;
    for (int e = tid; e < E; e += blockDim.x) {
      float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (live) {
        const uint4 xr = *reinterpret_cast<const uint4*>(x + (size_t)b * K + 8 * e);
        const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) { v[2 * i] = bf16_lo(xw[i]); v[2 * i + 1] = bf16_hi(xw[i]); }
        if (ADD) {
          const uint4 rr = *reinterpret_cast<const uint4*>(residual + (size_t)b * K + 8 * e);
          const uint32_t rw[4] = {rr.x, rr.y, rr.z, rr.w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[2 * i] = round_bf16(v[2 * i] + bf16_lo(rw[i]));
            v[2 * i + 1] = round_bf16(v[2 * i + 1] + bf16_hi(rw[i]));
            __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            o[i] = *reinterpret_cast<uint32_t*>(&p);
          }
          if (summed && writer)
            *reinterpret_cast<uint4*>(summed + (size_t)b * K + 8 * e) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
      xs[(b * 2 + 0) * E + e] = make_float4(v[0], v[1], v[2], v[3]);
      xs[(b * 2 + 1) * E + e] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (NORM) {
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float tot = 0.f;
      for (int w = 0; w < nwarp; ++w) tot += red[w];
      __syncthreads();
      const float inv = 1.0f / sqrtf(tot / (float)K + eps);
      for (int e = tid; e < E; e += blockDim.x) {
        const uint4 wr = *reinterpret_cast<const uint4*>(norm_w + 8 * e);
        const uint32_t ww[4] = {wr.x, wr.y, wr.z, wr.w};
        float4 lo = xs[(b * 2 + 0) * E + e], hi = xs[(b * 2 + 1) * E + e];
        float v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float wv = (i & 1) ? bf16_hi(ww[i >> 1]) : bf16_lo(ww[i >> 1]);
          v[i] = live ? round_bf16(round_bf16(v[i] * inv) * wv) : 0.f;
        }
        xs[(b * 2 + 0) * E + e] = make_float4(v[0], v[1], v[2], v[3]);
        xs[(b * 2 + 1) * E + e] = make_float4(v[4], v[5], v[6], v[7]);
        if (normed && writer && live) {
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            o[i] = *reinterpret_cast<uint32_t*>(&p);
          }
          *reinterpret_cast<uint4*>(normed + (size_t)b * K + 8 * e) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void dot8(uint4 w, float4 xa, float4 xb, float2& acc) {
  acc = __ffma2_rn(make_float2(bf16_lo(w.x), bf16_hi(w.x)), make_float2(xa.x, xa.y), acc);
  acc = __ffma2_rn(make_float2(bf16_lo(w.y), bf16_hi(w.y)), make_float2(xa.z, xa.w), acc);
  acc = __ffma2_rn(make_float2(bf16_lo(w.z), bf16_hi(w.z)), make_float2(xb.x, xb.y), acc);
  acc = __ffma2_rn(make_float2(bf16_lo(w.w), bf16_hi(w.w)), make_float2(xb.z, xb.w), acc);
}

// Dot products of RR weight rows with B staged activations; result per lane.
template <int B, int RR>
__device__ __forceinline__ void rows_dot(const __nv_bfloat16* w, const size_t (&rows)[RR], int K,
                                         const float4* xs, float (&acc)[B][RR]) {
  const int E = K >> 3, lane = threadIdx.x & 31;
#pragma unroll
  for (int b = 0; b < B; ++b)
#pragma unroll
    for (int r = 0; r < RR; ++r) acc[b][r] = 0.f;
  const int chunks = (E + 31) >> 5;
  uint4 wn[RR];
  if (lane < E)
#pragma unroll
    for (int r = 0; r < RR; ++r) wn[r] = ld_stream_v4(w + rows[r] * K + (size_t)lane * 8);
  for (int c = 0; c < chunks; ++c) {
    const int e = (c << 5) + lane;
    uint4 wc[RR];
#pragma unroll
    for (int r = 0; r < RR; ++r) wc[r] = wn[r];
    if (c + 1 < chunks && e + 32 < E)
#pragma unroll
      for (int r = 0; r < RR; ++r) wn[r] = ld_stream_v4(w + rows[r] * K + (size_t)(e + 32) * 8);
    if (e < E) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float4 xa = xs[(b * 2 + 0) * E + e], xb = xs[(b * 2 + 1) * E + e];
#pragma unroll
        for (int r = 0; r < RR; ++r) {
          float2 d = make_float2(0.f, 0.f);
          dot8(wc[r], xa, xb, d);
          acc[b][r] += d.x + d.y;
        }
      }
    }
  }
#pragma unroll
  for (int b = 0; b < B; ++b)
#pragma unroll
    for (int r = 0; r < RR; ++r) acc[b][r] = warp_sum(acc[b][r]);
}

template <int B, int R, bool NORM, bool ADD, bool PAIRED>
__global__ void __launch_bounds__(256, B == 1 ? 2 : 1) bf16_gemv(Bf16Args a) {
  extern __shared__ __align__(16) float4 smem[];
  __shared__ float red[32];
  constexpr int RR = PAIRED ? 2 * R : R;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
  const int n_out = PAIRED ? a.n / 2 : a.n, tasks = n_out / R;
  const int gw = warp * gridDim.x + blockIdx.x, tw = gridDim.x * nwarp;
  if (lane == 0 && gw < tasks) {
#pragma unroll
    for (int h = 0; h < (PAIRED ? 2 : 1); ++h)
      prefetch_l2_bulk(a.w + ((size_t)gw * R + (size_t)h * n_out) * a.k, (uint32_t)(R * a.k * 2));
  }
  pdl_wait();
  pdl_trigger();
  stage_bf16<B, NORM, ADD>(a.x, a.residual, a.norm_w, a.summed, a.batch, a.k, a.eps, smem, red,
                           blockIdx.x == 0);
  for (int t = gw; t < tasks; t += tw) {
    size_t rows[RR];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      rows[i] = (size_t)t * R + i;
      if (PAIRED) rows[R + i] = rows[i] + n_out;
    }
    float acc[B][RR];
    rows_dot<B, RR>(a.w, rows, a.k, smem, acc);
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b >= a.batch) break;
#pragma unroll
        for (int i = 0; i < R; ++i) {
          float v = acc[b][i];
          if (PAIRED) {  // src/moss_tts/_runtime/fused_mlp.py:18-23
            const float gate = round_bf16(v), up = round_bf16(acc[b][R + i]);
            v = round_bf16(gate / (1.0f + expf(-gate))) * up;
          }
          a.y[(size_t)b * n_out + rows[i]] = to_bf16(v);
        }
      }
    }
  }
}

struct HeadsArgs {
  const __nv_bfloat16* x;            // [H] last sublayer output
  const __nv_bfloat16* residual;     // [H] residual stream
  const __nv_bfloat16* norm_w;       // [H] final norm weight
  __nv_bfloat16* hidden;             // [H] normalized hidden (optional output)
  const __nv_bfloat16* text_head;    // [n_text, H]
  const __nv_bfloat16* audio_heads;  // [n_cb * V, H]
  __nv_bfloat16* text_logits;        // [n_text]
  __nv_bfloat16* audio_logits;       // [n_cb * V]
  const int64_t* text_ids;           // [n_text]
  const int64_t* audio_length;       // [1]
  const int64_t* delay_length;       // [1]
  int64_t* next_ids;                 // [1 + n_vq]
  unsigned long long* best;          // [1 + n_cb] scratch, zero on entry and exit
  unsigned* ticket;                  // [1] scratch, zero on entry and exit
  int H, n_text, n_cb, V, cb_offset, n_vq;
  int delay_slot_id, audio_end_id, pad_code;
  int text_owner;                    // this shard selects the text token
  float eps;
};

__device__ __forceinline__ unsigned long long pack_key(float v, int idx) {
  return ((unsigned long long)ordered_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(256, 2) heads_greedy(HeadsArgs a) {
  extern __shared__ __align__(16) float4 smem[];
  __shared__ float red[32];
  __shared__ unsigned last;
  constexpr int R = 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
  const int audio_tasks = a.n_cb * a.V / R;
  const int tasks = audio_tasks + (a.text_owner ? 1 : 0);
  const int gw = warp * gridDim.x + blockIdx.x, tw = gridDim.x * nwarp;
  if (lane == 0 && gw < audio_tasks)
    prefetch_l2_bulk(a.audio_heads + (size_t)gw * R * a.H, (uint32_t)(R * a.H * 2));
  pdl_wait();
  pdl_trigger();
  stage_bf16<1, true, true>(a.x, a.residual, a.norm_w, nullptr, 1, a.H, a.eps, smem, red,
                            blockIdx.x == 0, a.hidden);
  for (int t = gw; t < tasks; t += tw) {
    const bool text = t == audio_tasks;
    const __nv_bfloat16* w = text ? a.text_head : a.audio_heads;
    size_t rows[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int r = text ? min(i, a.n_text - 1) : t * R + i;
      rows[i] = (size_t)r;
    }
    float acc[1][R];
    rows_dot<1, R>(w, rows, a.H, smem, acc);
    if (lane == 0) {
      unsigned long long key = 0ull;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const __nv_bfloat16 lb = to_bf16(acc[0][i]);
        const float lv = __bfloat162float(lb);
        if (text) {
          if (i < a.n_text) {
            a.text_logits[i] = lb;
            const unsigned long long k2 = pack_key(lv, i);
            key = k2 > key ? k2 : key;
          }
        } else {
          a.audio_logits[rows[i]] = lb;
          const unsigned long long k2 = pack_key(lv, (int)(rows[i] % a.V));
          key = k2 > key ? k2 : key;
        }
      }
      const int slot = text ? 0 : 1 + (int)(rows[0] / a.V);
      atomicMax(a.best + slot, key);
    }
  }
  // The last CTA to finish turns the argmax keys into next-step token ids.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(a.ticket, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int64_t delay = *a.delay_length, alen = *a.audio_length;
  // Entries owned by other tensor-parallel shards are zeroed so that one integer
  // all-reduce (sum) over the shards assembles the full id vector.
  if (!a.text_owner && threadIdx.x == 0) a.next_ids[0] = 0;
  for (int ch = threadIdx.x; ch < a.n_vq; ch += blockDim.x)
    if (ch < a.cb_offset || ch >= a.cb_offset + a.n_cb) a.next_ids[1 + ch] = 0;
  if (threadIdx.x == 0 && a.text_owner) {  // llm.py:280-283
    const unsigned long long k = __ldcg(a.best);
    const int idx = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    int64_t tok = a.text_ids[idx < a.n_text ? idx : 0];
    if (delay >= 0) tok = a.delay_slot_id;
    if (delay == 32) tok = a.audio_end_id;
    a.next_ids[0] = tok;
    a.best[0] = 0ull;
  }
  for (int c = threadIdx.x; c < a.n_cb; c += blockDim.x) {  // llm.py:284-286
    const unsigned long long k = __ldcg(a.best + 1 + c);
    const int idx = (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    const int ch = a.cb_offset + c;
    const bool valid = ch < alen && (delay < 0 || ch >= delay);
    a.next_ids[1 + ch] = valid ? (int64_t)idx : (int64_t)a.pad_code;
    a.best[1 + c] = 0ull;
  }
  if (threadIdx.x == 0) *a.ticket = 0u;
}

template <int B, int R, bool NORM, bool ADD, bool PAIRED>
static cudaError_t launch_bf16(const Bf16Args& a, cudaStream_t s, int flags) {
  const int tasks = (PAIRED ? a.n / 2 : a.n) / R;
  const size_t smem = (size_t)B * a.k * 4;
  int blocks = sm_count() * ((B > 1 || smem > 100 * 1024) ? 1 : 2);
  if (blocks > tasks) blocks = tasks;
  return launch(bf16_gemv<B, R, NORM, ADD, PAIRED>, dim3(blocks), dim3(256), smem, s, flags, a);
}

template <int B, bool NORM, bool ADD>
static cudaError_t bf16_paired(const Bf16Args& a, bool paired, cudaStream_t s, int flags) {
  return paired ? launch_bf16<B, 2, NORM, ADD, true>(a, s, flags) : launch_bf16<B, 4, NORM, ADD, false>(a, s, flags);
}

template <int B>
static cudaError_t bf16_mode(const Bf16Args& a, int mode, cudaStream_t s, int flags) {
  const bool paired = mode & 4;
  if (mode & 2) return bf16_paired<B, true, true>(a, paired, s, flags);
  if (mode & 1) return bf16_paired<B, true, false>(a, paired, s, flags);
  return bf16_paired<B, false, false>(a, paired, s, flags);
}

cudaError_t heads_stream_dispatch(const struct HeadsArgs& a, int flags, cudaStream_t s);
struct Bf16StreamArgs {  // bf16_stream.cu; field order and types match it
  const __nv_bfloat16* x;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* summed;
  const __nv_bfloat16* w;
  __nv_bfloat16* y;
  int n, k;
  float eps;
  int unit0, units;
};
bool bf16_stream_linear(const Bf16StreamArgs& args, int mode, int flags, cudaStream_t s, cudaError_t* err);
bool heads_stream_supported(int hidden_size, int n_text, int n_cb, int vocab, int text_owner);

}  // namespace mt

using namespace mt;

// bf16 decode GEMV. Replaces linear_decode (src/moss_tts/_runtime/kernels.py:93-108) and,
// with mode bit 4, the paired gate/up + SiLU GEMV fp8_silu_decode (fused_mlp.py:7-30);
// mode bits 1/2 add the RMSNorm / residual-add prologue (same contract as mt_w4a16_linear).
MT_API int mt_bf16_linear(const void* x, const void* residual, const void* norm_w, float eps,
                          void* summed, const void* w, void* y, int batch, int n, int k, int mode,
                          int flags, void* stream) {
  const bool paired = mode & 4;
  if (!x || !w || !y || batch < 1 || batch > 8 || k < 256 || k % 256 || n < 4 ||
      n % (paired ? 8 : 4) || (mode & ~7))
    return kBadArgument;
  if ((mode & 2) && (!(mode & 1) || !residual)) return kBadArgument;
  if ((mode & 1) && !norm_w) return kBadArgument;
  if (!aligned(x, 16) || !aligned(w, 16) || (residual && !aligned(residual, 16)) ||
      (summed && !aligned(summed, 16)) || (norm_w && !aligned(norm_w, 16)))
    return kBadArgument;
  int chunk = batch;
  auto padded = [](int b) { return b == 1 ? 1 : b == 2 ? 2 : b <= 4 ? 4 : 8; };
  while (chunk > 1 && (size_t)padded(chunk) * k * 4 > 200 * 1024) chunk = (chunk + 1) / 2;
  if ((size_t)k * 4 > 200 * 1024) return kBadArgument;
  const int n_out = paired ? n / 2 : n;
  cudaStream_t s = (cudaStream_t)stream;
  if (batch == 1 && !(flags & 2)) {
    Bf16StreamArgs sa;
    sa.x = (const __nv_bfloat16*)x;
    sa.residual = (const __nv_bfloat16*)residual;
    sa.norm_w = (const __nv_bfloat16*)norm_w;
    sa.summed = (__nv_bfloat16*)summed;
    sa.w = (const __nv_bfloat16*)w;
    sa.y = (__nv_bfloat16*)y;
    sa.n = n;
    sa.k = k;
    sa.eps = eps;
    sa.unit0 = 0;
    sa.units = n_out;
    cudaError_t e = cudaSuccess;
    if (bf16_stream_linear(sa, mode, flags & kFlagPdl, s, &e)) return (int)e;
  }
  for (int b0 = 0; b0 < batch; b0 += chunk) {
    Bf16Args a;
    a.x = (const __nv_bfloat16*)x + (size_t)b0 * k;
    a.residual = residual ? (const __nv_bfloat16*)residual + (size_t)b0 * k : nullptr;
    a.norm_w = (const __nv_bfloat16*)norm_w;
    a.summed = summed ? (__nv_bfloat16*)summed + (size_t)b0 * k : nullptr;
    a.w = (const __nv_bfloat16*)w;
    a.y = (__nv_bfloat16*)y + (size_t)b0 * n_out;
    a.batch = batch - b0 < chunk ? batch - b0 : chunk;
    a.n = n;
    a.k = k;
    a.eps = eps;
    cudaError_t e;
    switch (padded(a.batch)) {
      case 1: e = bf16_mode<1>(a, mode, s, flags); break;
      case 2: e = bf16_mode<2>(a, mode, s, flags); break;
      case 4: e = bf16_mode<4>(a, mode, s, flags); break;
      default: e = bf16_mode<8>(a, mode, s, flags); break;
    }
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

// Output heads of one decode step with greedy selection. Replaces the head half of
// FastLLM._decode (src/moss_tts/_runtime/llm.py:268-287, greedy=True): final
// add_rmsnorm (llm.py:259), text head rows [n_text, H] and audio heads [n_cb * V, H]
// (llm.py:188-191, 271-274), argmax (llm.py:11-12) and the delay masks (llm.py:282-286).
// For tensor-parallel shards, `cb_offset` names the first codebook this shard owns and
// only its entries of next_ids are written (text only when text_owner != 0).
MT_API int mt_heads_greedy(const void* x, const void* residual, const void* norm_w, float eps,
                           void* hidden, const void* text_head, const void* audio_heads,
                           void* text_logits, void* audio_logits, const void* text_ids,
                           const void* audio_length, const void* delay_length, void* next_ids,
                           void* best, void* ticket, int hidden_size, int n_text, int n_cb, int vocab,
                           int cb_offset, int n_vq, int delay_slot_id, int audio_end_id, int pad_code,
                           int text_owner, int flags, void* stream) {
  if (!x || !residual || !norm_w || !audio_heads || !audio_logits || !audio_length ||
      !delay_length || !next_ids || !best || !ticket || hidden_size < 256 || hidden_size % 256 ||
      n_cb < 0 || vocab < 4 || vocab % 4 || cb_offset < 0 || cb_offset + n_cb > n_vq)
    return kBadArgument;
  if (text_owner && (!text_head || !text_logits || !text_ids || n_text < 1 || n_text > 4))
    return kBadArgument;
  if (!aligned(x, 16) || !aligned(residual, 16) || !aligned(norm_w, 16) || !aligned(audio_heads, 16) ||
      (hidden && !aligned(hidden, 16)) || (text_head && !aligned(text_head, 16)))
    return kBadArgument;
  HeadsArgs a;
  a.x = (const __nv_bfloat16*)x;
  a.residual = (const __nv_bfloat16*)residual;
  a.norm_w = (const __nv_bfloat16*)norm_w;
  a.hidden = (__nv_bfloat16*)hidden;
  a.text_head = (const __nv_bfloat16*)text_head;
  a.audio_heads = (const __nv_bfloat16*)audio_heads;
  a.text_logits = (__nv_bfloat16*)text_logits;
  a.audio_logits = (__nv_bfloat16*)audio_logits;
  a.text_ids = (const int64_t*)text_ids;
  a.audio_length = (const int64_t*)audio_length;
  a.delay_length = (const int64_t*)delay_length;
  a.next_ids = (int64_t*)next_ids;
  a.best = (unsigned long long*)best;
  a.ticket = (unsigned*)ticket;
  a.H = hidden_size;
  a.n_text = n_text;
  a.n_cb = n_cb;
  a.V = vocab;
  a.cb_offset = cb_offset;
  a.n_vq = n_vq;
  a.delay_slot_id = delay_slot_id;
  a.audio_end_id = audio_end_id;
  a.pad_code = pad_code;
  a.text_owner = text_owner;
  a.eps = eps;
  if (!(flags & 2) && heads_stream_supported(hidden_size, n_text, n_cb, vocab, text_owner))
    return (int)heads_stream_dispatch(a, flags & kFlagPdl, (cudaStream_t)stream);
  const int tasks = n_cb * vocab / 4 + (text_owner ? 1 : 0);
  int blocks = sm_count() * 2;
  const int need = (tasks + 7) / 8;
  if (blocks > need) blocks = need;
  if (blocks < 1) blocks = 1;
  return launch(heads_greedy, dim3(blocks), dim3(256), (size_t)hidden_size * 4,
                (cudaStream_t)stream, flags & kFlagPdl, a);
}
