// Prompt prefill kernels for the MOSS-TTS backbone on B200 (sm_100a).
//
// The reference runs a prompt as one batched backbone pass (FastLLM.prefill /
// _prefill_forward, src/moss_tts/_runtime/llm.py:204-226, 303-318): per layer the q|k|v
// projection of every prompt row, per-head RMSNorm + RoPE with the new K/V rows written into
// the static cache (prefill_qkv.project, prefill_qkv.py:7-69, or the transformers path of
// _attention, llm.py:115-125), then causal scaled-dot-product attention over cache rows
// 0..position of each row (llm.py:126-133). The projections run on the batched W4A16 GEMM;
// these two kernels are the rest:
//   * prefill_qk_rope_kv: token t of n (position start + t): head RMSNorm + rotate-half RoPE
//     of its q and k heads (kernels.py:158-163 rounding points), q to q_out, K/V rows to the
//     single-sequence cache [nkv, max_len, 128];
//   * prefill_attention: causal GQA attention. One CTA per (KV head, 16-token query tile)
//     serves the tile's rows of every query head of that KV head (64 query rows), streams the
//     cache in 32-key tiles through shared memory and keeps an online softmax per row: each
//     K/V byte of a tile is read once for the four query heads. fp32 logits, softmax and
//     accumulation, 1/sqrt(128) scale (kernels.py:183); keys past a row's position are masked.
#include "common.cuh"

namespace mt {
namespace prefill {

constexpr int kHeadDim = 128;
constexpr float kScale = 0.08838834764831845f;  // 1/sqrt(128)
constexpr int kTokens = 16;                     // query tokens per CTA
constexpr int kKeys = 32;                       // keys per shared-memory tile (static smem < 48 KB)
constexpr int kThreads = 256;

// One warp per (token, head): head RMSNorm + RoPE, as the decode kernels (attention.cu).
__global__ void __launch_bounds__(32) qk_rope_kv(const __nv_bfloat16* __restrict__ qkv,
                                                 const __nv_bfloat16* __restrict__ q_norm,
                                                 const __nv_bfloat16* __restrict__ k_norm,
                                                 const __nv_bfloat16* __restrict__ cos_tab,
                                                 const __nv_bfloat16* __restrict__ sin_tab, int start,
                                                 __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                                 __nv_bfloat16* __restrict__ v_cache, int nq, int nkv, int max_len,
                                                 float eps) {
  const int h = blockIdx.x, t = blockIdx.y, lane = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const int p = start + t;
  const __nv_bfloat16* src = qkv + (size_t)t * (nq + 2 * nkv) * kHeadDim;
  const bool is_q = h < nq;
  const uint2 r = *reinterpret_cast<const uint2*>(src + (size_t)h * kHeadDim + 4 * lane);
  float x[4] = {bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y)};
  const __nv_bfloat16* w = is_q ? q_norm : k_norm;
  const __nv_bfloat16* c = cos_tab + (size_t)p * kHeadDim;
  const __nv_bfloat16* s = sin_tab + (size_t)p * kHeadDim;
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / 128.f + eps);
  float y[4], part[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) y[i] = round_bf16(round_bf16(x[i] * inv) * bf16f(w[4 * lane + i]));
#pragma unroll
  for (int i = 0; i < 4; ++i) part[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);  // rotate_half partner d +- 64
  const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = 4 * lane + i;
    x[i] = round_bf16(round_bf16(y[i] * bf16f(c[d])) + round_bf16(sign * part[i] * bf16f(s[d])));
  }
  __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
  uint2 o;
  o.x = *reinterpret_cast<uint32_t*>(&lo);
  o.y = *reinterpret_cast<uint32_t*>(&hi);
  if (is_q) {
    *reinterpret_cast<uint2*>(q_out + ((size_t)t * nq + h) * kHeadDim + 4 * lane) = o;
  } else {
    const int kh = h - nq;
    const size_t row = ((size_t)kh * max_len + p) * kHeadDim + 4 * lane;
    *reinterpret_cast<uint2*>(k_cache + row) = o;
    *reinterpret_cast<uint2*>(v_cache + row) =
        *reinterpret_cast<const uint2*>(src + (size_t)(nq + nkv + kh) * kHeadDim + 4 * lane);
  }
}

// CTA (KV head kh, tile of kTokens query tokens): rows rr = head * kTokens + token for the REP
// query heads of kh. Thread (row, quarter): tid = row * 4 + quarter for up to 64 rows.
template <int REP>
__global__ void __launch_bounds__(kThreads) attention(const __nv_bfloat16* __restrict__ q,
                                                      const __nv_bfloat16* __restrict__ k_cache,
                                                      const __nv_bfloat16* __restrict__ v_cache,
                                                      __nv_bfloat16* __restrict__ out, int start, int n, int nq,
                                                      int max_len) {
  constexpr int kRows = REP * kTokens;        // query rows of this CTA (<= 64)
  __shared__ __align__(16) __nv_bfloat16 ks[kKeys][kHeadDim + 8];   // +8: rows on different banks
  __shared__ __align__(16) __nv_bfloat16 vs[kKeys][kHeadDim + 8];
  __shared__ float ps[kRows][kKeys + 1];
  const int kh = blockIdx.x, t0 = blockIdx.y * kTokens, tid = threadIdx.x;
  const int row = tid >> 2, qt = tid & 3;      // query row, 32-dim quarter
  const bool active = row < kRows;
  const int head = kh * REP + row / kTokens, tok = t0 + row % kTokens;
  const bool valid = active && tok < n;
  const int qpos = start + tok;                // this row's position: attends keys 0..qpos
  pdl_wait();
  pdl_trigger();
  // this thread's quarter of its query row, fp32, pre-scaled
  float qv[32];
  if (valid) {
    const uint4* src = reinterpret_cast<const uint4*>(q + ((size_t)tok * nq + head) * kHeadDim + qt * 32);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 w = src[j];
      const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        qv[8 * j + 2 * i] = bf16_lo(a[i]) * kScale;
        qv[8 * j + 2 * i + 1] = bf16_hi(a[i]) * kScale;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) qv[i] = 0.f;
  }
  float m_run = -INFINITY, l_run = 0.f, acc[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i] = 0.f;
  const int last_tok = min(t0 + kTokens, n) - 1;
  const int kend = start + last_tok + 1;       // keys any row of this CTA needs
  const size_t base = (size_t)kh * max_len * kHeadDim;
  for (int k0 = 0; k0 < kend; k0 += kKeys) {
    const int nk = min(kKeys, kend - k0);
    __syncthreads();  // every thread is done with the previous tile
    for (int i = tid; i < nk * (kHeadDim / 8); i += kThreads) {
      const int kr = i / (kHeadDim / 8), c = i - kr * (kHeadDim / 8);
      *reinterpret_cast<uint4*>(&ks[kr][c * 8]) =
          *reinterpret_cast<const uint4*>(k_cache + base + (size_t)(k0 + kr) * kHeadDim + c * 8);
      *reinterpret_cast<uint4*>(&vs[kr][c * 8]) =
          *reinterpret_cast<const uint4*>(v_cache + base + (size_t)(k0 + kr) * kHeadDim + c * 8);
    }
    __syncthreads();
    // logits of this row against the tile's keys: quarter partial dots, summed over the 4 lanes
    float mt = -INFINITY;
    for (int j = 0; j < nk; ++j) {
      float d = 0.f;
      if (active) {
        const uint4* kk = reinterpret_cast<const uint4*>(&ks[j][qt * 32]);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 w = kk[u];
          const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            d = fmaf(qv[8 * u + 2 * i], bf16_lo(a[i]), d);
            d = fmaf(qv[8 * u + 2 * i + 1], bf16_hi(a[i]), d);
          }
        }
      }
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      const bool seen = valid && k0 + j <= qpos;  // causal mask
      const float lg = seen ? d : -INFINITY;
      if (qt == 0 && active) ps[row][j] = lg;
      mt = fmaxf(mt, lg);
    }
    __syncwarp();
    // online softmax: rescale the running output, exponentiate this tile's logits
    const float mnew = fmaxf(m_run, mt);
    const float sc = mnew == -INFINITY ? 1.f : expf(m_run - mnew);
    float lsum = 0.f;
    for (int j = qt; j < nk; j += 4) {
      const float lg = active ? ps[row][j] : -INFINITY;
      const float e = lg == -INFINITY ? 0.f : expf(lg - mnew);
      if (active) ps[row][j] = e;
      lsum += e;
    }
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
    __syncwarp();
    l_run = l_run * sc + lsum;
    m_run = mnew;
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] *= sc;
    if (active) {
      for (int j = 0; j < nk; ++j) {
        const float pj = ps[row][j];
        const uint4* vv = reinterpret_cast<const uint4*>(&vs[j][qt * 32]);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 w = vv[u];
          const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[8 * u + 2 * i] = fmaf(pj, bf16_lo(a[i]), acc[8 * u + 2 * i]);
            acc[8 * u + 2 * i + 1] = fmaf(pj, bf16_hi(a[i]), acc[8 * u + 2 * i + 1]);
          }
        }
      }
    }
  }
  if (!valid) return;
  const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
  __nv_bfloat16* dst = out + (size_t)tok * nq * kHeadDim + (size_t)head * kHeadDim + qt * 32;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 pr = __floats2bfloat162_rn(acc[8 * j + 2 * i] * inv, acc[8 * j + 2 * i + 1] * inv);
      o[i] = *reinterpret_cast<uint32_t*>(&pr);
    }
    reinterpret_cast<uint4*>(dst)[j] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace prefill
}  // namespace mt

using namespace mt;

// Prompt rows t = 0..n-1 at positions start + t: QK head RMSNorm + RoPE into q_out bf16
// [n, nq, 128], new K/V rows into the single-sequence cache [nkv, max_len, 128].
MT_API int mt_prefill_qk_rope_kv(const void* qkv, const void* q_norm, const void* k_norm, const void* cos_tab,
                                 const void* sin_tab, int start, void* q_out, void* k_cache, void* v_cache, int n,
                                 int nq, int nkv, int max_len, float eps, int flags, void* stream) {
  if (!qkv || !q_norm || !k_norm || !cos_tab || !sin_tab || !q_out || !k_cache || !v_cache || n < 1 || nkv < 1 ||
      nq < nkv || nq % nkv || start < 0 || start + n > max_len || n > 65535)
    return kBadArgument;
  if (!aligned(qkv, 8) || !aligned(q_out, 8) || !aligned(k_cache, 8) || !aligned(v_cache, 8)) return kBadArgument;
  return (int)launch(prefill::qk_rope_kv, dim3(nq + nkv, n), dim3(32), 0, (cudaStream_t)stream, flags,
                     (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)q_norm, (const __nv_bfloat16*)k_norm,
                     (const __nv_bfloat16*)cos_tab, (const __nv_bfloat16*)sin_tab, start, (__nv_bfloat16*)q_out,
                     (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, nq, nkv, max_len, eps);
}

// Causal GQA attention of prompt rows t = 0..n-1 (position start + t) over cache rows
// 0..start + t: q bf16 [n, nq, 128], caches bf16 [nkv, max_len, 128], out bf16 [n, nq * 128].
MT_API int mt_prefill_attention(const void* q, const void* k_cache, const void* v_cache, void* out, int start, int n,
                                int nq, int nkv, int max_len, int flags, void* stream) {
  if (!q || !k_cache || !v_cache || !out || n < 1 || nkv < 1 || nq < nkv || nq % nkv || start < 0 ||
      start + n > max_len)
    return kBadArgument;
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 16)) return kBadArgument;
  const int rep = nq / nkv;
  const dim3 grid(nkv, (n + prefill::kTokens - 1) / prefill::kTokens);
  cudaStream_t s = (cudaStream_t)stream;
  const __nv_bfloat16 *qq = (const __nv_bfloat16*)q, *kc = (const __nv_bfloat16*)k_cache,
                      *vc = (const __nv_bfloat16*)v_cache;
  __nv_bfloat16* o = (__nv_bfloat16*)out;
  switch (rep) {
    case 4: return (int)launch(prefill::attention<4>, grid, dim3(prefill::kThreads), 0, s, flags, qq, kc, vc, o, start, n,
                               nq, max_len);
    case 2: return (int)launch(prefill::attention<2>, grid, dim3(prefill::kThreads), 0, s, flags, qq, kc, vc, o, start, n,
                               nq, max_len);
    case 1: return (int)launch(prefill::attention<1>, grid, dim3(prefill::kThreads), 0, s, flags, qq, kc, vc, o, start, n,
                               nq, max_len);
    default: return kBadArgument;
  }
}
