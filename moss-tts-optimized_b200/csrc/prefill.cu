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
//   * prefill_attention (default, tensor cores): causal GQA attention as an online-softmax
//     ("flash") loop on mma.sync m16n8k16 bf16 -> fp32: one CTA of 4 warps per (64-row query
//     tile, query head), 16 rows per warp; Q stays in registers, 64-key K/V tiles stream
//     through double-buffered shared memory (cp.async, zero-filled past the cache), S = Q K^T
//     and O += P V on the tensor cores with P rounded to bf16 (the accumulator fragments of S
//     are the A fragments of P V), fp32 row max / sum, 1/sqrt(128) scale (kernels.py:183);
//     keys past a row's position are masked;
//   * prefill_attention with flags bit 1: the CUDA-core kernel, one CTA per (KV head,
//     16-token query tile) for every query head of that KV head, 32-key tiles, fp32 logits,
//     softmax and accumulation.
#include "common.cuh"

namespace mt {
namespace prefill {

constexpr int kHeadDim = 128;
constexpr float kScale = 0.08838834764831845f;  // 1/sqrt(128)
constexpr int kTokens = 16;                     // query tokens per CTA
constexpr int kKeys = 32;                       // keys per shared-memory tile (static smem < 48 KB)
constexpr int kThreads = 256;

// One warp per (token, head), eight per CTA: head RMSNorm + RoPE, as the decode kernels
// (attention.cu).
constexpr int kRopeWarps = 8;
__global__ void __launch_bounds__(kRopeWarps * 32) qk_rope_kv(const __nv_bfloat16* __restrict__ qkv,
                                                 const __nv_bfloat16* __restrict__ q_norm,
                                                 const __nv_bfloat16* __restrict__ k_norm,
                                                 const __nv_bfloat16* __restrict__ cos_tab,
                                                 const __nv_bfloat16* __restrict__ sin_tab, int start,
                                                 __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_cache,
                                                 __nv_bfloat16* __restrict__ v_cache, int nq, int nkv, int max_len,
                                                 float eps, int n) {
  const int item = blockIdx.x * kRopeWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int h = item % (nq + nkv), t = item / (nq + nkv);
  pdl_wait();
  pdl_trigger();
  if (t >= n) return;
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

// ---- tensor-core kernel ----
constexpr int kMmaRows = 64;          // query rows per CTA (4 warps x 16)
constexpr int kMmaKeys = 64;          // keys per shared-memory tile
constexpr int kLd = kHeadDim + 8;     // smem row stride (bf16): 272 B, ldmatrix rows on distinct banks
constexpr int kMmaThreads = 128;
constexpr size_t kMmaSmem = (size_t)5 * kMmaRows * kLd * 2;  // Q, 2 x K, 2 x V

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// CTA (query tile of 64 rows, query head h). Warp w owns rows q0 + 16 w .. + 15; lane (g =
// lane / 4, t = lane % 4) holds rows g and g + 8 of its warp in every fragment.
__global__ void __launch_bounds__(kMmaThreads) attention_mma(const __nv_bfloat16* __restrict__ q,
                                                            const __nv_bfloat16* __restrict__ k_cache,
                                                            const __nv_bfloat16* __restrict__ v_cache,
                                                            __nv_bfloat16* __restrict__ out, int start, int n,
                                                            int nq, int rep, int max_len) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sk = sq + kMmaRows * kLd;      // [2][64][kLd]
  __nv_bfloat16* sv = sk + 2 * kMmaKeys * kLd;  // [2][64][kLd]
  const int q0 = blockIdx.x * kMmaRows, h = blockIdx.y, kh = h / rep;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int rows_here = min(kMmaRows, n - q0);
  const int kend = start + q0 + rows_here;  // keys 0 .. kend - 1 are needed by some row
  const int nkb = (kend + kMmaKeys - 1) / kMmaKeys;
  const __nv_bfloat16* kbase = k_cache + (size_t)kh * max_len * kHeadDim;
  const __nv_bfloat16* vbase = v_cache + (size_t)kh * max_len * kHeadDim;
  auto load_kv = [&](int kb, int buf) {  // 64 rows x 16 chunks of 16 B, K and V
    for (int i = tid; i < kMmaKeys * (kHeadDim / 8); i += kMmaThreads) {
      const int r = i >> 4, c = (i & 15) * 8, key = kb * kMmaKeys + r;
      const bool ok = key < kend;
      const size_t off = (size_t)(ok ? key : 0) * kHeadDim + c;
      cp_async16(sk + ((size_t)buf * kMmaKeys + r) * kLd + c, kbase + off, ok);
      cp_async16(sv + ((size_t)buf * kMmaKeys + r) * kLd + c, vbase + off, ok);
    }
  };
  pdl_wait();
  pdl_trigger();
  for (int i = tid; i < kMmaRows * (kHeadDim / 8); i += kMmaThreads) {
    const int r = i >> 4, c = (i & 15) * 8;
    const bool ok = r < rows_here;
    cp_async16(sq + (size_t)r * kLd + c, q + ((size_t)(ok ? q0 + r : 0) * nq + h) * kHeadDim + c, ok);
  }
  load_kv(0, 0);
  cp_async_commit();

  // rows of this lane: r0 = warp row g, r1 = g + 8; positions
  const int wr0 = q0 + warp * 16;
  const int pos0 = start + wr0 + g, pos1 = pos0 + 8;
  const int wpos_max = start + wr0 + 15;  // the warp's last row position
  constexpr float kLog2e = 1.4426950408889634f;
  const float sl2 = kScale * kLog2e;      // logits to base-2 exponents
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  uint32_t qa[8][4];

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) load_kv(kb + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        ldsm_x4(qa[kk], sq + (size_t)(warp * 16 + (lane & 15)) * kLd + kk * 16 + (lane >> 4) * 8);
    }
    if (kb * kMmaKeys <= wpos_max) {  // some key of this tile is visible to a row of this warp
      const __nv_bfloat16* kt = sk + (size_t)buf * kMmaKeys * kLd;
      const __nv_bfloat16* vt = sv + (size_t)buf * kMmaKeys * kLd;
      float s[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk += 2) {
          uint32_t b[4];
          ldsm_x4(b, kt + (size_t)(8 * j + (lane & 7)) * kLd + kk * 16 + (lane >> 3) * 8);
          mma_bf16(s[j], qa[kk], b[0], b[1]);
          mma_bf16(s[j], qa[kk + 1], b[2], b[3]);
        }
      }
      // causal mask (only tiles that reach past a row's position), then the online softmax
      const bool diag = kb * kMmaKeys + kMmaKeys - 1 > start + wr0;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kb * kMmaKeys + 8 * j + 2 * t + e;
          if (diag && key > pos0) s[j][e] = -INFINITY;
          if (diag && key > pos1) s[j][2 + e] = -INFINITY;
          mx0 = fmaxf(mx0, s[j][e]);
          mx1 = fmaxf(mx1, s[j][2 + e]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      // a row with every key so far masked keeps m = -inf: its factors are 1 and its p are 0
      const float c0 = mn0 == -INFINITY ? 1.f : exp2f((m0 - mn0) * sl2);
      const float c1 = mn1 == -INFINITY ? 1.f : exp2f((m1 - mn1) * sl2);
      const float b0 = mn0 == -INFINITY ? 0.f : mn0 * sl2, b1 = mn1 == -INFINITY ? 0.f : mn1 * sl2;
      float rs0 = 0.f, rs1 = 0.f;
      uint32_t pa[4][4];  // P as A fragments of the 4 key steps of 16
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float p0 = exp2f(fmaf(s[j][0], sl2, -b0)), p1 = exp2f(fmaf(s[j][1], sl2, -b0));
        const float p2 = exp2f(fmaf(s[j][2], sl2, -b1)), p3 = exp2f(fmaf(s[j][3], sl2, -b1));
        rs0 += p0 + p1;
        rs1 += p2 + p3;
        pa[j >> 1][(j & 1) * 2] = pack_bf16(p0, p1);
        pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16(p2, p3);
      }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      l0 = l0 * c0 + rs0;
      l1 = l1 * c1 + rs1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= c0;
        o[j][1] *= c0;
        o[j][2] *= c1;
        o[j][3] *= c1;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int jd = 0; jd < 16; jd += 2) {
          uint32_t b[4];
          ldsm_x4_t(b, vt + (size_t)(16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1)) * kLd + 8 * jd + 8 * (lane >> 4));
          mma_bf16(o[jd], pa[kk], b[0], b[1]);
          mma_bf16(o[jd + 1], pa[kk], b[2], b[3]);
        }
      }
    }
    __syncthreads();  // the tile's buffer is refilled by the next iteration's loads
  }
  cp_async_wait<0>();
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int r0 = wr0 + g, r1 = r0 + 8;
#pragma unroll
  for (int jd = 0; jd < 16; ++jd) {
    const int d = 8 * jd + 2 * t;
    if (r0 < n)
      *reinterpret_cast<uint32_t*>(out + ((size_t)r0 * nq + h) * kHeadDim + d) = pack_bf16(o[jd][0] * i0, o[jd][1] * i0);
    if (r1 < n)
      *reinterpret_cast<uint32_t*>(out + ((size_t)r1 * nq + h) * kHeadDim + d) = pack_bf16(o[jd][2] * i1, o[jd][3] * i1);
  }
}

// ---- CUDA-core kernel ----
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
  const long long items = (long long)(nq + nkv) * n;
  return (int)launch(prefill::qk_rope_kv, dim3((unsigned)((items + prefill::kRopeWarps - 1) / prefill::kRopeWarps)),
                     dim3(prefill::kRopeWarps * 32), 0, (cudaStream_t)stream, flags, (const __nv_bfloat16*)qkv,
                     (const __nv_bfloat16*)q_norm, (const __nv_bfloat16*)k_norm, (const __nv_bfloat16*)cos_tab,
                     (const __nv_bfloat16*)sin_tab, start, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_cache,
                     (__nv_bfloat16*)v_cache, nq, nkv, max_len, eps, n);
}

// Causal GQA attention of prompt rows t = 0..n-1 (position start + t) over cache rows
// 0..start + t: q bf16 [n, nq, 128], caches bf16 [nkv, max_len, 128], out bf16 [n, nq * 128].
// Tensor-core kernel by default; flags bit 1 selects the CUDA-core kernel.
MT_API int mt_prefill_attention(const void* q, const void* k_cache, const void* v_cache, void* out, int start, int n,
                                int nq, int nkv, int max_len, int flags, void* stream) {
  if (!q || !k_cache || !v_cache || !out || n < 1 || nkv < 1 || nq < nkv || nq % nkv || start < 0 ||
      start + n > max_len)
    return kBadArgument;
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 16)) return kBadArgument;
  const int rep = nq / nkv;
  cudaStream_t s = (cudaStream_t)stream;
  if (!(flags & 2)) {
    static bool attr = false;
    if (!attr) {
      const cudaError_t e = cudaFuncSetAttribute(prefill::attention_mma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)prefill::kMmaSmem);
      if (e != cudaSuccess) return (int)e;
      attr = true;
    }
    return (int)launch(prefill::attention_mma, dim3((n + prefill::kMmaRows - 1) / prefill::kMmaRows, nq),
                       dim3(prefill::kMmaThreads), prefill::kMmaSmem, s, flags & kFlagPdl, (const __nv_bfloat16*)q,
                       (const __nv_bfloat16*)k_cache, (const __nv_bfloat16*)v_cache, (__nv_bfloat16*)out, start, n, nq,
                       rep, max_len);
  }
  const dim3 grid(nkv, (n + prefill::kTokens - 1) / prefill::kTokens);
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
