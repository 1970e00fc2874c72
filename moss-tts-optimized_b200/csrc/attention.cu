// Decode attention for the MOSS-TTS backbone on B200 (sm_100a).
//
// One launch per layer does what the reference spreads over three
// (src/moss_tts/_runtime/kernels.py:142-251 and attention_native.cu:31-97):
//   1. QK head RMSNorm + rotate-half RoPE of the fresh projection (kernels.py:142-170),
//      the new K/V rows written into the static cache at `position`;
//   2. split-K GQA attention over cache rows 0..position: CTA (kv head, split, seq)
//      serves all query heads of its KV head, so every K/V byte is read once per
//      layer (the reference reads each KV head once per query head);
//   3. the log-sum-exp merge of the splits, done by the last CTA of each KV head
//      to finish (a ticket counter in scratch memory, reset by that CTA).
// Split boundaries follow the live length read on the device (span = max(64, ceil(len /
// splits)) tokens), so a graph captured once serves every position. Each CTA fetches its
// contiguous K and V row ranges into shared memory with two bulk copies issued before
// the programmatic-dependency wait.
// Scratch (fp32 partials, LSE, tickets) is caller-provided global memory.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "w4_tiles.cuh"

namespace cg = cooperative_groups;

namespace mt {

constexpr int kHeadDim = 128;
constexpr float kScale = 0.08838834764831845f;  // 1/sqrt(128), kernels.py:183

struct AttnArgs {
  const __nv_bfloat16* qkv;      // [B, (nq + 2 nkv) * 128]  q | k | v
  const __nv_bfloat16* q_norm;   // [128]
  const __nv_bfloat16* k_norm;   // [128]
  const __nv_bfloat16* cos_tab;  // [max_len, 128]
  const __nv_bfloat16* sin_tab;  // [max_len, 128]
  const int64_t* positions;      // [B] cache row written this step; attends 0..position
  __nv_bfloat16* k_cache;        // [B, nkv, max_len, 128]
  __nv_bfloat16* v_cache;        // [B, nkv, max_len, 128]
  __nv_bfloat16* out;            // [B, nq * 128]
  float* partial;                // [B, nkv, splits, rep, 128]
  float* lse;                    // [B, nkv, splits, rep]
  unsigned* tickets;             // [B, nkv], zero on entry, zero on exit
  int nq, nkv, max_len, splits;
  float eps;
  int* status;                   // optional: set to 1 when a position is out of range
  // o_proj folded into the tail (mt_attention_oproj_decode, one sequence): W_o in the packed
  // slice-block layout of mt_w4a16_pack, fp32 partials [nkv][n_out] (one per KV head), merge
  // counters [cluster ranks] (zero on entry and exit) and the bf16 projection [n_out]
  const uint8_t* wo;
  int wo_zeros, n_out;
  float* opart;
  unsigned* otickets;
  __nv_bfloat16* oout;
};

// Head RMSNorm + RoPE for one 128-wide head held as 4 values per lane
// (dims 4*lane .. 4*lane+3). Rounding points follow kernels.py:158-163.
__device__ __forceinline__ void norm_rope_head(float (&x)[4], const __nv_bfloat16* w,
                                               const __nv_bfloat16* c, const __nv_bfloat16* s,
                                               float eps, int lane) {
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / 128.f + eps);
  float y[4], part[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) y[i] = round_bf16(round_bf16(x[i] * inv) * bf16f(w[4 * lane + i]));
  // rotate_half partner of dim d is d +- 64: held by lane ^ 16
#pragma unroll
  for (int i = 0; i < 4; ++i) part[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);
  const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = 4 * lane + i;
    x[i] = round_bf16(round_bf16(y[i] * bf16f(c[d])) + round_bf16(sign * part[i] * bf16f(s[d])));
  }
}

constexpr int kMinSpan = 64;  // fewest tokens a split handles (short contexts use few splits)

// Tokens of the longest split for a cache of max_len rows and `splits` splits.
__host__ __device__ __forceinline__ int attn_cap(int max_len, int splits) {
  const int even = (max_len + splits - 1) / splits;
  return even > kMinSpan ? even : kMinSpan;
}

__device__ __forceinline__ uint32_t attn_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Rotated 16-byte chunk of row t: thread-specific start so that eight threads reading
// different 256-byte rows at the same step touch eight different bank groups.
__device__ __forceinline__ int rot(int j, int t) { return (j + t) & 15; }

template <int REP>
__global__ void __launch_bounds__(128) attention_decode(AttnArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(16) __nv_bfloat16 qs[REP][kHeadDim];
  __shared__ float stat[REP][2];
  __shared__ __align__(8) uint64_t bar;
  __shared__ unsigned last;
  const int kh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qkv_w = (a.nq + 2 * a.nkv) * kHeadDim;
  const int cap = attn_cap(a.max_len, a.splits);
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(sm);                  // [cap][128]
  __nv_bfloat16* vs = ks + (size_t)cap * kHeadDim;                           // [cap][128]
  float* lg = reinterpret_cast<float*>(vs + (size_t)cap * kHeadDim);         // [REP][cap]

  // The position and every cache row before it were written before this kernel's
  // predecessor started (earlier steps), so the K/V rows of this split are fetched
  // before the dependency wait; row `position` itself is recomputed below.
  int64_t pos = a.positions[b];
  const bool bad_pos = pos < 0 || pos >= a.max_len;
  if (bad_pos) pos = pos < 0 ? 0 : a.max_len - 1;
  const int p = (int)pos, len = p + 1;
  int span = (len + a.splits - 1) / a.splits;
  if (span < kMinSpan) span = kMinSpan;
  const int t0 = split * span, t1 = min(t0 + span, len);
  const int n = t1 > t0 ? t1 - t0 : 0;
  const size_t kv_base = ((size_t)b * a.nkv + kh) * a.max_len * kHeadDim;
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(attn_smem_u32(&bar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (n > 0) {
      const unsigned bytes = (unsigned)(n * kHeadDim * 2);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(attn_smem_u32(&bar)),
                   "r"(2 * bytes) : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       attn_smem_u32(ks)), "l"(a.k_cache + kv_base + (size_t)t0 * kHeadDim), "r"(bytes),
                   "r"(attn_smem_u32(&bar)) : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       attn_smem_u32(vs)), "l"(a.v_cache + kv_base + (size_t)t0 * kHeadDim), "r"(bytes),
                   "r"(attn_smem_u32(&bar)) : "memory");
    }
  }
  __syncthreads();  // the barrier is initialised before any thread polls it
  pdl_wait();
  pdl_trigger();
  if (bad_pos && a.status && tid == 0) atomicExch(a.status, 1);
  const __nv_bfloat16* src = a.qkv + (size_t)b * qkv_w;

  // 1. Query heads of this KV head (warp w < REP handles head kh*REP + w), rounded to bf16
  //    as the reference stores them (kernels.py:165).
  if (warp < REP) {
    const int h = kh * REP + warp;
    float x[4];
    const uint2 r = *reinterpret_cast<const uint2*>(src + h * kHeadDim + 4 * lane);
    x[0] = bf16_lo(r.x); x[1] = bf16_hi(r.x); x[2] = bf16_lo(r.y); x[3] = bf16_hi(r.y);
    norm_rope_head(x, a.q_norm, a.cos_tab + (size_t)p * kHeadDim, a.sin_tab + (size_t)p * kHeadDim, a.eps, lane);
    __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&lo);
    o.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(&qs[warp][4 * lane]) = o;
  }
  // 2. The split holding the newest token computes and writes this step's K/V rows.
  const bool owner = t0 <= p && p < t1;
  uint2 krow = make_uint2(0, 0), vrow = make_uint2(0, 0);
  if (owner && warp == 0) {
    float x[4];
    const uint2 r = *reinterpret_cast<const uint2*>(src + (a.nq + kh) * kHeadDim + 4 * lane);
    x[0] = bf16_lo(r.x); x[1] = bf16_hi(r.x); x[2] = bf16_lo(r.y); x[3] = bf16_hi(r.y);
    norm_rope_head(x, a.k_norm, a.cos_tab + (size_t)p * kHeadDim, a.sin_tab + (size_t)p * kHeadDim, a.eps, lane);
    __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
    krow.x = *reinterpret_cast<uint32_t*>(&lo);
    krow.y = *reinterpret_cast<uint32_t*>(&hi);
    vrow = *reinterpret_cast<const uint2*>(src + (a.nq + a.nkv + kh) * kHeadDim + 4 * lane);
    *reinterpret_cast<uint2*>(a.k_cache + kv_base + (size_t)p * kHeadDim + 4 * lane) = krow;
    *reinterpret_cast<uint2*>(a.v_cache + kv_base + (size_t)p * kHeadDim + 4 * lane) = vrow;
  }
  // 3. Wait (bounded) for this split's K/V rows; patch in the fresh row.
  auto wait_copies = [&]() -> bool {
    for (long it = 0; it < (1L << 22); ++it) {
      uint32_t done;
      asm volatile("{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], 0;\n selp.u32 %0, 1, 0, q;\n}"
                   : "=r"(done) : "r"(attn_smem_u32(&bar)) : "memory");
      if (done) return true;
    }
    return false;
  };
  const bool ok = n > 0 ? wait_copies() : true;
  const bool copied = __syncthreads_and(ok ? 1 : 0) != 0;
  if (!copied) {
    // The copies did not complete within the bound: raise the status and give them one more
    // bounded chance to land (they target this CTA's shared memory). The split then counts as
    // empty (zero partial, log-sum-exp -inf) but still takes its ticket below, so the head's
    // counter returns to zero and the merge never starts before every split has reported.
    if (tid == 0) {
      if (a.status) atomicExch(a.status, 3);
      wait_copies();
    }
    __syncthreads();
  }
  if (copied && owner && warp == 0) {
    *reinterpret_cast<uint2*>(ks + (size_t)(p - t0) * kHeadDim + 4 * lane) = krow;
    *reinterpret_cast<uint2*>(vs + (size_t)(p - t0) * kHeadDim + 4 * lane) = vrow;
  }
  __syncthreads();

  const size_t slot = (((size_t)b * a.nkv + kh) * a.splits + split) * REP;
  if (copied && n > 0) {
    // 4. logits: item (token t, head i) per thread; 16-byte chunks in rotated order.
    for (int item = tid; item < n * REP; item += 128) {
      const int t = item / REP, i = item - t * REP;
      const uint4* krow4 = reinterpret_cast<const uint4*>(ks + (size_t)t * kHeadDim);
      const uint4* q4 = reinterpret_cast<const uint4*>(&qs[i][0]);
      float d0 = 0.f, d1 = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = rot(j, t);
        const uint4 kk = krow4[c], qq = q4[c];
        d0 = fmaf(bf16_lo(qq.x), bf16_lo(kk.x), d0);
        d1 = fmaf(bf16_hi(qq.x), bf16_hi(kk.x), d1);
        d0 = fmaf(bf16_lo(qq.y), bf16_lo(kk.y), d0);
        d1 = fmaf(bf16_hi(qq.y), bf16_hi(kk.y), d1);
        d0 = fmaf(bf16_lo(qq.z), bf16_lo(kk.z), d0);
        d1 = fmaf(bf16_hi(qq.z), bf16_hi(kk.z), d1);
        d0 = fmaf(bf16_lo(qq.w), bf16_lo(kk.w), d0);
        d1 = fmaf(bf16_hi(qq.w), bf16_hi(kk.w), d1);
      }
      lg[i * cap + t] = (d0 + d1) * kScale;
    }
    __syncthreads();
    // 5. softmax statistics: warp i handles head i.
    if (warp < REP) {
      float m = -INFINITY;
      for (int t = lane; t < n; t += 32) m = fmaxf(m, lg[warp * cap + t]);
      m = warp_max(m);
      float sum = 0.f;
      for (int t = lane; t < n; t += 32) {
        const float e = expf(lg[warp * cap + t] - m);
        lg[warp * cap + t] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) { stat[warp][0] = m; stat[warp][1] = sum; }
    }
    __syncthreads();
    // 6. weighted V: thread d accumulates dim d for every head.
    float o[REP];
#pragma unroll
    for (int i = 0; i < REP; ++i) o[i] = 0.f;
    const __nv_bfloat16* vcol = vs + tid;
#pragma unroll 8
    for (int t = 0; t < n; ++t) {
      const float v = bf16f(vcol[(size_t)t * kHeadDim]);
#pragma unroll
      for (int i = 0; i < REP; ++i) o[i] = fmaf(lg[i * cap + t], v, o[i]);
    }
#pragma unroll
    for (int i = 0; i < REP; ++i) a.partial[(slot + i) * kHeadDim + tid] = o[i] / stat[i][1];
    if (tid < REP) a.lse[slot + tid] = stat[tid][0] + logf(stat[tid][1]);
  } else {
#pragma unroll
    for (int i = 0; i < REP; ++i) a.partial[(slot + i) * kHeadDim + tid] = 0.f;
    if (tid < REP) a.lse[slot + tid] = -INFINITY;
  }

  // 7. The last CTA of this KV head merges all splits (kernels.py:198-208).
  __threadfence();
  __syncthreads();
  unsigned* ticket = a.tickets + (size_t)b * a.nkv + kh;
  if (tid == 0) last = (atomicAdd(ticket, 1u) == (unsigned)a.splits - 1u) ? 1u : 0u;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const size_t base = ((size_t)b * a.nkv + kh) * a.splits * REP;
  const int active = (len + span - 1) / span;  // splits beyond this one hold no tokens
#pragma unroll
  for (int i = 0; i < REP; ++i) {
    float m = -INFINITY;
#pragma unroll 8
    for (int s = 0; s < active; ++s) m = fmaxf(m, __ldcg(a.lse + base + s * REP + i));
    float wsum = 0.f, acc = 0.f;
#pragma unroll 8
    for (int s = 0; s < active; ++s) {
      const float l = __ldcg(a.lse + base + s * REP + i);
      const float w = l == -INFINITY ? 0.f : expf(l - m);  // a failed split contributes nothing
      wsum += w;
      acc = fmaf(w, __ldcg(a.partial + (base + s * REP + i) * kHeadDim + tid), acc);
    }
    a.out[(size_t)b * a.nq * kHeadDim + (kh * REP + i) * kHeadDim + tid] = to_bf16(wsum > 0.f ? acc / wsum : 0.f);
  }
  if (tid == 0) *ticket = 0u;
}

// ----------------------------------------------------------------------------
// Cluster decode attention: one thread-block cluster of kClusterCtas CTAs per (sequence,
// KV head). CTA r of the cluster owns tokens [r*span, (r+1)*span), span = ceil(len / C),
// streams them in kChunk-token chunks (K and V rows are contiguous in the cache: two bulk
// copies per chunk, double-buffered, the first two issued before the dependency wait) and
// keeps an online softmax per query head. Everything independent of the previous kernel
// (position, RoPE rows, norm weights) is read before the wait. Per chunk:
//   logits  - item (token, head, quarter of the 128 dims) per thread, quarters combined by
//             two lane shuffles (q in shared memory padded per quarter: conflict free);
//   softmax - one warp per query head (max, exp, sum, running rescale);
//   P.V     - thread (pair of dims, token group of four) accumulates all query heads.
// The CTAs then merge through distributed shared memory: each pushes its running max, sum
// and the 16-dim slice of its unnormalised output owned by rank s into rank s's inbox,
// one cluster barrier publishes them, and every rank finishes its 16 dims locally.
constexpr int kClusterCtas = 8;
// Tokens per streamed chunk: 128 for one sequence (latency: one CTA per SM is enough), 32
// for batches (four CTAs share an SM, so one CTA's fixed latency overlaps the others' streams;
// at 64 sequences x 2,200 tokens: 128 -> 21.1 ms, 64 -> 16.8 ms, 32 -> 15.1 ms per step; one
// sequence at 512+ tokens: 128 -> 1.536 ms, 64 -> 1.600 ms, 32 -> 1.690 ms per step).
constexpr int kAttnThreads = 256;               // 8 warps per CTA (16 measured no faster)
constexpr int kTokenGroups = kAttnThreads / 64;  // P.V token groups of 64 dim-pair threads

// Helpers of the tensor-core kernel (attention_ws below): ldmatrix, mma.sync m16n8k16 bf16
// with zero A rows 8..15, bf16 packing, and the 128-byte swizzle of the TMA boxes (16-byte
// piece c of row r stored at piece c ^ (r & 7)), which keeps 8-row ldmatrix reads on eight
// different bank groups.
__device__ __forceinline__ void attn_ldsm_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void attn_ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void attn_mma(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  // A rows 8..15 (fragments a1, a3) are zero: only rows g < 8 can carry a query head
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t attn_pack(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// Byte offset of 16-byte piece `piece` (0..15 over the 128 dims) of staged row r in a chunk of
// kChunk rows: box piece / 8 (dims 0-63 | 64-127), swizzled piece within the box's row.
template <int kChunk>
__device__ __forceinline__ uint32_t attn_swz(int r, int piece) {
  return (uint32_t)((piece >> 3) * kChunk * 128 + r * 128 + (((piece & 7) ^ (r & 7)) << 4));
}

template <int REP, int kChunk>
__global__ void __launch_bounds__(kAttnThreads) attention_cluster(AttnArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];  // 2 slots x {K[kChunk][128], V[kChunk][128]} bf16
  constexpr int kQStride = 36;                     // floats per 32-dim quarter of q (+4 pad)
  __shared__ __align__(16) float qs[REP * 4 * kQStride];
  __shared__ __align__(16) float pr[kChunk][REP];  // logits, then probabilities
  __shared__ __align__(16) float red[kTokenGroups][REP][kHeadDim];
  __shared__ __align__(16) float inbox[kClusterCtas][REP][16];
  __shared__ float minbox[kClusterCtas][REP], linbox[kClusterCtas][REP];
  __shared__ float m_run[REP], l_run[REP], scale[REP];
  __shared__ __align__(8) uint64_t full[2];
  __shared__ int failed;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int kh = blockIdx.x / kClusterCtas, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qkv_w = (a.nq + 2 * a.nkv) * kHeadDim;
  constexpr size_t kRowBytes = kHeadDim * 2, kSlotBytes = (size_t)kChunk * kRowBytes * 2;

  int64_t pos = a.positions[b];
  const bool bad_pos = pos < 0 || pos >= a.max_len;
  if (bad_pos) pos = pos < 0 ? 0 : a.max_len - 1;
  const int p = (int)pos, len = p + 1;
  const int span = (len + kClusterCtas - 1) / kClusterCtas;
  const int t0 = rank * span, t1 = min(t0 + span, len);
  const int n = t1 > t0 ? t1 - t0 : 0;
  const int chunks = (n + kChunk - 1) / kChunk;
  const size_t kv_base = ((size_t)b * a.nkv + kh) * a.max_len * kHeadDim;
  const bool owner = t0 <= p && p < t1;

  auto issue = [&](int c) {
    const int slot = c & 1, cs = t0 + c * kChunk, rows = min(kChunk, t1 - cs);
    const unsigned bytes = (unsigned)(rows * kRowBytes);
    uint8_t* kdst = sm + (size_t)slot * kSlotBytes;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(attn_smem_u32(&full[slot])),
                 "r"(2 * bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     attn_smem_u32(kdst)), "l"(a.k_cache + kv_base + (size_t)cs * kHeadDim), "r"(bytes),
                 "r"(attn_smem_u32(&full[slot])) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     attn_smem_u32(kdst + kSlotBytes / 2)), "l"(a.v_cache + kv_base + (size_t)cs * kHeadDim),
                 "r"(bytes), "r"(attn_smem_u32(&full[slot])) : "memory");
  };
  auto wait_slot = [&](int c) -> bool {
    for (long it = 0; it < (1L << 22); ++it) {
      uint32_t done;
      asm volatile("{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n selp.u32 %0, 1, 0, q;\n}"
                   : "=r"(done) : "r"(attn_smem_u32(&full[c & 1])), "r"((unsigned)((c >> 1) & 1)) : "memory");
      if (done) return true;
    }
    return false;
  };

  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(attn_smem_u32(&full[0])) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(attn_smem_u32(&full[1])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    failed = 0;
    // rows before `position` were written by earlier steps: fetch before the wait
    for (int c = 0; c < 2 && c < chunks; ++c) issue(c);
  }
  if (tid < REP) { m_run[tid] = -INFINITY; l_run[tid] = 0.f; }
  // Inputs that do not depend on the previous kernel: this row's RoPE factors and the
  // head-norm weights, for warps that rotate a head (q heads: warps < REP; k: warp REP).
  const bool rotates = warp < REP || (warp == REP && owner);
  uint2 cw = make_uint2(0, 0), sw = make_uint2(0, 0), nw = make_uint2(0, 0);
  if (rotates) {
    cw = *reinterpret_cast<const uint2*>(a.cos_tab + (size_t)p * kHeadDim + 4 * lane);
    sw = *reinterpret_cast<const uint2*>(a.sin_tab + (size_t)p * kHeadDim + 4 * lane);
    nw = *reinterpret_cast<const uint2*>((warp < REP ? a.q_norm : a.k_norm) + 4 * lane);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (bad_pos && a.status && tid == 0 && rank == 0) atomicExch(a.status, 1);
  const __nv_bfloat16* src = a.qkv + (size_t)b * qkv_w;

  // Head RMSNorm + rotate-half RoPE (kernels.py:158-163); q rounded to bf16 as the reference
  // stores it (kernels.py:165), kept as fp32 for the dot products.
  uint2 krow = make_uint2(0, 0), vrow = make_uint2(0, 0);
  if (rotates) {
    const int row = warp < REP ? kh * REP + warp : a.nq + kh;
    const uint2 r = *reinterpret_cast<const uint2*>(src + (size_t)row * kHeadDim + 4 * lane);
    if (warp == REP) vrow = *reinterpret_cast<const uint2*>(src + (size_t)(a.nq + a.nkv + kh) * kHeadDim + 4 * lane);
    float x[4] = {bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y)};
    const float wv[4] = {bf16_lo(nw.x), bf16_hi(nw.x), bf16_lo(nw.y), bf16_hi(nw.y)};
    const float cv[4] = {bf16_lo(cw.x), bf16_hi(cw.x), bf16_lo(cw.y), bf16_hi(cw.y)};
    const float sv[4] = {bf16_lo(sw.x), bf16_hi(sw.x), bf16_lo(sw.y), bf16_hi(sw.y)};
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / 128.f + a.eps);
    float y[4], part[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] = round_bf16(round_bf16(x[i] * inv) * wv[i]);
#pragma unroll
    for (int i = 0; i < 4; ++i) part[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);  // partner d +- 64
    const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = round_bf16(round_bf16(y[i] * cv[i]) + round_bf16(sign * part[i] * sv[i]));
    if (warp < REP) {
      // dims 4 lane .. +3 sit in quarter lane / 8
      *reinterpret_cast<float4*>(&qs[(warp * 4 + (lane >> 3)) * kQStride + 4 * (lane & 7)]) =
          make_float4(x[0], x[1], x[2], x[3]);
    } else {
      __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
      krow.x = *reinterpret_cast<uint32_t*>(&lo);
      krow.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(a.k_cache + kv_base + (size_t)p * kHeadDim + 4 * lane) = krow;
      *reinterpret_cast<uint2*>(a.v_cache + kv_base + (size_t)p * kHeadDim + 4 * lane) = vrow;
    }
  }

  // P.V accumulators: thread (pair of dims dp, token group tg), all query heads.
  const int dp = tid & 63, tg = tid >> 6;
  float acc[REP][2];
#pragma unroll
  for (int h = 0; h < REP; ++h) acc[h][0] = acc[h][1] = 0.f;
  __syncthreads();

  int c = 0;
  for (; c < chunks; ++c) {
    if (!__syncthreads_and(wait_slot(c) ? 1 : 0)) break;
    // every thread is past chunk c - 1: its slot (and pr) may be reused
    if (tid == 0 && c >= 1 && c + 1 < chunks) issue(c + 1);
    const int slot = c & 1, cs = t0 + c * kChunk, rows = min(kChunk, t1 - cs);
    const __nv_bfloat16* ks = reinterpret_cast<const __nv_bfloat16*>(sm + (size_t)slot * kSlotBytes);
    const __nv_bfloat16* vs = ks + (size_t)kChunk * kHeadDim;
    if (owner && p >= cs && p < cs + rows) {  // the chunk holding this step's row (CTA-uniform)
      if (warp == REP) {
        *reinterpret_cast<uint2*>(const_cast<__nv_bfloat16*>(ks) + (size_t)(p - cs) * kHeadDim + 4 * lane) = krow;
        *reinterpret_cast<uint2*>(const_cast<__nv_bfloat16*>(vs) + (size_t)(p - cs) * kHeadDim + 4 * lane) = vrow;
      }
      __syncthreads();
    }
    // logits: item = ((t * REP) + h) * 4 + quarter; four consecutive lanes share (t, h)
    const int items = rows * REP * 4;
    for (int base = 0; base < items; base += kAttnThreads) {
      const int item = base + tid;
      const int qt = item & 3, h = (item >> 2) % REP, t = (item >> 2) / REP;
      float d0 = 0.f, d1 = 0.f;
      if (item < items) {
        const uint4* k4 = reinterpret_cast<const uint4*>(ks + (size_t)t * kHeadDim + qt * 32);
        const float4* q4 = reinterpret_cast<const float4*>(&qs[(h * 4 + qt) * kQStride]);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = (jj + qt) & 3;  // quarters 0 / 2 (1 / 3) share banks: rotate the order
          const uint4 kk = k4[j];
          const float4 qa = q4[2 * j], qb = q4[2 * j + 1];
          d0 = fmaf(qa.x, bf16_lo(kk.x), d0);
          d1 = fmaf(qa.y, bf16_hi(kk.x), d1);
          d0 = fmaf(qa.z, bf16_lo(kk.y), d0);
          d1 = fmaf(qa.w, bf16_hi(kk.y), d1);
          d0 = fmaf(qb.x, bf16_lo(kk.z), d0);
          d1 = fmaf(qb.y, bf16_hi(kk.z), d1);
          d0 = fmaf(qb.z, bf16_lo(kk.w), d0);
          d1 = fmaf(qb.w, bf16_hi(kk.w), d1);
        }
      }
      float v = d0 + d1;
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (item < items && qt == 0) pr[t][h] = v * kScale;
    }
    __syncthreads();
    // online softmax: warp h owns query head h
    if (warp < REP) {
      const int h = warp;
      float m = -INFINITY;
      for (int t = lane; t < rows; t += 32) m = fmaxf(m, pr[t][h]);
      m = warp_max(m);
      const float mnew = fmaxf(m_run[h], m);
      float s = 0.f;
      for (int t = lane; t < rows; t += 32) {
        const float e = expf(pr[t][h] - mnew);
        pr[t][h] = e;
        s += e;
      }
      s = warp_sum(s);
      if (lane == 0) {
        const float sc = expf(m_run[h] - mnew);
        scale[h] = sc;
        l_run[h] = l_run[h] * sc + s;
        m_run[h] = mnew;
      }
    }
    __syncthreads();
    {
      float scl[REP];
#pragma unroll
      for (int h = 0; h < REP; ++h) scl[h] = scale[h];
#pragma unroll
      for (int h = 0; h < REP; ++h) { acc[h][0] *= scl[h]; acc[h][1] *= scl[h]; }
      const uint32_t* v2 = reinterpret_cast<const uint32_t*>(vs) + dp;
#pragma unroll 4
      for (int t = tg; t < rows; t += kTokenGroups) {
        const uint32_t vv = v2[(size_t)t * (kHeadDim / 2)];
        const float va = bf16_lo(vv), vb = bf16_hi(vv);
#pragma unroll
        for (int h = 0; h < REP; ++h) {
          const float ph = pr[t][h];
          acc[h][0] = fmaf(ph, va, acc[h][0]);
          acc[h][1] = fmaf(ph, vb, acc[h][1]);
        }
      }
    }
  }
  if (c < chunks) {  // a copy did not land within the bound
    if (tid == 0) {
      failed = 1;
      if (a.status) atomicExch(a.status, 3);
      for (int k = c; k < chunks && k < c + 2; ++k) wait_slot(k);  // drain this CTA's copies
    }
    __syncthreads();
  }
  // sum the token groups, push each 16-dim slice to its owner rank's inbox
#pragma unroll
  for (int h = 0; h < REP; ++h) *reinterpret_cast<float2*>(&red[tg][h][2 * dp]) = make_float2(acc[h][0], acc[h][1]);
  __syncthreads();
  for (int item = tid; item < REP * kHeadDim; item += kAttnThreads) {
    const int h = item / kHeadDim, d = item - h * kHeadDim;
    float o = 0.f;
#pragma unroll
    for (int g = 0; g < kTokenGroups; ++g) o += red[g][h][d];
    *cluster.map_shared_rank(&inbox[rank][h][d & 15], d >> 4) = o;
  }
  if (tid < REP * kClusterCtas) {
    const int h = tid % REP, dst = tid / REP;
    *cluster.map_shared_rank(&minbox[rank][h], dst) = m_run[h];
    *cluster.map_shared_rank(&linbox[rank][h], dst) = l_run[h];
  }
  cluster.sync();  // publishes every push; afterwards only local shared memory is read
  if (tid < REP * 16) {
    const int h = tid >> 4, dd = tid & 15;
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kClusterCtas; ++r) M = fmaxf(M, minbox[r][h]);
    float S = 0.f, O = 0.f;
#pragma unroll
    for (int r = 0; r < kClusterCtas; ++r) {
      const float mr = minbox[r][h];
      const float w = mr == -INFINITY ? 0.f : expf(mr - M);
      S = fmaf(w, linbox[r][h], S);
      O = fmaf(w, inbox[r][h][dd], O);
    }
    a.out[(size_t)b * a.nq * kHeadDim + (kh * REP + h) * kHeadDim + 16 * rank + dd] = to_bf16(O / S);
  }
}

// ----------------------------------------------------------------------------
// Warp-split tensor-core decode attention (default): the same cluster, copies, QK-norm / RoPE
// and distributed-shared-memory merge as attention_cluster, but inside a CTA every warp keeps
// its own online softmax over 16-token sub-blocks of each chunk (sub-block i of a chunk goes to
// warp i mod 8): S = Q K^T for its 16 tokens (2 n-tiles x 8 k-steps of mma.sync with the query
// heads as zero-padded A rows), the max / exp / sum over its lane quad, P straight from the S
// accumulator registers into the A fragments of O += P V (P as bf16 hi + lo), O for all 128
// dims in registers. No CTA barrier per chunk: each warp releases a slot through an mbarrier
// ("empty", one arrival per warp) and the last warp refills it; the warps' (m, l, O) are
// merged once at the end, then the cluster merge as before over CL = 8, 4 or 2 CTAs per KV
// head (fewer for large batches: longer spans per CTA). K and V chunks arrive as four TMA
// tensor boxes with the 128-byte swizzle (attn_swz), so every ldmatrix is conflict-free.
constexpr int kWsWarps = kAttnThreads / 32;

template <int REP, int kChunk, int CL, bool OPROJ = false>
__global__ void __launch_bounds__(kAttnThreads, OPROJ ? 1 : 2)
    attention_ws(AttnArgs a, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(128) uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kQStride = 36;  // floats per 32-dim quarter of q (+4 pad)
  constexpr size_t kSlotBytes = (size_t)kChunk * kHeadDim * 2 * 2;
  __shared__ __align__(16) float qs[REP * 4 * kQStride];
  // each warp's unnormalised O; with the o_proj tail it lives in the K/V slots (free by then),
  // which leaves the shared memory to this CTA's W_o blocks
  __shared__ __align__(16) float wo_s[OPROJ ? 1 : kWsWarps][REP][OPROJ ? 1 : kHeadDim];
  float (*wo)[REP][kHeadDim] = OPROJ ? reinterpret_cast<float (*)[REP][kHeadDim]>(sm)
                                     : reinterpret_cast<float (*)[REP][kHeadDim]>(&wo_s[0][0][0]);
  constexpr int kOw = OPROJ ? REP * kHeadDim : 1;  // this KV head's slice of the o_proj input
  constexpr int kSpk = OPROJ ? REP * kHeadDim / kSliceCols : 1;  // its 256-column slices
  __shared__ __align__(16) float att_s[kOw];          // the gathered attention output (bf16 values)
  __shared__ __align__(16) uint4 oxp[OPROJ ? kOw / 8 : 1];  // fp16 operand pairs (GEMV layout)
  __shared__ float oxsum[OPROJ ? kOw / 32 : 1];       // c * sum of each 32-column group
  __shared__ float oscale[kSpk];                      // 2^24 / c per slice
  __shared__ __align__(16) uint4 ozero16[4];
  __shared__ __align__(8) uint64_t wbar;              // W_o blocks landed
  __shared__ int olast;
  __shared__ float wm[kWsWarps][REP], wl[kWsWarps][REP];
  constexpr int kSl = kHeadDim / CL;  // output dims each rank finishes
  __shared__ __align__(16) float inbox[CL][REP][kSl];
  __shared__ float minbox[CL][REP], linbox[CL][REP];
  __shared__ float m_run[REP], l_run[REP];
  __shared__ __align__(8) uint64_t full[2];
  __shared__ __align__(8) uint64_t empty[2];
  __shared__ int failed;
  __shared__ int issued;  // chunks whose copies were issued (drained on failure)
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int kh = blockIdx.x / CL, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int qkv_w = (a.nq + 2 * a.nkv) * kHeadDim;

  int64_t pos = a.positions[b];
  const bool bad_pos = pos < 0 || pos >= a.max_len;
  if (bad_pos) pos = pos < 0 ? 0 : a.max_len - 1;
  const int p = (int)pos, len = p + 1;
  const int span = (len + CL - 1) / CL;
  const int t0 = rank * span, t1 = min(t0 + span, len);
  const int n = t1 > t0 ? t1 - t0 : 0;
  const int chunks = (n + kChunk - 1) / kChunk;
  const size_t kv_base = ((size_t)b * a.nkv + kh) * a.max_len * kHeadDim;
  const bool owner = t0 <= p && p < t1;

  auto issue = [&](int c) {  // one thread: four boxes of 64 dims x kChunk rows
    const int slot = c & 1, cs = t0 + c * kChunk;
    const int y = (int)(((size_t)b * a.nkv + kh) * a.max_len) + cs;
    uint8_t* dst = sm + (size_t)slot * kSlotBytes;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(attn_smem_u32(&full[slot])),
                 "r"((unsigned)(4 * kChunk * 128)) : "memory");
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const CUtensorMap* map = q < 2 ? &kmap : &vmap;
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
              attn_smem_u32(dst + (size_t)q * kChunk * 128)),
          "l"(reinterpret_cast<uint64_t>(map)), "r"((q & 1) * 64), "r"(y), "r"(attn_smem_u32(&full[slot]))
          : "memory");
    }
  };
  auto wait_bar = [&](uint64_t* bar, unsigned parity) -> bool {
    for (long it = 0; it < (1L << 22); ++it) {
      uint32_t done;
      asm volatile("{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n selp.u32 %0, 1, 0, q;\n}"
                   : "=r"(done) : "r"(attn_smem_u32(bar)), "r"(parity) : "memory");
      if (done) return true;
    }
    return false;
  };

  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(attn_smem_u32(&full[0])) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(attn_smem_u32(&full[1])) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(attn_smem_u32(&empty[0])), "r"(kWsWarps) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(attn_smem_u32(&empty[1])), "r"(kWsWarps) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    failed = 0;
    issued = min(2, chunks);
    // rows before `position` were written by earlier steps: fetch before the wait
    for (int c = 0; c < 2 && c < chunks; ++c) issue(c);
    if constexpr (OPROJ) {
      // this CTA's W_o blocks never depend on the previous kernel either: tiles
      // [rank * tpc, +tpc) of the output, slices [kh * kSpk, +kSpk) of the input (the query
      // heads of this KV head), one bulk copy of kSpk consecutive blocks per tile
      const int S = a.nq * kHeadDim / kSliceCols, tpc = a.n_out / 16 / CL;
      const unsigned bb = (unsigned)(kCodeBytes + kScaleBytes + (a.wo_zeros ? kZeroBytes : 0));
      uint8_t* wdst = sm + 2 * kSlotBytes;
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(attn_smem_u32(&wbar)) : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(attn_smem_u32(&wbar)),
                   "r"((unsigned)(tpc * kSpk) * bb) : "memory");
      for (int t = 0; t < tpc; ++t) {
        const uint8_t* src = a.wo + ((size_t)(rank * tpc + t) * S + (size_t)kh * kSpk) * bb;
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         attn_smem_u32(wdst + (size_t)t * kSpk * bb)),
                     "l"(src), "r"(kSpk * bb), "r"(attn_smem_u32(&wbar))
                     : "memory");
      }
    }
  }
  if (OPROJ && tid < 4) ozero16[tid] = make_uint4(0, 0, 0, 0);
  // Inputs that do not depend on the previous kernel: this row's RoPE factors and the
  // head-norm weights, for warps that rotate a head (q heads: warps < REP; k: warp REP).
  const bool rotates = warp < REP || (warp == REP && owner);
  uint2 cw = make_uint2(0, 0), sw = make_uint2(0, 0), nw = make_uint2(0, 0);
  if (rotates) {
    cw = *reinterpret_cast<const uint2*>(a.cos_tab + (size_t)p * kHeadDim + 4 * lane);
    sw = *reinterpret_cast<const uint2*>(a.sin_tab + (size_t)p * kHeadDim + 4 * lane);
    nw = *reinterpret_cast<const uint2*>((warp < REP ? a.q_norm : a.k_norm) + 4 * lane);
  }
  __syncthreads();
  pdl_wait();
  pdl_trigger();
  if (bad_pos && a.status && tid == 0 && rank == 0) atomicExch(a.status, 1);
  const __nv_bfloat16* src = a.qkv + (size_t)b * qkv_w;

  // Head RMSNorm + rotate-half RoPE (kernels.py:158-163); q rounded to bf16 as the reference
  // stores it (kernels.py:165); the new K / V row goes to the cache (and, below, to the chunk).
  uint2 krow = make_uint2(0, 0), vrow = make_uint2(0, 0);
  if (rotates) {
    const int row = warp < REP ? kh * REP + warp : a.nq + kh;
    const uint2 r = *reinterpret_cast<const uint2*>(src + (size_t)row * kHeadDim + 4 * lane);
    if (warp == REP) vrow = *reinterpret_cast<const uint2*>(src + (size_t)(a.nq + a.nkv + kh) * kHeadDim + 4 * lane);
    float x[4] = {bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y)};
    const float wv[4] = {bf16_lo(nw.x), bf16_hi(nw.x), bf16_lo(nw.y), bf16_hi(nw.y)};
    const float cv[4] = {bf16_lo(cw.x), bf16_hi(cw.x), bf16_lo(cw.y), bf16_hi(cw.y)};
    const float sv[4] = {bf16_lo(sw.x), bf16_hi(sw.x), bf16_lo(sw.y), bf16_hi(sw.y)};
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / 128.f + a.eps);
    float y[4], part[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] = round_bf16(round_bf16(x[i] * inv) * wv[i]);
#pragma unroll
    for (int i = 0; i < 4; ++i) part[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);  // partner d +- 64
    const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = round_bf16(round_bf16(y[i] * cv[i]) + round_bf16(sign * part[i] * sv[i]));
    if (warp < REP) {
      *reinterpret_cast<float4*>(&qs[(warp * 4 + (lane >> 3)) * kQStride + 4 * (lane & 7)]) =
          make_float4(x[0], x[1], x[2], x[3]);
    } else {
      __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
      krow.x = *reinterpret_cast<uint32_t*>(&lo);
      krow.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(a.k_cache + kv_base + (size_t)p * kHeadDim + 4 * lane) = krow;
      *reinterpret_cast<uint2*>(a.v_cache + kv_base + (size_t)p * kHeadDim + 4 * lane) = vrow;
    }
  }
  __syncthreads();

  // lane (g, t4): query head g < REP is A row g; S / P / O fragments hold rows g (and g + 8:
  // zero A rows, never read)
  const int g = lane >> 2, t4 = lane & 3;
  const bool hrow = g < REP;
  uint32_t qa[8][2];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {  // dims 16 kk + 2 t4 (+1) and + 8: quarter kk / 2 of qs
    const float* qrow = &qs[((hrow ? g : 0) * 4 + (kk >> 1)) * kQStride + (kk & 1) * 16 + 2 * t4];
    qa[kk][0] = hrow ? attn_pack(qrow[0], qrow[1]) : 0u;
    qa[kk][1] = hrow ? attn_pack(qrow[8], qrow[9]) : 0u;
  }
  float o[16][4] = {};
  float mrow = -INFINITY, lrow = 0.f;  // head g's running max and sum over this warp's tokens
  constexpr int kSub = kChunk / 16;     // 16-token sub-blocks per chunk
  volatile int* vfailed = &failed;
  for (int c = 0; c < chunks; ++c) {
    const int slot = c & 1, cs = t0 + c * kChunk, rows = min(kChunk, t1 - cs);
    const bool got = !*vfailed && __all_sync(0xffffffffu, wait_bar(&full[slot], (unsigned)((c >> 1) & 1)));
    if (!got && lane == 0) *vfailed = 1;
    uint8_t* kbase = sm + (size_t)slot * kSlotBytes;
    uint8_t* vbase = kbase + kSlotBytes / 2;
    // this step's row (the copy may predate its write) and, in a short last chunk, zero V rows
    // past the end (they meet zero weights); both CTA-uniform, the only barriers in the loop
    const bool fresh_here = owner && p >= cs && p < cs + rows;
    const bool pad_v = rows < kChunk;
    if (fresh_here || pad_v) {
      if (got) {
        if (fresh_here && warp == REP) {
          const uint32_t off = attn_swz<kChunk>(p - cs, lane >> 1) + 8 * (lane & 1);
          *reinterpret_cast<uint2*>(kbase + off) = krow;
          *reinterpret_cast<uint2*>(vbase + off) = vrow;
        }
        if (pad_v)
          for (int i = tid; i < 2 * (kChunk - rows) * 8; i += kAttnThreads) {
            const int box = i / ((kChunk - rows) * 8), rem = i - box * (kChunk - rows) * 8;
            *reinterpret_cast<uint4*>(vbase + (size_t)box * kChunk * 128 + (size_t)(rows + rem / 8) * 128 +
                                      (rem & 7) * 16) = make_uint4(0, 0, 0, 0);
          }
      }
      __syncthreads();
    }
    if (got) {
      const uint32_t kb = attn_smem_u32(kbase), vb = attn_smem_u32(vbase);
      for (int i = warp; i < kSub && 16 * i < rows; i += kWsWarps) {
        const int tok0 = 16 * i;
        float s[2][4] = {};
#pragma unroll
        for (int jn = 0; jn < 2; ++jn)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            uint32_t b0, b1;
            attn_ldsm_x2(b0, b1, kb + attn_swz<kChunk>(tok0 + 8 * jn + (lane & 7), 2 * kk + ((lane >> 3) & 1)));
            attn_mma(s[jn], qa[kk][0], qa[kk][1], b0, b1);
          }
        // logits of tokens tok0 + 8 jn + 2 t4 + e (rows past the chunk: -inf), the quad's max
        float bm = -INFINITY;
#pragma unroll
        for (int jn = 0; jn < 2; ++jn)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const bool live = tok0 + 8 * jn + 2 * t4 + e < rows;
            s[jn][e] = live ? s[jn][e] * kScale : -INFINITY;
            bm = fmaxf(bm, s[jn][e]);
          }
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
        const float mnew = fmaxf(mrow, bm);  // finite: every sub-block holds a live token
        const float corr = mrow == -INFINITY ? 0.f : expf(mrow - mnew);
        float pv[2][2], psum = 0.f;
#pragma unroll
        for (int jn = 0; jn < 2; ++jn)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            pv[jn][e] = s[jn][e] == -INFINITY ? 0.f : expf(s[jn][e] - mnew);
            psum += pv[jn][e];
          }
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        lrow = lrow * corr + psum;
        mrow = mnew;
#pragma unroll
        for (int jd = 0; jd < 16; ++jd) {
          o[jd][0] *= corr;
          o[jd][1] *= corr;
        }
        // P (k = the sub-block's 16 tokens) as A fragments, bf16 hi + lo; zero for rows g >= REP
        const uint32_t h0 = hrow ? attn_pack(pv[0][0], pv[0][1]) : 0u, h2 = hrow ? attn_pack(pv[1][0], pv[1][1]) : 0u;
        const uint32_t l0 = hrow ? attn_pack(pv[0][0] - bf16_lo(h0), pv[0][1] - bf16_hi(h0)) : 0u;
        const uint32_t l2 = hrow ? attn_pack(pv[1][0] - bf16_lo(h2), pv[1][1] - bf16_hi(h2)) : 0u;
#pragma unroll
        for (int jp = 0; jp < 8; ++jp) {  // dims 16 jp .. 16 jp + 15: n-tiles 2 jp, 2 jp + 1
          uint32_t bv[4];
          attn_ldsm_x4_t(bv, vb + attn_swz<kChunk>(tok0 + (lane & 7) + 8 * ((lane >> 3) & 1), 2 * jp + (lane >> 4)));
          attn_mma(o[2 * jp], h0, h2, bv[0], bv[1]);
          attn_mma(o[2 * jp + 1], h0, h2, bv[2], bv[3]);
          attn_mma(o[2 * jp], l0, l2, bv[0], bv[1]);
          attn_mma(o[2 * jp + 1], l0, l2, bv[2], bv[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(attn_smem_u32(&empty[slot])) : "memory");
    // the last warp refills this slot with chunk c + 2 once every warp has released it
    if (warp == kWsWarps - 1 && lane == 0 && c + 2 < chunks && !*vfailed) {
      if (wait_bar(&empty[slot], (unsigned)((c >> 1) & 1))) {
        issue(c + 2);
        issued = c + 3;
      } else {
        *vfailed = 1;
      }
    }
  }
  __syncthreads();
  if (failed) {  // a copy or a slot release did not come within the bound: drain, flag, merge what there is
    if (tid == 0) {
      if (a.status) atomicExch(a.status, 3);
      // at most the last copy of each slot can still be in flight
      for (int k = max(0, issued - 2); k < issued; ++k) wait_bar(&full[k & 1], (unsigned)((k >> 1) & 1));
    }
    __syncthreads();
  }
  // the warps' (m, l, O) -> the CTA's
  if (hrow && t4 == 0) {
    wm[warp][g] = mrow;
    wl[warp][g] = lrow;
  }
  if (hrow) {
#pragma unroll
    for (int jd = 0; jd < 16; ++jd)
      *reinterpret_cast<float2*>(&wo[warp][g][8 * jd + 2 * t4]) = make_float2(o[jd][0], o[jd][1]);
  }
  __syncthreads();
  if (tid < REP) {
    float M = -INFINITY, L = 0.f;
    for (int w = 0; w < kWsWarps; ++w) M = fmaxf(M, wm[w][tid]);
    for (int w = 0; w < kWsWarps; ++w) {
      const float f = wm[w][tid] == -INFINITY ? 0.f : expf(wm[w][tid] - M);
      wm[w][tid] = f;  // now the warp's weight
      L = fmaf(f, wl[w][tid], L);
    }
    m_run[tid] = M;
    l_run[tid] = L;
  }
  __syncthreads();
  for (int item = tid; item < REP * kHeadDim; item += kAttnThreads) {
    const int h = item / kHeadDim, d = item - h * kHeadDim;
    float ov = 0.f;
#pragma unroll
    for (int w = 0; w < kWsWarps; ++w) ov = fmaf(wm[w][h], wo[w][h][d], ov);
    *cluster.map_shared_rank(&inbox[rank][h][d % kSl], d / kSl) = ov;
  }
  if (tid < REP * CL) {
    const int h = tid % REP, dst = tid / REP;
    *cluster.map_shared_rank(&minbox[rank][h], dst) = m_run[h];
    *cluster.map_shared_rank(&linbox[rank][h], dst) = l_run[h];
  }
  cluster.sync();  // publishes every push; afterwards only local shared memory is read
  for (int item = tid; item < REP * kSl; item += kAttnThreads) {
    const int h = item / kSl, dd = item % kSl;
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < CL; ++r) M = fmaxf(M, minbox[r][h]);
    float S = 0.f, O = 0.f;
#pragma unroll
    for (int r = 0; r < CL; ++r) {
      const float mr = minbox[r][h];
      const float w = mr == -INFINITY ? 0.f : expf(mr - M);
      S = fmaf(w, linbox[r][h], S);
      O = fmaf(w, inbox[r][h][dd], O);
    }
    const __nv_bfloat16 ob = to_bf16(O / S);
    a.out[(size_t)b * a.nq * kHeadDim + (kh * REP + h) * kHeadDim + kSl * rank + dd] = ob;
    if constexpr (OPROJ) {  // every CTA of the cluster needs the whole head group as o_proj input
      const float ov = __bfloat162float(ob);
#pragma unroll
      for (int r = 0; r < CL; ++r) *cluster.map_shared_rank(&att_s[h * kHeadDim + kSl * rank + dd], r) = ov;
    }
  }
  if constexpr (OPROJ) {
    cluster.sync();  // the gathered input is complete in every CTA (and no CTA writes remote memory later)
    // ---- o_proj, split-K over the KV heads: y_kh = W_o[:, kh's columns] . attention(kh) ----
    // The input slices as the packed GEMV takes them (w4a16_stream.cu): per 256-column slice a
    // power-of-two scale c, fp16 pairs (x_j c, x_{j+4} c) / (x_{j+1} c / 16, x_{j+5} c / 16)
    // and c times each 32-column group's sum for the zero-point term.
    if (warp < kSpk) {
      const int word = warp * 32 + lane;
      float v8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v8[i] = att_s[word * 8 + i];
      float mx = 0.f, wsum = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        mx = fmaxf(mx, fabsf(v8[i]));
        wsum += v8[i];
      }
      mx = warp_max(mx);
      const int ex = mx > 0.f ? min(max((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127, -100), 100) : 0;
      const float cs = __uint_as_float((uint32_t)(127 + 9 - ex) << 23);
      oxp[word] = make_uint4(pack_half2(v8[0] * cs, v8[4] * cs), pack_half2(v8[1] * cs * 0.0625f, v8[5] * cs * 0.0625f),
                             pack_half2(v8[2] * cs, v8[6] * cs), pack_half2(v8[3] * cs * 0.0625f, v8[7] * cs * 0.0625f));
      wsum += __shfl_xor_sync(0xffffffffu, wsum, 1);
      wsum += __shfl_xor_sync(0xffffffffu, wsum, 2);
      if ((lane & 3) == 0) oxsum[word >> 2] = wsum * cs;
      if (lane == 0) oscale[warp] = __uint_as_float((uint32_t)(127 + 24 - 9 + ex) << 23);
    }
    __syncthreads();
    const bool wok = __all_sync(0xffffffffu, wait_bar(&wbar, 0u));
    if (!wok && lane == 0 && a.status) atomicExch(a.status, 3);
    const int tpc = a.n_out / 16 / CL, S = a.nq * kHeadDim / kSliceCols;
    (void)S;
    const bool zeros = a.wo_zeros != 0;
    const int bb = kCodeBytes + kScaleBytes + (zeros ? kZeroBytes : 0);
    const uint8_t* wsrc = sm + 2 * kSlotBytes;
    const int r = lane >> 2, c = lane & 3, hsel = r - 2 * c;
    constexpr int kTpw = 4;  // tiles per warp per pass
    for (int t0 = warp; t0 < tpc; t0 += kWsWarps * kTpw) {
      float acc[kTpw][2] = {};
#pragma unroll
      for (int sl = 0; sl < kSpk; ++sl) {
        uint32_t bl[16], bh[16];
        const uint4* pl = hsel == 0 ? oxp + sl * 32 + 8 * c : ozero16;
        const uint4* ph = hsel == 1 ? oxp + sl * 32 + 8 * c + 4 : ozero16;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 ql = pl[u], qh = ph[u];
          bl[4 * u] = ql.x; bl[4 * u + 1] = ql.y; bl[4 * u + 2] = ql.z; bl[4 * u + 3] = ql.w;
          bh[4 * u] = qh.x; bh[4 * u + 1] = qh.y; bh[4 * u + 2] = qh.z; bh[4 * u + 3] = qh.w;
        }
        const float z0 = hsel == 0 ? -oxsum[sl * 8 + 2 * c] : 0.f;
        const float z1 = hsel == 1 ? -oxsum[sl * 8 + 2 * c + 1] * 0.0625f : 0.f;
        const float h0 = __half2float(__float2half_rn(z0)), h1 = __half2float(__float2half_rn(z1));
        const uint32_t bz0 = pack_half2(h0, h1), bz1 = pack_half2(z0 - h0, z1 - h1);
        const float scale = oscale[sl];
#pragma unroll
        for (int i = 0; i < kTpw; ++i) {
          const int t = t0 + kWsWarps * i;
          if (t >= tpc || !wok) continue;
          const BlockRegs bk = load_block(wsrc + ((size_t)t * kSpk + sl) * bb, lane, zeros);
          float va, vb;
          block_dot<2>(bk, bl, bh, bz0, bz1, va, vb);
          acc[i][0] += va * scale;
          acc[i][1] += vb * scale;
        }
      }
      if (c == 0) {
#pragma unroll
        for (int i = 0; i < kTpw; ++i) {
          const int t = t0 + kWsWarps * i;
          if (t >= tpc) continue;
          const int row = (rank * tpc + t) * 16 + r;
          a.opart[(size_t)kh * a.n_out + row] = acc[i][0];
          a.opart[(size_t)kh * a.n_out + row + 8] = acc[i][1];
        }
      }
    }
    // The KV heads' partials of this CTA's rows are summed by the last of their nkv CTAs, in
    // KV-head order (deterministic); the counter is left at zero for the next call.
    __threadfence();
    __syncthreads();
    if (tid == 0) olast = atomicAdd(&a.otickets[rank], 1u) == (unsigned)(a.nkv - 1) ? 1 : 0;
    __syncthreads();
    if (olast) {
      __threadfence();
      for (int i = tid; i < tpc * 16; i += kAttnThreads) {
        const int row = rank * tpc * 16 + i;
        float y = 0.f;
        for (int k = 0; k < a.nkv; ++k) y += __ldcg(a.opart + (size_t)k * a.n_out + row);
        a.oout[row] = to_bf16(y);
      }
      if (tid == 0) a.otickets[rank] = 0u;
    }
  }
}

// MT_ATTN_TC = 0 selects the CUDA-core chunk arithmetic (fp32 FMAs on shared memory); the
// default is the tensor-core one.
static bool attention_tc() {
  static int v = -1;
  if (v < 0) {
    const char* env = getenv("MT_ATTN_TC");
    v = (env && env[0] == '0' && env[1] == 0) ? 0 : 1;
  }
  return v == 1;
}

// TMA map of a cache [rows, 128] bf16 (rows = batch x nkv x max_len): boxes of 64 dims x ch
// rows with the 128-byte swizzle; rows past the end read as zeros. Encoded maps are kept per
// (pointer, rows, box) so that eager decode steps do not re-encode them every layer.
static bool cache_map(CUtensorMap* map, const void* base, long long rows, int ch) {
  struct Entry {
    const void* base;
    long long rows;
    int ch;
    CUtensorMap map;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int used = 0, next = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].base == base && cache[i].rows == rows && cache[i].ch == ch) {
      *map = cache[i].map;
      return true;
    }
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kHeadDim * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)ch};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  cache[next] = Entry{base, rows, ch, *map};
  next = (next + 1) % 64;
  if (used < 64) ++used;
  return true;
}

template <int REP, int CH>
static cudaError_t launch_cluster_rep(cudaLaunchConfig_t& cfg, const AttnArgs& a, int batch) {
  CUtensorMap kmap, vmap;
  memset(&kmap, 0, sizeof(kmap));
  memset(&vmap, 0, sizeof(vmap));
  const long long rows = (long long)batch * a.nkv * a.max_len;
  const bool tc = CH >= 64 && attention_tc() && rows < (1LL << 31) && cache_map(&kmap, a.k_cache, rows, CH) &&
                  cache_map(&vmap, a.v_cache, rows, CH);
  cudaError_t e;
  if constexpr (CH >= 64) {
    if (tc) {
      // CTAs per KV head: the fewest of 8, 4, 2 that still put at least 1.5 CTAs on every SM
      // (longer spans per CTA amortise its fixed cost; fewer CTAs leave SMs idle). Measured at
      // 32 x 2048: 8 -> 85.5 us, 4 -> 63.7, 2 -> 55.6; at 4 x 2048: 8 -> 14.2, 4 -> 16.5.
      // MT_ATTN_CLUSTER = 2, 4 or 8 overrides.
      static int forced = -1;
      if (forced < 0) {
        const char* env = getenv("MT_ATTN_CLUSTER");
        forced = (env && (env[0] == '2' || env[0] == '4' || env[0] == '8') && env[1] == 0) ? env[0] - '0' : 0;
      }
      int cl = forced ? forced : 8;
      if (!forced)
        while (cl > 2 && 2LL * batch * a.nkv * (cl / 2) >= 3LL * sm_count()) cl /= 2;
      cfg.gridDim.x = (unsigned)(cl * a.nkv);
      cfg.attrs[0].val.clusterDim.x = (unsigned)cl;
      cfg.dynamicSmemBytes = 2 * (size_t)CH * kHeadDim * 2 * 2 + 1024;
      auto kern = cl == 2 ? attention_ws<REP, CH, 2> : cl == 4 ? attention_ws<REP, CH, 4> : attention_ws<REP, CH, 8>;
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
      if (e != cudaSuccess) return e;
      return cudaLaunchKernelEx(&cfg, kern, a, kmap, vmap);
    }
  }
  cfg.dynamicSmemBytes = 2 * (size_t)CH * kHeadDim * 2 * 2;
  e = cudaFuncSetAttribute(attention_cluster<REP, CH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)cfg.dynamicSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, attention_cluster<REP, CH>, a);
}

// Chunk size of the cluster kernel: MT_ATTN_CHUNK (32, 64 or 128) overrides the default:
// 128 tokens for one sequence (8 CTAs per KV head, one per SM), 64 while the batch's CTAs fit
// three per SM in one wave, 32 (four and more per SM) beyond. Measured at contexts
// U[256, 4096] (tokens/s, chunk 128 / 64 / 32): B = 2 886 / 938 / 815, B = 3 804 / 816 / 735,
// B = 4 1013 / 993 / 885, B = 6 1217 / 1279 / 1190; B = 64: 32 is 1.5x faster than 128.
static int attention_chunk(int batch, int nkv) {
  static int forced = -1;
  if (forced < 0) {
    const char* env = getenv("MT_ATTN_CHUNK");
    const int v = env ? atoi(env) : 0;
    forced = (v == 32 || v == 64 || v == 128) ? v : 0;
  }
  if (forced) return forced;
  if (batch == 1) return 128;
  if (attention_tc()) return 64;  // the tensor-core kernel: 4 sub-blocks of 16 tokens per chunk
  return (long long)batch * nkv * kClusterCtas <= 3LL * sm_count() ? 64 : 32;
}

static cudaError_t launch_cluster_attention(const AttnArgs& a, int batch, int rep, cudaStream_t s, int flags) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kClusterCtas * a.nkv, 1, batch);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kClusterCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & kFlagPdl) ? 2 : 1;
  const int ch = attention_chunk(batch, a.nkv);
  switch (rep) {
    case 4: return ch == 128 ? launch_cluster_rep<4, 128>(cfg, a, batch) : ch == 64 ? launch_cluster_rep<4, 64>(cfg, a, batch)
                                                                           : launch_cluster_rep<4, 32>(cfg, a, batch);
    case 2: return ch == 128 ? launch_cluster_rep<2, 128>(cfg, a, batch) : ch == 64 ? launch_cluster_rep<2, 64>(cfg, a, batch)
                                                                           : launch_cluster_rep<2, 32>(cfg, a, batch);
    default: return ch == 128 ? launch_cluster_rep<1, 128>(cfg, a, batch) : ch == 64 ? launch_cluster_rep<1, 64>(cfg, a, batch)
                                                                            : launch_cluster_rep<1, 32>(cfg, a, batch);
  }
}

// The warp-split kernel with the o_proj tail (one sequence, 8-CTA clusters, 64-token chunks:
// the two K/V slots and this CTA's W_o blocks share the shared memory).
template <int REP>
static cudaError_t launch_attention_oproj(const AttnArgs& a, cudaStream_t s, int flags) {
  constexpr int CH = 64, CL = 8;
  const long long rows = (long long)a.nkv * a.max_len;
  CUtensorMap kmap, vmap;
  memset(&kmap, 0, sizeof(kmap));
  memset(&vmap, 0, sizeof(vmap));
  if (!(rows < (1LL << 31) && cache_map(&kmap, a.k_cache, rows, CH) && cache_map(&vmap, a.v_cache, rows, CH)))
    return cudaErrorNotSupported;
  const size_t bb = kCodeBytes + kScaleBytes + (a.wo_zeros ? kZeroBytes : 0);
  const size_t wbytes = (size_t)(a.n_out / 16 / CL) * (REP * kHeadDim / kSliceCols) * bb;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CL * a.nkv, 1, 1);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.stream = s;
  cfg.dynamicSmemBytes = 2 * (size_t)CH * kHeadDim * 2 * 2 + wbytes + 1024;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & kFlagPdl) ? 2 : 1;
  auto kern = attention_ws<REP, CH, CL, true>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, kern, a, kmap, vmap);
}

static size_t attn_smem_bytes(int rep, int max_len, int splits) {
  const size_t cap = (size_t)attn_cap(max_len, splits);
  return cap * kHeadDim * 2 * 2 + (size_t)rep * cap * sizeof(float);
}

// Standalone QK-norm + RoPE + cache write (kernels.py:142-170): grid (nq + nkv, B).
__global__ void __launch_bounds__(32) qk_rope_kv(AttnArgs a, __nv_bfloat16* q_out) {
  const int h = blockIdx.x, b = blockIdx.y, lane = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  int64_t pos = a.positions[b];
  if (pos < 0 || pos >= a.max_len) {
    if (a.status && lane == 0) atomicExch(a.status, 1);
    return;
  }
  const int p = (int)pos;
  const __nv_bfloat16* src = a.qkv + (size_t)b * (a.nq + 2 * a.nkv) * kHeadDim;
  const bool is_q = h < a.nq;
  float x[4];
  const uint2 r = *reinterpret_cast<const uint2*>(src + h * kHeadDim + 4 * lane);
  x[0] = bf16_lo(r.x); x[1] = bf16_hi(r.x); x[2] = bf16_lo(r.y); x[3] = bf16_hi(r.y);
  norm_rope_head(x, is_q ? a.q_norm : a.k_norm, a.cos_tab + (size_t)p * kHeadDim,
                 a.sin_tab + (size_t)p * kHeadDim, a.eps, lane);
  __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
  uint2 o;
  o.x = *reinterpret_cast<uint32_t*>(&lo);
  o.y = *reinterpret_cast<uint32_t*>(&hi);
  if (is_q) {
    *reinterpret_cast<uint2*>(q_out + ((size_t)b * a.nq + h) * kHeadDim + 4 * lane) = o;
  } else {
    const int kh = h - a.nq;
    const size_t row = (((size_t)b * a.nkv + kh) * a.max_len + p) * kHeadDim + 4 * lane;
    *reinterpret_cast<uint2*>(a.k_cache + row) = o;
    *reinterpret_cast<uint2*>(a.v_cache + row) =
        *reinterpret_cast<const uint2*>(src + (a.nq + a.nkv + kh) * kHeadDim + 4 * lane);
  }
}

static int attn_check(const AttnArgs& a, int batch) {
  if (!a.qkv || !a.q_norm || !a.k_norm || !a.cos_tab || !a.sin_tab || !a.positions || !a.k_cache ||
      !a.v_cache || batch < 1 || a.nkv < 1 || a.nq < a.nkv || a.nq % a.nkv || a.max_len < 1)
    return kBadArgument;
  if (!aligned(a.qkv, 8) || !aligned(a.k_cache, 16) || !aligned(a.v_cache, 16) ||
      !aligned(a.positions, 8))
    return kBadArgument;
  return 0;
}

}  // namespace mt

using namespace mt;

// Fused decode attention. Replaces qk_rope_decode (src/moss_tts/_runtime/kernels.py:211-251)
// with launch_attention_ordered (attention_native.cu:91-97) and the split reduction
// (kernels.py:198-208 / attention_quant.py:7-23). `positions` is a device int64 [batch]
// array (graph-capturable). Scratch: partial fp32 [batch*nkv*splits*rep*128],
// lse fp32 [batch*nkv*splits*rep], tickets uint32 [batch*nkv] zero-initialised once.
MT_API int mt_attention_decode(const void* qkv, const void* q_norm, const void* k_norm,
                               const void* cos_tab, const void* sin_tab, const void* positions,
                               void* k_cache, void* v_cache, void* out, void* partial, void* lse,
                               void* tickets, int batch, int nq, int nkv, int max_len, int splits,
                               float eps, void* status, int flags, void* stream) {
  AttnArgs a;
  a.qkv = (const __nv_bfloat16*)qkv;
  a.q_norm = (const __nv_bfloat16*)q_norm;
  a.k_norm = (const __nv_bfloat16*)k_norm;
  a.cos_tab = (const __nv_bfloat16*)cos_tab;
  a.sin_tab = (const __nv_bfloat16*)sin_tab;
  a.positions = (const int64_t*)positions;
  a.k_cache = (__nv_bfloat16*)k_cache;
  a.v_cache = (__nv_bfloat16*)v_cache;
  a.out = (__nv_bfloat16*)out;
  a.partial = (float*)partial;
  a.lse = (float*)lse;
  a.tickets = (unsigned*)tickets;
  a.nq = nq;
  a.nkv = nkv;
  a.max_len = max_len;
  a.splits = splits;
  a.eps = eps;
  a.status = (int*)status;
  if (attn_check(a, batch) || !out || !partial || !lse || !tickets || splits < 1 || splits > 1024)
    return kBadArgument;
  const int rep = nq / nkv;
  if (rep != 4 && rep != 1 && rep != 2) return kBadArgument;
  cudaStream_t s = (cudaStream_t)stream;
  // Default: the cluster kernel (its merge needs no scratch). Flags bit 1 selects the
  // split-K kernel with the caller's scratch and `splits` splits.
  if (!(flags & 2)) return (int)launch_cluster_attention(a, batch, rep, s, flags & kFlagPdl);
  flags &= kFlagPdl;
  const size_t smem = attn_smem_bytes(rep, max_len, splits);
  if (smem > 200 * 1024) return kBadArgument;
  const dim3 grid(nkv, splits, batch);
  switch (rep) {
    case 4: return launch(attention_decode<4>, grid, dim3(128), smem, s, flags, a);
    case 2: return launch(attention_decode<2>, grid, dim3(128), smem, s, flags, a);
    default: return launch(attention_decode<1>, grid, dim3(128), smem, s, flags, a);
  }
}

// Standalone QK-norm + RoPE + K/V cache write (kernels.py:142-170, grid nq + nkv heads).
MT_API int mt_qk_rope_kv(const void* qkv, const void* q_norm, const void* k_norm,
                         const void* cos_tab, const void* sin_tab, const void* positions,
                         void* q_out, void* k_cache, void* v_cache, int batch, int nq, int nkv,
                         int max_len, float eps, void* status, int flags, void* stream) {
  AttnArgs a = {};
  a.qkv = (const __nv_bfloat16*)qkv;
  a.q_norm = (const __nv_bfloat16*)q_norm;
  a.k_norm = (const __nv_bfloat16*)k_norm;
  a.cos_tab = (const __nv_bfloat16*)cos_tab;
  a.sin_tab = (const __nv_bfloat16*)sin_tab;
  a.positions = (const int64_t*)positions;
  a.k_cache = (__nv_bfloat16*)k_cache;
  a.v_cache = (__nv_bfloat16*)v_cache;
  a.nq = nq;
  a.nkv = nkv;
  a.max_len = max_len;
  a.eps = eps;
  a.status = (int*)status;
  if (attn_check(a, batch) || !q_out || !aligned(q_out, 8)) return kBadArgument;
  return launch(qk_rope_kv, dim3(nq + nkv, batch), dim3(32), 0, (cudaStream_t)stream, flags, a,
                (__nv_bfloat16*)q_out);
}

// ----------------------------------------------------------------------------
// Scratch-free decode attention.
//
// Some callers of this library cannot allocate device memory for the split-K
// partials: real-time audio callbacks that must not block on an allocator (a
// cudaMalloc can synchronise the device and stall for milliseconds), and
// foreign-function hosts (plugins, embedded runtimes) that own no device
// allocator at all. For them the partials, log-sum-exp values and merge tickets
// live in one fixed array of this library's own device memory. Every GPU that
// loads the library holds that array (about 1.04 MiB) until the process exits.
// The array is shared by all calls on a device and keeps the previous call's
// contents; calls whose kernels overlap on the GPU (for example, from two streams
// at once) race on it and must be serialised by the caller.
#include <mutex>

namespace mt {
namespace {
constexpr size_t kNoAllocPartial = 262144;  // fp32 partials: batch*nkv*splits*(nq/nkv)*128
constexpr size_t kNoAllocLse = 8192;        // fp32 log-sum-exp: batch*nkv*splits*(nq/nkv)
constexpr size_t kNoAllocTickets = 1024;    // merge counters: batch*nkv

struct NoAllocScratch {
  float partial[kNoAllocPartial];
  float lse[kNoAllocLse];
  unsigned tickets[kNoAllocTickets];
};

static __device__ __align__(256) NoAllocScratch g_attention_scratch;

std::mutex g_scratch_mutex;
NoAllocScratch* g_scratch_address[128] = {};

// Device address of the scratch array for the current device. The symbol's name is
// only a host-side handle, so it is resolved once per device (with that device
// current) through cudaGetSymbolAddress and cached.
cudaError_t scratch_for_current_device(NoAllocScratch** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_address[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_address[dev] = static_cast<NoAllocScratch*>(p);
  }
  *out = g_scratch_address[dev];
  return cudaSuccess;
}
}  // namespace
}  // namespace mt

// No counterpart in the reference: mt_attention_decode without caller-provided scratch.
// Decode attention of one sequence with the attention output projection folded into its
// tail: out = attention (as mt_attention_decode), proj = bf16(W_o . out) with W_o [n_out,
// nq * 128] in the packed layout of mt_w4a16_pack (wo_zeros: blocks carry zero points). The
// o_proj is split over the KV heads: each 8-CTA cluster multiplies its head group's 512
// columns (the blocks fetched into shared memory before the dependency wait), and the
// partials are summed in KV-head order by the last CTA per row block. workspace:
// nkv * n_out * 4 + 64 bytes, zero-filled once (calls leave it reusable). Requires nq / nkv
// = 2 or 4, n_out % 128 == 0, and the tensor-core attention path (MT_ATTN_TC unset).
// Replaces the reference's attention + o_proj pair of FastLLM.hidden (llm.py:246-252).
MT_API int mt_attention_oproj_decode(const void* qkv, const void* q_norm, const void* k_norm, const void* cos_tab,
                                     const void* sin_tab, const void* positions, void* k_cache, void* v_cache,
                                     void* out, const void* wo_packed, int wo_zeros, void* proj, int n_out,
                                     void* workspace, int nq, int nkv, int max_len, float eps, void* status,
                                     int flags, void* stream) {
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.qkv = (const __nv_bfloat16*)qkv;
  a.q_norm = (const __nv_bfloat16*)q_norm;
  a.k_norm = (const __nv_bfloat16*)k_norm;
  a.cos_tab = (const __nv_bfloat16*)cos_tab;
  a.sin_tab = (const __nv_bfloat16*)sin_tab;
  a.positions = (const int64_t*)positions;
  a.k_cache = (__nv_bfloat16*)k_cache;
  a.v_cache = (__nv_bfloat16*)v_cache;
  a.out = (__nv_bfloat16*)out;
  a.nq = nq;
  a.nkv = nkv;
  a.max_len = max_len;
  a.splits = 1;
  a.eps = eps;
  a.status = (int*)status;
  a.wo = (const uint8_t*)wo_packed;
  a.wo_zeros = wo_zeros ? 1 : 0;
  a.n_out = n_out;
  a.opart = (float*)workspace;
  a.otickets = (unsigned*)((uint8_t*)workspace + (size_t)nkv * n_out * sizeof(float));
  a.oout = (__nv_bfloat16*)proj;
  if (attn_check(a, 1) || !out || !wo_packed || !proj || !workspace || n_out < 128 || n_out % 128 ||
      n_out > (1 << 20) || !aligned(wo_packed, 16) || !aligned(workspace, 16))
    return kBadArgument;
  const int rep = nq / nkv;
  if ((rep != 4 && rep != 2) || !attention_tc()) return kBadArgument;
  cudaStream_t s = (cudaStream_t)stream;
  return (int)(rep == 4 ? launch_attention_oproj<4>(a, s, flags & kFlagPdl) : launch_attention_oproj<2>(a, s, flags & kFlagPdl));
}

MT_API int mt_attention_decode_noalloc(const void* qkv, const void* q_norm, const void* k_norm,
                                       const void* cos_tab, const void* sin_tab, const void* positions,
                                       void* k_cache, void* v_cache, void* out, int batch, int nq, int nkv,
                                       int max_len, int splits, float eps, void* status, int flags,
                                       void* stream) {
  if (batch < 1 || nkv < 1 || nq < nkv || nq % nkv || splits < 1 || splits > 1024) return kBadArgument;
  const int rep = nq / nkv;
  if (rep != 4 && rep != 1 && rep != 2) return kBadArgument;
  const size_t slots = (size_t)batch * nkv * splits * rep;
  if (slots * kHeadDim > kNoAllocPartial || slots > kNoAllocLse || (size_t)batch * nkv > kNoAllocTickets)
    return (int)cudaErrorMemoryAllocation;  // request exceeds the fixed scratch
  AttnArgs a;
  a.qkv = (const __nv_bfloat16*)qkv;
  a.q_norm = (const __nv_bfloat16*)q_norm;
  a.k_norm = (const __nv_bfloat16*)k_norm;
  a.cos_tab = (const __nv_bfloat16*)cos_tab;
  a.sin_tab = (const __nv_bfloat16*)sin_tab;
  a.positions = (const int64_t*)positions;
  a.k_cache = (__nv_bfloat16*)k_cache;
  a.v_cache = (__nv_bfloat16*)v_cache;
  a.out = (__nv_bfloat16*)out;
  a.nq = nq;
  a.nkv = nkv;
  a.max_len = max_len;
  a.splits = splits;
  a.eps = eps;
  a.status = (int*)status;
  if (attn_check(a, batch) || !out) return kBadArgument;
  const size_t smem = attn_smem_bytes(rep, max_len, splits);
  if (smem > 200 * 1024) return kBadArgument;
  NoAllocScratch* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return (int)e;
  a.partial = scratch->partial;
  a.lse = scratch->lse;
  a.tickets = scratch->tickets;
  cudaStream_t s = (cudaStream_t)stream;
  // The merge counters must start at zero; clear them on the stream so each call is
  // independent of whatever an earlier (possibly failed) call left behind.
  e = cudaMemsetAsync(scratch->tickets, 0, (size_t)batch * nkv * sizeof(unsigned), s);
  if (e != cudaSuccess) return (int)e;
  const dim3 grid(nkv, splits, batch);
  switch (rep) {
    case 4: return launch(attention_decode<4>, grid, dim3(128), smem, s, flags, a);
    case 2: return launch(attention_decode<2>, grid, dim3(128), smem, s, flags, a);
    default: return launch(attention_decode<1>, grid, dim3(128), smem, s, flags, a);
  }
}
