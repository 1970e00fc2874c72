// The batch-1 decode step's whole layer stack as ONE persistent kernel (sm_100a).
//
// What it replaces: the per-layer launch chain of the decode step -- W4A16 RMSNorm + q|k|v,
// fused QK-norm/RoPE/KV write + attention, o_proj, add + RMSNorm + gate/up + SiLU, down --
// i.e. the body of the reference's FastLLM.hidden (src/moss_tts/_runtime/llm.py:227-260) and
// qkv_cluster_model.Hidden (qkv_cluster_model.py:50-72), which launches seven kernels per layer.
//
// Why one kernel: a batch-1 step streams ~4.4 GB of weights, and a per-layer chain of
// launches pays, at every one of its 180 edges, the wait for the previous grid's slowest CTA
// and an activation prologue during which HBM sits idle. Here the weight stream never
// stops: the weights do not depend on the activations, so each CTA's producer warp streams
// its whole schedule -- every layer's projection blocks and its slice of the KV cache -- into
// a 4-stage shared-memory ring (142 KB per SM, ~21 MB in flight over the GPU), while the 15
// consumer warps step through the phases and meet the other CTAs at grid barriers. A barrier
// or an attention chain then costs consumer time only; the ring keeps filling meanwhile.
//
// Grid: one CTA per SM (148 on B200), all co-resident (one CTA fills an SM's shared memory).
// Phases of layer L, each ended by a grid barrier (arrive after the phase, wait before the
// next one; the waits are bounded by a deadline and an abort flag):
//   QKV   x = RMSNorm(bf16(res + bf16(down of L-1)))  (layer 0: RMSNorm(embedding)),
//         q|k|v (6144 rows) split-K over the CTAs; each CTA adds its row sums into fp32
//         accumulators with red.add. A row gets at most two contributions (every CTA range
//         spans at least one whole tile), and fp32 addition of two terms onto zero is
//         commutative, so the sums are deterministic.
//   ATTN  CTA (kv head h, split s) for s < SPL = SMs / 8: QK-norm + RoPE of q/k from the
//         accumulators, the owner of `position` writes the new K/V rows, online softmax over
//         its tokens (streamed by the producer in 64-token chunks), unnormalised partials to
//         global scratch; the last split of a head to finish (ticket) merges by log-sum-exp
//         into the bf16 attention output.
//   OUT   o_proj (4096 rows, K 4096) split-K into fp32 accumulators.
//   GU    x = RMSNorm(bf16(res + bf16(o))); gate/up pair (tiles of 8 gate + 8 up rows) on
//         whole tiles per CTA, SiLU(gate) * up finished in the CTA -> bf16 `mid`.
//   DOWN  down (4096 rows, K = intermediate) split-K into fp32 accumulators.
// After the last layer the last CTA to finish (ticket) writes bf16(down) for the heads kernel,
// zeroes the first layer's accumulators for the next call and resets the barrier counters.
// Accumulators of layer L + 1 are zeroed by every CTA during layer L (before first use).
//
// Numerics: the same slice-block dequantise-and-dot (w4_tiles.cuh), activation scaling and
// rounding points as mt_w4a16_linear_packed; bf16 outputs are bf16(fp32 row sum) as there.
#include <stdlib.h>

#include "w4_tiles.cuh"

namespace mt {

__device__ int g_persist_error;  // 1: a bounded copy wait expired; 3: a grid barrier expired

namespace persist {

using namespace pipe;

// 15 consumer warps + 1 producer warp: 16 warps may hold 128 registers each (warps get
// registers in groups of four, so a 17th warp would cap every warp at 96 and spill)
constexpr int kCW = 15;                     // consumer warps
constexpr int kNS = 4;                      // ring stages
constexpr int kSB = kCW;                    // slice blocks per stage: one per consumer warp
constexpr int kConsumers = kCW * 32;        // 480 consumer threads
constexpr int kTG = kConsumers / 64;        // P.V token groups of 64 dim-pair threads (7)
constexpr int kHeadDim = 128, kRep = 4, kNq = 32, kNkv = 8, kHidden = 4096, kQkvRows = 6144;
constexpr int kChunk = 64;                  // attention tokens per stage (K and V rows: 32 KB)
constexpr int kAccPerLayer = kQkvRows + 2 * kHidden;  // q|k|v, o, down fp32 accumulators
constexpr int kOffO = kQkvRows, kOffDown = kQkvRows + kHidden;
constexpr float kAttnScale = 0.08838834764831845f;  // 1/sqrt(128), kernels.py:183
constexpr unsigned long long kBarrierDeadlineNs = 500ull * 1000 * 1000;
enum { P_QKV = 0, P_ATTN = 1, P_OUT = 2, P_GU = 3, P_DOWN = 4, kPhases = 5 };

struct Args {
  const mt_decode_layer* layers;  // device table, one entry per layer
  int n_layers, inter, zeros, block_b, stage_b, max_tiles, spl, max_len;
  float eps;
  const __nv_bfloat16* x_in;      // layer-0 input (embedding sum) [4096]
  const int64_t* positions;       // [1]
  const __nv_bfloat16* cos_tab;   // [max_len, 128]
  const __nv_bfloat16* sin_tab;
  __nv_bfloat16* res_b;           // residual stream after each layer's attention add (caller's buffer)
  __nv_bfloat16* mlp_out;         // bf16(down) of the last layer
  int* status;
  unsigned* barrier;              // arrivals at grid barriers during this call (0 between calls)
  unsigned* done;                 // CTAs finished (0 between calls)
  unsigned* tickets;              // [8] attention merge counters (0 between phases)
  int* abort;                     // set when a CTA gives up a grid barrier
  float* acc;                     // [n_layers][kAccPerLayer]
  float* att_o;                   // [8][spl][kRep][128] unnormalised partial outputs
  float* att_m;                   // [8][spl][kRep] running max
  float* att_l;                   // [8][spl][kRep] running sum
  __nv_bfloat16* attn;            // [4096]
  __nv_bfloat16* mid;             // [inter]
  __nv_bfloat16* res_a;           // [4096] residual stream before each layer's attention add
};

struct Range {
  const uint8_t* w;
  int b0, b1, S, n_out;
};

// Blocks of projection `p` that CTA c of G streams: split-K (even block counts) for q|k|v,
// o_proj and down; whole tiles for the gate/up pair, whose SiLU needs complete rows.
__device__ __forceinline__ Range phase_range(const Args& a, const mt_decode_layer& ly, int p, int c, int G) {
  Range r;
  r.S = kHidden / kSliceCols;
  if (p == P_QKV) {
    r.w = (const uint8_t*)ly.qkv;
    r.n_out = kQkvRows;
  } else if (p == P_OUT) {
    r.w = (const uint8_t*)ly.out;
    r.n_out = kHidden;
  } else if (p == P_GU) {
    r.w = (const uint8_t*)ly.gate_up;
    r.n_out = a.inter;
    const int T = a.inter / 8;
    r.b0 = (int)((long long)c * T / G) * r.S;
    r.b1 = (int)((long long)(c + 1) * T / G) * r.S;
    return r;
  } else {
    r.w = (const uint8_t*)ly.down;
    r.n_out = kHidden;
    r.S = a.inter / kSliceCols;
  }
  const long long nb = (long long)(r.n_out / 16) * r.S;
  r.b0 = (int)((long long)c * nb / G);
  r.b1 = (int)((long long)(c + 1) * nb / G);
  return r;
}

struct Item {
  int has, h, s, t0, t1, chunks;
};

__device__ __forceinline__ Item attn_item(int c, int spl, int len) {
  Item it = {};
  if (c >= kNkv * spl) return it;
  it.has = 1;
  it.h = c / spl;
  it.s = c - it.h * spl;
  const int span = (len + spl - 1) / spl;
  it.t0 = it.s * span;
  it.t1 = min(it.t0 + span, len);
  const int n = it.t1 > it.t0 ? it.t1 - it.t0 : 0;
  it.chunks = (n + kChunk - 1) / kChunk;
  return it;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__device__ __forceinline__ int clamp_position(const Args& a, bool* bad) {
  int64_t pos = a.positions[0];
  *bad = pos < 0 || pos >= a.max_len;
  if (*bad) pos = pos < 0 ? 0 : a.max_len - 1;
  return (int)pos;
}

// Producer (one lane): the CTA's whole weight / KV schedule into the ring, in consumer order.
__device__ void producer(const Args& a, uint8_t* ring, uint64_t* full, uint64_t* empty, volatile int* cta_abort) {
  const int G = gridDim.x, c = blockIdx.x;
  long g = 0;
  bool waited = false, ok = true;
  int len = -1;
  auto acquire = [&](long gg) -> bool {  // the ring slot of stage gg is free again
    if (gg < kNS) return true;
    uint64_t* bar = &empty[gg % kNS];
    const unsigned parity = (unsigned)(((gg / kNS) - 1) & 1);
    unsigned long long t0 = globaltimer_ns();
    for (long i = 0; i < kSpinLimit; ++i) {
      if (mbar_try_wait_sleep(bar, parity, 2000)) return true;  // sleeps instead of spinning
      if (*cta_abort || globaltimer_ns() - t0 > kWaitDeadlineNs) return false;
    }
    return false;
  };
  for (int L = 0; L < a.n_layers && ok; ++L) {
    const mt_decode_layer& ly = a.layers[L];
    for (int p = 0; p < kPhases && ok; ++p) {
      if (p == P_ATTN) {
        // cache rows of earlier steps (and the position) come from earlier kernels
        if (!waited) { pdl_wait(); waited = true; }
        if (len < 0) {
          bool bad;
          len = clamp_position(a, &bad) + 1;
        }
        const Item it = attn_item(c, a.spl, len);
        for (int ch = 0; ch < it.chunks; ++ch) {
          if (!acquire(g)) { ok = false; break; }
          const int ts = it.t0 + ch * kChunk, rows = min(kChunk, it.t1 - ts);
          const unsigned bytes = (unsigned)rows * kHeadDim * 2;
          uint8_t* dst = ring + (size_t)(g % kNS) * a.stage_b;
          const size_t off = ((size_t)it.h * a.max_len + ts) * kHeadDim;
          mbar_expect_tx(&full[g % kNS], 2 * bytes);
          bulk_copy(dst, (const __nv_bfloat16*)ly.k_cache + off, bytes, &full[g % kNS]);
          bulk_copy(dst + kChunk * kHeadDim * 2, (const __nv_bfloat16*)ly.v_cache + off, bytes, &full[g % kNS]);
          ++g;
        }
      } else {
        const Range r = phase_range(a, ly, p, c, G);
        const int nblk = r.b1 - r.b0, stages = (nblk + kSB - 1) / kSB;
        for (int st = 0; st < stages; ++st) {
          // weights never depend on earlier kernels: the first kNS stages go out before the wait
          if (g >= kNS && !waited) { pdl_wait(); waited = true; }
          if (!acquire(g)) { ok = false; break; }
          const int nb = min(kSB, nblk - st * kSB);
          mbar_expect_tx(&full[g % kNS], (unsigned)(nb * a.block_b));
          bulk_copy(ring + (size_t)(g % kNS) * a.stage_b, r.w + (size_t)(r.b0 + st * kSB) * a.block_b,
                    (unsigned)(nb * a.block_b), &full[g % kNS]);
          ++g;
        }
      }
    }
  }
  if (!ok) {  // the consumers stopped: wait (bounded) for the copies still in flight, then leave
    if (!*cta_abort) atomicExch(&g_persist_error, 1);
    for (long d = g - kNS; d < g; ++d)
      if (d >= 0) mbar_wait_bounded(&full[d % kNS], (unsigned)((d / kNS) & 1));
  }
}

// Attention phase of one layer for this CTA. Reads the arguments from their shared-memory copy;
// reports a copy-wait failure through *sm.fail_flag, uniformly per CTA.
struct AttnSmem {
  uint8_t* ring;
  uint64_t* full;
  uint64_t* empty;
  uint4* xp;
  float* qs;
  float (*pr)[kRep];
  float* m_run;
  float* l_run;
  float* scl;
  volatile int* fail_flag;
  int* bcast;
};

__device__ __forceinline__ void attention_phase(const Args* a, const mt_decode_layer* ly, const float* acc_l, int pos,
                                             int len, long* g_io, const AttnSmem* smp) {
  const int c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const AttnSmem sm = *smp;
  uint8_t* ring = sm.ring;
  uint64_t* full = sm.full;
  uint64_t* empty = sm.empty;
  uint4* xp = sm.xp;
  float* qs = sm.qs;
  float (*pr)[kRep] = sm.pr;
  float* m_run = sm.m_run;
  float* l_run = sm.l_run;
  float* scl = sm.scl;
  volatile int& fail_flag = *sm.fail_flag;
  int& bcast = *sm.bcast;
  long g = *g_io;
        const Item it = attn_item(c, a->spl, len);
        if (it.has) {
          const int h = it.h;
          const bool owner = it.t0 <= pos && pos < it.t1;
          uint2 krow = make_uint2(0, 0), vrow = make_uint2(0, 0);
          const bool rotates = warp < kRep || (warp == kRep && owner);
          if (rotates) {
            // head RMSNorm + rotate-half RoPE (kernels.py:158-163) of the q|k|v projection
            // output, bf16(fp32 row sum); q kept as bf16-exact fp32
            const int row = warp < kRep ? h * kRep + warp : kNq + h;
            const float4 av = __ldcg(reinterpret_cast<const float4*>(acc_l + row * kHeadDim) + lane);
            float x[4] = {round_bf16(av.x), round_bf16(av.y), round_bf16(av.z), round_bf16(av.w)};
            const uint2 nw = *reinterpret_cast<const uint2*>(
                (const __nv_bfloat16*)(warp < kRep ? ly->q_norm : ly->k_norm) + 4 * lane);
            const uint2 cw = *reinterpret_cast<const uint2*>(a->cos_tab + (size_t)pos * kHeadDim + 4 * lane);
            const uint2 sw = *reinterpret_cast<const uint2*>(a->sin_tab + (size_t)pos * kHeadDim + 4 * lane);
            const float wv[4] = {bf16_lo(nw.x), bf16_hi(nw.x), bf16_lo(nw.y), bf16_hi(nw.y)};
            const float cv[4] = {bf16_lo(cw.x), bf16_hi(cw.x), bf16_lo(cw.y), bf16_hi(cw.y)};
            const float sv[4] = {bf16_lo(sw.x), bf16_hi(sw.x), bf16_lo(sw.y), bf16_hi(sw.y)};
            float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
            ss = warp_sum(ss);
            const float inv = 1.0f / sqrtf(ss / 128.f + a->eps);
            float y[4], part[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) y[i] = round_bf16(round_bf16(x[i] * inv) * wv[i]);
#pragma unroll
            for (int i = 0; i < 4; ++i) part[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);  // partner d +- 64
            const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = round_bf16(round_bf16(y[i] * cv[i]) + round_bf16(sign * part[i] * sv[i]));
            if (warp < kRep) {
              *reinterpret_cast<float4*>(&qs[(warp * 4 + (lane >> 3)) * 36 + 4 * (lane & 7)]) =
                  make_float4(x[0], x[1], x[2], x[3]);
            } else {
              __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
              krow.x = *reinterpret_cast<uint32_t*>(&lo);
              krow.y = *reinterpret_cast<uint32_t*>(&hi);
              const float4 vv = __ldcg(reinterpret_cast<const float4*>(acc_l + (kNq + kNkv + h) * kHeadDim) + lane);
              __nv_bfloat162 vlo = __floats2bfloat162_rn(vv.x, vv.y), vhi = __floats2bfloat162_rn(vv.z, vv.w);
              vrow.x = *reinterpret_cast<uint32_t*>(&vlo);
              vrow.y = *reinterpret_cast<uint32_t*>(&vhi);
              const size_t cell = ((size_t)h * a->max_len + pos) * kHeadDim + 4 * lane;
              *reinterpret_cast<uint2*>((__nv_bfloat16*)ly->k_cache + cell) = krow;
              *reinterpret_cast<uint2*>((__nv_bfloat16*)ly->v_cache + cell) = vrow;
            }
          }
          if (tid < kRep) { m_run[tid] = -INFINITY; l_run[tid] = 0.f; }
          const int dp = tid & 63, tg = tid >> 6;  // P.V: dim pair, token group (tg < kTG take part)
          float accv[kRep][2];
#pragma unroll
          for (int hh = 0; hh < kRep; ++hh) accv[hh][0] = accv[hh][1] = 0.f;
          for (int ch = 0; ch < it.chunks; ++ch) {
            // every thread waits (bounded) for the chunk; a failure anywhere stops the whole CTA
            // at the same chunk, so no thread skips a named barrier the others wait on
            if (!mbar_wait_bounded(&full[g % kNS], (unsigned)((g / kNS) & 1))) fail_flag = 1;
            named_sync(1, kConsumers);  // q / m_run ready; every thread is past the previous chunk's pr
            if (fail_flag) break;
            const int slot = (int)(g % kNS), cs = it.t0 + ch * kChunk, rows = min(kChunk, it.t1 - cs);
            __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(ring + (size_t)slot * a->stage_b);
            __nv_bfloat16* vs = ks + kChunk * kHeadDim;
            if (owner && pos >= cs && pos < cs + rows) {  // this chunk holds this step's row
              if (warp == kRep) {
                *reinterpret_cast<uint2*>(ks + (size_t)(pos - cs) * kHeadDim + 4 * lane) = krow;
                *reinterpret_cast<uint2*>(vs + (size_t)(pos - cs) * kHeadDim + 4 * lane) = vrow;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before the slot is refilled
              }
              named_sync(1, kConsumers);
            }
            // logits: item ((t * kRep) + h) * 4 + quarter; four lanes share (t, h)
            const int items = rows * kRep * 4;
            for (int base = 0; base < items; base += kConsumers) {
              const int item = base + tid;
              const int qt = item & 3, hh = (item >> 2) % kRep, t = (item >> 2) / kRep;
              float d0 = 0.f, d1 = 0.f;
              if (item < items) {
                const uint4* k4 = reinterpret_cast<const uint4*>(ks + (size_t)t * kHeadDim + qt * 32);
                const float4* q4 = reinterpret_cast<const float4*>(&qs[(hh * 4 + qt) * 36]);
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                  const int j = (jj + qt) & 3;
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
              if (item < items && qt == 0) pr[t][hh] = v * kAttnScale;
            }
            named_sync(1, kConsumers);
            if (warp < kRep) {  // online softmax, warp hh owns query head hh
              const int hh = warp;
              float m = -INFINITY;
              for (int t = lane; t < rows; t += 32) m = fmaxf(m, pr[t][hh]);
              m = warp_max(m);
              const float mnew = fmaxf(m_run[hh], m);
              float s = 0.f;
              for (int t = lane; t < rows; t += 32) {
                const float e = expf(pr[t][hh] - mnew);
                pr[t][hh] = e;
                s += e;
              }
              s = warp_sum(s);
              if (lane == 0) {
                const float sc = expf(m_run[hh] - mnew);
                scl[hh] = sc;
                l_run[hh] = l_run[hh] * sc + s;
                m_run[hh] = mnew;
              }
            }
            named_sync(1, kConsumers);
            {
              float sc[kRep];
#pragma unroll
              for (int hh = 0; hh < kRep; ++hh) sc[hh] = scl[hh];
#pragma unroll
              for (int hh = 0; hh < kRep; ++hh) { accv[hh][0] *= sc[hh]; accv[hh][1] *= sc[hh]; }
              const uint32_t* v2 = reinterpret_cast<const uint32_t*>(vs) + dp;
#pragma unroll 4
              for (int t = tg; tg < kTG && t < rows; t += kTG) {
                const uint32_t vv = v2[(size_t)t * (kHeadDim / 2)];
                const float va = bf16_lo(vv), vb = bf16_hi(vv);
#pragma unroll
                for (int hh = 0; hh < kRep; ++hh) {
                  const float ph = pr[t][hh];
                  accv[hh][0] = fmaf(ph, va, accv[hh][0]);
                  accv[hh][1] = fmaf(ph, vb, accv[hh][1]);
                }
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            ++g;
          }
          if (!fail_flag) {
            // token groups -> one unnormalised partial per (query head, dim) of this split
            float* redv = reinterpret_cast<float*>(xp);  // [kTG token groups][kRep][128]
            if (tg < kTG) {
#pragma unroll
              for (int hh = 0; hh < kRep; ++hh)
                *reinterpret_cast<float2*>(&redv[(tg * kRep + hh) * kHeadDim + 2 * dp]) =
                    make_float2(accv[hh][0], accv[hh][1]);
            }
            named_sync(1, kConsumers);
            for (int item = tid; item < kRep * kHeadDim; item += kConsumers) {
              const int hh = item >> 7, d = item & (kHeadDim - 1);
              float o = 0.f;
#pragma unroll
              for (int q = 0; q < kTG; ++q) o += redv[(q * kRep + hh) * kHeadDim + d];
              const size_t cell = ((size_t)h * a->spl + it.s) * kRep + hh;
              a->att_o[cell * kHeadDim + d] = o;
              if (d == 0) {
                a->att_m[cell] = m_run[hh];
                a->att_l[cell] = l_run[hh];
              }
            }
            named_sync(1, kConsumers);
            // the last split of this KV head to report merges all of them (kernels.py:198-208)
            if (tid == 0) {
              __threadfence();
              bcast = atomicAdd(a->tickets + h, 1u) == (unsigned)(a->spl - 1);
            }
            named_sync(1, kConsumers);
            if (bcast) {
              __threadfence();
              // the splits' statistics into shared memory (one parallel load), then per (head,
              // dim) the weighted sum of the partials, their loads issued in batches of 16
              const size_t base = (size_t)h * a->spl;
              float* st_m = redv + kTG * kRep * kHeadDim;  // [spl][kRep]
              float* st_w = st_m + a->spl * kRep;          // [spl][kRep]: exp(m_s - M), then / L
              for (int i = tid; i < a->spl * kRep; i += kConsumers) {
                st_m[i] = __ldcg(a->att_m + base * kRep + i);
                st_w[i] = __ldcg(a->att_l + base * kRep + i);
              }
              named_sync(1, kConsumers);
              if (tid < kRep) {
                float M = -INFINITY, lsum = 0.f;
                for (int s = 0; s < a->spl; ++s) M = fmaxf(M, st_m[s * kRep + tid]);
                for (int s = 0; s < a->spl; ++s) {
                  const float m = st_m[s * kRep + tid];
                  const float w = m == -INFINITY ? 0.f : expf(m - M);  // a split without tokens adds nothing
                  lsum = fmaf(w, st_w[s * kRep + tid], lsum);
                  st_m[s * kRep + tid] = w;
                }
                const float inv_l = lsum > 0.f ? 1.f / lsum : 0.f;
                for (int s = 0; s < a->spl; ++s) st_w[s * kRep + tid] = st_m[s * kRep + tid] * inv_l;
              }
              named_sync(1, kConsumers);
              for (int item = tid; item < kRep * kHeadDim; item += kConsumers) {
                const int hh = item >> 7, d = item & (kHeadDim - 1);
                float osum = 0.f;
                for (int s0 = 0; s0 < a->spl; s0 += 16) {
                  float ov[16];
#pragma unroll
                  for (int u = 0; u < 16; ++u)
                    ov[u] = s0 + u < a->spl ? __ldcg(a->att_o + ((base + s0 + u) * kRep + hh) * kHeadDim + d) : 0.f;
#pragma unroll
                  for (int u = 0; u < 16; ++u)
                    if (s0 + u < a->spl) osum = fmaf(st_w[(s0 + u) * kRep + hh], ov[u], osum);
                }
                a->attn[(h * kRep + hh) * kHeadDim + d] = to_bf16(osum);
              }
              if (tid == 0) a->tickets[h] = 0u;
            }
          }
        }
  *g_io = g;
}

__global__ void __launch_bounds__(kConsumers + 32, 1) decode_persistent(Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kNS];
  __shared__ __align__(8) uint64_t empty[kNS];
  __shared__ float red[kCW], redmax[kCW], redw[kCW];
  __shared__ __align__(16) uint4 zero16[4];
  __shared__ volatile int cta_abort;
  __shared__ volatile int fail_flag;  // set by any consumer thread whose bounded wait expired
  __shared__ int bcast;
  __shared__ __align__(16) float qs[kRep * 4 * 36];  // query heads, 32-dim quarters padded to 36
  __shared__ __align__(16) float pr[kChunk][kRep];   // logits, then probabilities
  __shared__ float m_run[kRep], l_run[kRep], scl[kRep];
  __shared__ Args a_sh;          // the arguments, addressable by the out-of-line attention phase
  __shared__ AttnSmem attn_sm;

  const int G = gridDim.x, c = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kmax = a.inter > kHidden ? a.inter : kHidden;
  const int xp_bytes = max(kmax / 8 * 16, (kRep * kTG * kHeadDim + 2 * kRep * a.spl) * 4);
  uint8_t* ring = smem;
  uint4* xp = reinterpret_cast<uint4*>(smem + (size_t)kNS * a.stage_b);  // [K / 8] fp16 pairs
  float* xsum = reinterpret_cast<float*>(smem + (size_t)kNS * a.stage_b + xp_bytes);  // [K / 32]
  float* partial = xsum + kmax / 32;  // [kCW][max_tiles][16]

  if (tid == kConsumers) {
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);
    }
    cta_abort = 0;
    fail_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid < 4) zero16[tid] = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    a_sh = a;
    attn_sm = AttnSmem{ring, full, empty, xp, qs, pr, m_run, l_run, scl, &fail_flag, &bcast};
  }
  __syncthreads();
  if (warp == kCW) {
    if (lane == 0) producer(a, ring, full, empty, &cta_abort);
    return;
  }

  // ------------------------------------------------------------------ consumers
  pdl_wait();
  pdl_trigger();
  bool bad_pos;
  const int pos = clamp_position(a, &bad_pos), len = pos + 1;
  if (bad_pos && c == 0 && tid == 0 && a.status) atomicExch(a.status, 1);
  const int r = lane >> 2, cq = lane & 3, hsel = r - 2 * cq;
  long g = 0;  // ring stages consumed
  unsigned bar_k = 0;
  bool ok = true;

  auto fail = [&](int code) {
    if (tid == 0) {
      atomicExch(&g_persist_error, code);
      atomicExch(a.abort, 1);
      cta_abort = 1;
    }
  };
  // grid barrier, split in arrive (after a phase) and wait (before the next)
  auto arrive = [&]() {
    named_sync(1, kConsumers);
    if (tid == 0) {
      __threadfence();
      atomicAdd(a.barrier, 1u);
    }
  };
  auto grid_wait = [&]() -> bool {
    ++bar_k;
    if (tid == 0) {
      const unsigned target = bar_k * (unsigned)G;
      const unsigned long long t0 = globaltimer_ns();
      int passed = 1;
      for (unsigned it = 0;; ++it) {
        if ((int)(ld_acquire_u32(a.barrier) - target) >= 0) break;
        if ((it & 63) == 63 && (*(volatile int*)a.abort || globaltimer_ns() - t0 > kBarrierDeadlineNs)) {
          passed = 0;
          break;
        }
      }
      __threadfence();
      bcast = passed;
    }
    named_sync(1, kConsumers);
    return bcast != 0;
  };
  auto wait_full = [&](long gg) -> bool {
    const bool got = mbar_wait_bounded(&full[gg % kNS], (unsigned)((gg / kNS) & 1));
    return __all_sync(0xffffffffu, got);
  };

  for (int L = 0; L < a.n_layers && ok; ++L) {
    const mt_decode_layer& ly = a.layers[L];
    float* acc_l = a.acc + (size_t)L * kAccPerLayer;
    for (int p = 0; p < kPhases && ok; ++p) {
      // ---- work that needs no other CTA: clear the row sums, zero the next layer's accumulators
      if (p != P_ATTN)
        for (int i = tid; i < kCW * a.max_tiles * 16; i += kConsumers) partial[i] = 0.f;
      if (p == P_OUT && L + 1 < a.n_layers) {
        float* nxt = a.acc + (size_t)(L + 1) * kAccPerLayer;
        const int z0 = (int)((long long)c * kAccPerLayer / G), z1 = (int)((long long)(c + 1) * kAccPerLayer / G);
        for (int i = z0 + tid; i < z1; i += kConsumers) nxt[i] = 0.f;
      }
      if (!(L == 0 && p == P_QKV) && !grid_wait()) {
        fail(3);
        ok = false;
        break;
      }

      if (p == P_ATTN) {
        // ============================================================ attention
        attention_phase(&a_sh, a.layers + L, acc_l, pos, len, &g, &attn_sm);
        named_sync(1, kConsumers);
        if (fail_flag) {
          fail(1);
          ok = false;
          break;
        }
        arrive();
        continue;
      }

      // ============================================================== projections
      const Range rg = phase_range(a, ly, p, c, G);
      const int K = p == P_DOWN ? a.inter : kHidden;
      const int S = rg.S, nblk = rg.b1 - rg.b0, stages = (nblk + kSB - 1) / kSB;
      const int t_first = rg.b0 / S, t_last = (rg.b1 - 1) / S, ntiles = t_last - t_first + 1;
      const bool norm = p == P_QKV || p == P_GU;
      const __nv_bfloat16* norm_w = (const __nv_bfloat16*)(p == P_QKV ? ly.input_norm : ly.post_norm);
      // ---- activation prologue: thread t owns the 8-value words t, t + 512, t + 1024. Pass 1
      // forms the bf16 input (with the residual add) into xp and the block statistics; pass 2
      // reads its own words back, applies the norm and writes the fp16 operand pairs in place.
      const int words = K / 8;
      float ss = 0.f, mv = 0.f, mw = 0.f;
      for (int word = tid; word < words; word += kConsumers) {
        uint4 xw;
        if (p == P_OUT) {
          xw = __ldcg(reinterpret_cast<const uint4*>(a.attn) + word);
        } else if (p == P_DOWN) {
          xw = __ldcg(reinterpret_cast<const uint4*>(a.mid) + word);
        } else if (p == P_QKV && L == 0) {
          xw = __ldcg(reinterpret_cast<const uint4*>(a.x_in) + word);
        } else {
          // bf16(residual + bf16(projection row sum)), the reference's add_rmsnorm sum
          const uint4 rw = __ldcg(reinterpret_cast<const uint4*>(p == P_QKV ? a.res_b : a.res_a) + word);
          const float* src = p == P_QKV ? a.acc + (size_t)(L - 1) * kAccPerLayer + kOffDown : acc_l + kOffO;
          const float4 f0 = __ldcg(reinterpret_cast<const float4*>(src) + 2 * word);
          const float4 f1 = __ldcg(reinterpret_cast<const float4*>(src) + 2 * word + 1);
          const float fv[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
          const uint32_t ra[4] = {rw.x, rw.y, rw.z, rw.w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float lo = round_bf16(round_bf16(fv[2 * i]) + bf16_lo(ra[i]));
            const float hi = round_bf16(round_bf16(fv[2 * i + 1]) + bf16_hi(ra[i]));
            __nv_bfloat162 pr2 = __floats2bfloat162_rn(lo, hi);
            o[i] = *reinterpret_cast<uint32_t*>(&pr2);
          }
          xw = make_uint4(o[0], o[1], o[2], o[3]);
        }
        if (norm && c == 0)  // the residual stream after this add, for the later phases
          reinterpret_cast<uint4*>(p == P_QKV ? a.res_a : a.res_b)[word] = xw;
        xp[word] = xw;
        const uint32_t xa[4] = {xw.x, xw.y, xw.z, xw.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float lo = bf16_lo(xa[i]), hi = bf16_hi(xa[i]);
          mv = fmaxf(mv, fmaxf(fabsf(lo), fabsf(hi)));
          ss += lo * lo + hi * hi;
        }
        if (norm) {
          const uint4 nw = reinterpret_cast<const uint4*>(norm_w)[word];
          const uint32_t na[4] = {nw.x, nw.y, nw.z, nw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) mw = fmaxf(mw, fmaxf(fabsf(bf16_lo(na[i])), fabsf(bf16_hi(na[i]))));
        }
      }
      ss = warp_sum(ss);
      mv = warp_max(mv);
      mw = warp_max(mw);
      if (lane == 0) { red[warp] = ss; redmax[warp] = mv; redw[warp] = mw; }
      named_sync(1, kConsumers);
      float tot = 0.f, mx = 0.f, mxw = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) {
        tot += red[w];
        mx = fmaxf(mx, redmax[w]);
        mxw = fmaxf(mxw, redw[w]);
      }
      const float inv = norm ? 1.0f / sqrtf(tot / (float)K + a.eps) : 1.f;
      if (norm) mx = mx * inv * mxw * 1.0079f;  // bound on |bf16(bf16(x inv) w)|
      // activation scale c = 2^(9 - e) (see w4a16_stream.cu)
      const int ex = mx > 0.f ? min(max((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127, -100), 100) : 0;
      const float cs = __uint_as_float((uint32_t)(127 + 9 - ex) << 23);
      const float inv_c = __uint_as_float((uint32_t)(127 + 24 - 9 + ex) << 23);
      for (int word = tid; word < words; word += kConsumers) {
        const uint4 xw = xp[word];
        const uint32_t xa[4] = {xw.x, xw.y, xw.z, xw.w};
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) { v[2 * i] = bf16_lo(xa[i]); v[2 * i + 1] = bf16_hi(xa[i]); }
        if (norm) {
          const uint4 nw = reinterpret_cast<const uint4*>(norm_w)[word];
          const uint32_t na[4] = {nw.x, nw.y, nw.z, nw.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[2 * i] = round_bf16(round_bf16(v[2 * i] * inv) * bf16_lo(na[i]));
            v[2 * i + 1] = round_bf16(round_bf16(v[2 * i + 1] * inv) * bf16_hi(na[i]));
          }
        }
        float wsum = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) wsum += v[i];
        xp[word] = make_uint4(pack_half2(v[0] * cs, v[4] * cs), pack_half2(v[1] * cs * 0.0625f, v[5] * cs * 0.0625f),
                              pack_half2(v[2] * cs, v[6] * cs), pack_half2(v[3] * cs * 0.0625f, v[7] * cs * 0.0625f));
        wsum += __shfl_xor_sync(0xffffffffu, wsum, 1);
        wsum += __shfl_xor_sync(0xffffffffu, wsum, 2);
        if ((lane & 3) == 0) xsum[word >> 2] = wsum * cs;
      }
      named_sync(1, kConsumers);

      // ---- the stages of this phase
      uint32_t bl[16], bh[16], bz0 = 0, bz1 = 0;
      int cur_j = -1;
      auto load_b = [&](int j) {
        const uint4* pl = hsel == 0 ? xp + j * 32 + 8 * cq : zero16;
        const uint4* ph = hsel == 1 ? xp + j * 32 + 8 * cq + 4 : zero16;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 ql = pl[u], qh = ph[u];
          bl[4 * u] = ql.x; bl[4 * u + 1] = ql.y; bl[4 * u + 2] = ql.z; bl[4 * u + 3] = ql.w;
          bh[4 * u] = qh.x; bh[4 * u + 1] = qh.y; bh[4 * u + 2] = qh.z; bh[4 * u + 3] = qh.w;
        }
        const float z0 = hsel == 0 ? -xsum[j * 8 + 2 * cq] : 0.f;
        const float z1 = hsel == 1 ? -xsum[j * 8 + 2 * cq + 1] * 0.0625f : 0.f;
        const float h0 = __half2float(__float2half_rn(z0)), h1 = __half2float(__float2half_rn(z1));
        bz0 = pack_half2(h0, h1);
        bz1 = pack_half2(z0 - h0, z1 - h1);
        cur_j = j;
      };
      int tt = (rg.b0 + warp) / S, jj = (rg.b0 + warp) - ((rg.b0 + warp) / S) * S;
      for (int st = 0; st < stages; ++st) {
        if (st > 0) {
          jj += kSB;
          while (jj >= S) {  // S >= kSB for every shape but the smallest: one subtraction
            jj -= S;
            ++tt;
          }
        }
        if (!wait_full(g)) {
          fail_flag = 1;
          break;
        }
        const int slot = (int)(g % kNS);
        const bool live = rg.b0 + st * kSB + warp < rg.b1;
        BlockRegs bk;
        if (live) bk = load_block(ring + (size_t)slot * a.stage_b + (size_t)warp * a.block_b, lane, a.zeros != 0);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (live) {
          if (jj != cur_j) load_b(jj);
          float va, vb;
          block_dot(bk, bl, bh, bz0, bz1, va, vb);
          if (cq == 0) {
            float* pp = partial + ((size_t)warp * a.max_tiles + (tt - t_first)) * 16;
            pp[r] += va;
            pp[r + 8] += vb;
          }
        }
        ++g;
      }
      named_sync(1, kConsumers);
      if (fail_flag) {
        fail(1);
        ok = false;
        break;
      }
      // ---- epilogue: the CTA's row sums
      if (p == P_GU) {
        for (int i = tid; i < ntiles * 8; i += kConsumers) {
          const int lt = i >> 3, tr = i & 7, o = (t_first + lt) * 8 + tr;
          float gsum = 0.f, usum = 0.f;
#pragma unroll 4
          for (int w = 0; w < kCW; ++w) {
            gsum += partial[((size_t)w * a.max_tiles + lt) * 16 + tr];
            usum += partial[((size_t)w * a.max_tiles + lt) * 16 + tr + 8];
          }
          if (o < a.inter) a.mid[o] = to_bf16(finish_row<true>(gsum * inv_c, usum * inv_c));
        }
      } else {
        float* dst = acc_l + (p == P_QKV ? 0 : p == P_OUT ? kOffO : kOffDown);
        for (int i = tid; i < ntiles * 16; i += kConsumers) {
          const int lt = i >> 4, tr = i & 15, o = (t_first + lt) * 16 + tr;
          float sum = 0.f;
#pragma unroll 4
          for (int w = 0; w < kCW; ++w) sum += partial[((size_t)w * a.max_tiles + lt) * 16 + tr];
          if (o < rg.n_out) red_add_f32(dst + o, sum * inv_c);
        }
      }
      if (!(L == a.n_layers - 1 && p == P_DOWN)) arrive();
    }
  }
  if (!ok) return;
  // ---- the last CTA to finish: bf16(down) of the last layer for the heads, reset for the next call
  named_sync(1, kConsumers);
  if (tid == 0) {
    __threadfence();
    bcast = atomicAdd(a.done, 1u) == (unsigned)G - 1u;
  }
  named_sync(1, kConsumers);
  if (!bcast) return;
  __threadfence();
  const float* last = a.acc + (size_t)(a.n_layers - 1) * kAccPerLayer + kOffDown;
  for (int i = tid; i < kHidden; i += kConsumers) a.mlp_out[i] = to_bf16(__ldcg(last + i));
  named_sync(1, kConsumers);
  for (int i = tid; i < kAccPerLayer; i += kConsumers) a.acc[i] = 0.f;
  named_sync(1, kConsumers);
  if (tid == 0) {
    *a.barrier = 0u;
    *a.done = 0u;
    __threadfence();
  }
}

}  // namespace persist
}  // namespace mt

namespace mt {
namespace persist {

// Workspace carve-up (every piece 256-byte aligned). Counters first, each on its own line.
struct WsLayout {
  size_t barrier = 0, done = 128, tickets = 256, abort = 512, acc, att_o, att_m, att_l, attn, mid, res_a, total;
  WsLayout(int n_layers, int inter, int spl) {
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    acc = 1024;
    att_o = up(acc + (size_t)n_layers * kAccPerLayer * 4);
    att_m = up(att_o + (size_t)kNkv * spl * kRep * kHeadDim * 4);
    att_l = up(att_m + (size_t)kNkv * spl * kRep * 4);
    attn = up(att_l + (size_t)kNkv * spl * kRep * 4);
    mid = up(attn + (size_t)kHidden * 2);
    res_a = up(mid + (size_t)inter * 2);
    total = up(res_a + (size_t)kHidden * 2);
  }
};

static int max_tiles_for(int inter, int G) {
  // split-K phases: a range of ceil(NB / G) blocks touches at most ceil(blocks / S) + 1 tiles;
  // gate/up: whole tiles, ceil(T / G)
  auto split = [&](int n_out, int S) {
    const long long nb = (long long)(n_out / 16) * S;
    const long long per = (nb + G - 1) / G;
    return (int)((per + S - 1) / S) + 1;
  };
  int m = split(kQkvRows, 16);
  m = max(m, split(kHidden, 16));
  m = max(m, split(kHidden, inter / kSliceCols));
  m = max(m, (inter / 8 + G - 1) / G);
  return m;
}

static size_t smem_bytes(int inter, int zeros, int max_tiles, int spl) {
  const int block_b = kCodeBytes + kScaleBytes + (zeros ? kZeroBytes : 0);
  const int kmax = inter > kHidden ? inter : kHidden;
  const int xp_bytes = max(kmax / 8 * 16, (kRep * kTG * kHeadDim + 2 * kRep * spl) * 4);
  return (size_t)kNS * kSB * block_b + xp_bytes + (size_t)kmax / 32 * 4 + (size_t)kCW * max_tiles * 16 * 4;
}

static bool shape_ok(int n_layers, int inter) {
  return n_layers >= 1 && n_layers <= 1024 && inter >= 256 && inter <= 16384 && inter % 256 == 0;
}

}  // namespace persist

cudaError_t persist_error_word(int* value, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_persist_error, sizeof(int));
  if (e != cudaSuccess) return e;
  if (v && !*value) *value = v;
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_persist_error, &zero, sizeof(int));
  }
  return e;
}

}  // namespace mt

using namespace mt;
using namespace mt::persist;

MT_API int mt_decode_layers_workspace(int n_layers, int inter, long long* bytes) {
  if (!bytes || !shape_ok(n_layers, inter)) return kBadArgument;
  const int G = sm_count();
  if (G < kNkv) return kBadArgument;
  *bytes = (long long)WsLayout(n_layers, inter, G / kNkv).total;
  return 0;
}

MT_API int mt_decode_layers(const void* layers, int n_layers, int inter, int has_zeros, const void* x,
                            const void* positions, const void* cos_tab, const void* sin_tab, int max_len, float eps,
                            void* residual, void* mlp_out, void* workspace, void* status, int flags, void* stream) {
  if (!layers || !x || !positions || !cos_tab || !sin_tab || !residual || !mlp_out || !workspace ||
      !shape_ok(n_layers, inter) || max_len < 1)
    return kBadArgument;
  if (!aligned(layers, 16) || !aligned(x, 16) || !aligned(positions, 8) || !aligned(cos_tab, 16) ||
      !aligned(sin_tab, 16) || !aligned(residual, 16) || !aligned(mlp_out, 16) || !aligned(workspace, 256))
    return kBadArgument;
  const int G = sm_count();
  // every split-K range must hold a whole tile (at most two contributions per row): 256 tiles
  if (G < kNkv || G > kHidden / 16) return kBadArgument;
  const WsLayout ws(n_layers, inter, G / kNkv);
  uint8_t* base = (uint8_t*)workspace;
  Args a = {};
  a.layers = (const mt_decode_layer*)layers;
  a.n_layers = n_layers;
  a.inter = inter;
  a.zeros = has_zeros ? 1 : 0;
  a.block_b = kCodeBytes + kScaleBytes + (has_zeros ? kZeroBytes : 0);
  a.stage_b = kSB * a.block_b;
  a.max_tiles = max_tiles_for(inter, G);
  a.spl = G / kNkv;
  a.max_len = max_len;
  a.eps = eps;
  a.x_in = (const __nv_bfloat16*)x;
  a.positions = (const int64_t*)positions;
  a.cos_tab = (const __nv_bfloat16*)cos_tab;
  a.sin_tab = (const __nv_bfloat16*)sin_tab;
  a.res_b = (__nv_bfloat16*)residual;
  a.mlp_out = (__nv_bfloat16*)mlp_out;
  a.status = (int*)status;
  a.barrier = (unsigned*)(base + ws.barrier);
  a.done = (unsigned*)(base + ws.done);
  a.tickets = (unsigned*)(base + ws.tickets);
  a.abort = (int*)(base + ws.abort);
  a.acc = (float*)(base + ws.acc);
  a.att_o = (float*)(base + ws.att_o);
  a.att_m = (float*)(base + ws.att_m);
  a.att_l = (float*)(base + ws.att_l);
  a.attn = (__nv_bfloat16*)(base + ws.attn);
  a.mid = (__nv_bfloat16*)(base + ws.mid);
  a.res_a = (__nv_bfloat16*)(base + ws.res_a);
  // a 64-token K + V chunk must fit one ring stage
  if (2 * kChunk * kHeadDim * 2 > a.stage_b) return kBadArgument;
  const size_t smem = smem_bytes(inter, a.zeros, a.max_tiles, a.spl);
  if (smem > 227 * 1024) return kBadArgument;
  cudaError_t e = cudaFuncSetAttribute(decode_persistent, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  // every CTA must be resident at once (grid barriers): one CTA per SM and a grid of SMs
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_persistent, kConsumers + 32, smem);
  if (e != cudaSuccess) return (int)e;
  if (per_sm < 1) return (int)cudaErrorLaunchOutOfResources;
  return (int)launch(decode_persistent, dim3(G), dim3(kConsumers + 32), smem, (cudaStream_t)stream, flags & kFlagPdl,
                     a);
}
