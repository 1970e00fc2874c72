// Batch-1 W4A16 G32 GEMV streamed through shared memory with bulk asynchronous copies.
//
// Structure (one CTA per SM, persistent):
//   * CTA c owns a contiguous, balanced range of output rows (in units of two rows);
//     its weight rows are one contiguous byte range per tensor (codes, scales, zeros),
//     so each pipeline stage of RS rows is a handful of cp.async.bulk copies that
//     complete on an mbarrier (transaction-count based);
//   * one thread issues the first NS stages *before* griddepcontrol.wait, so the
//     weight stream starts while the previous kernel of the decode step finishes;
//   * thread t owns quantization group g = t % G of partition p = t / G and keeps the
//     32 activation values of that group in registers for the whole kernel (after the
//     optional residual add + RMSNorm), so shared memory only carries weight bytes;
//   * partition p handles stage rows i = p, p + P, ...; per row a thread reads its 16
//     code bytes, its scale and zero point, and accumulates with magic-number
//     dequantization and packed FFMA2 (see w4a16.cu);
//   * rows are reduced across the warp with a transposed butterfly (one shuffle per
//     row per lane) and across the partition's warps through shared memory.
// Every mbarrier wait is bounded: on expiry the kernel raises the library error word,
// waits (bounded) for its outstanding copies and returns.
#include <stdlib.h>

#include "stream_pipeline.cuh"

namespace mt {

__device__ int g_error_word;  // non-zero after a bounded wait expired (see mt_error_word)

namespace {

__device__ __forceinline__ float magic_lo(uint32_t w) { return __uint_as_float((w & 0x000F0000u) | 0x43000000u); }
__device__ __forceinline__ float magic_hi(uint32_t w) { return __uint_as_float((w & 0x0000F000u) | 0x45000000u); }

__device__ __forceinline__ void dot_word(uint32_t w, const float* x, float2& acc) {
  const uint32_t r8 = __funnelshift_r(w, w, 8);
  const uint32_t r16 = __byte_perm(w, w, 0x1032);
  const uint32_t r24 = __funnelshift_r(w, w, 24);
  acc = __ffma2_rn(make_float2(magic_lo(r16), magic_hi(r24)), make_float2(x[0], x[1]), acc);
  acc = __ffma2_rn(make_float2(magic_lo(r24), magic_hi(w)), make_float2(x[2], x[3]), acc);
  acc = __ffma2_rn(make_float2(magic_lo(w), magic_hi(r8)), make_float2(x[4], x[5]), acc);
  acc = __ffma2_rn(make_float2(magic_lo(r8), magic_hi(r16)), make_float2(x[6], x[7]), acc);
}

}  // namespace

using namespace pipe;

struct StreamArgs {
  const __nv_bfloat16* x;
  const __nv_bfloat16* residual;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* summed;
  const uint8_t* qweight;
  const __nv_bfloat16* scales;
  const uint8_t* qzeros;
  __nv_bfloat16* y;
  int n, k;
  float eps;
};

// bf16 magic pairs: (w >> s) masked to nibbles at bits 0..3 and 16..19 with the bf16
// exponent of 128 gives the pair (128 + q_j, 128 + q_{j+4}) in one LOP3.
__device__ __forceinline__ uint32_t pair_magic(uint32_t w) { return (w & 0x000F000Fu) | 0x43004300u; }

// fp32 += bf16 * bf16 (exact product, one rounding): sm_100's mixed-precision FMA.
__device__ __forceinline__ float fma_bf16_lo(uint32_t a, uint32_t b, float c) {
  float d;
  asm("{.reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %1;\n mov.b32 {bl, bh}, %2;\n"
      " fma.rn.f32.bf16 %0, al, bl, %3;}" : "=f"(d) : "r"(a), "r"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fma_bf16_hi(uint32_t a, uint32_t b, float c) {
  float d;
  asm("{.reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %1;\n mov.b32 {bl, bh}, %2;\n"
      " fma.rn.f32.bf16 %0, ah, bh, %3;}" : "=f"(d) : "r"(a), "r"(b), "f"(c));
  return d;
}

// One 8-code word against the thread's activation pairs xp[i] = (x[i], x[i+4]) (bf16x2):
// acc.x/acc.y accumulate sum x * (128 + q) over the word. MULHI: the nibble shifts are
// done as 32x32 multiply-high (w * 2^(32-s)) >> 32, which issues outside the logic pipe.
template <bool MULHI>
__device__ __forceinline__ void dot_word_mixed(uint32_t w, const uint32_t* xp, float2& acc) {
  const uint32_t s4 = MULHI ? __umulhi(w, 1u << 28) : (w >> 4);
  const uint32_t s8 = MULHI ? __umulhi(w, 1u << 24) : (w >> 8);
  const uint32_t s12 = MULHI ? __umulhi(w, 1u << 20) : (w >> 12);
  const uint32_t p0 = pair_magic(w), p1 = pair_magic(s4), p2 = pair_magic(s8), p3 = pair_magic(s12);
  acc.x = fma_bf16_lo(p0, xp[0], acc.x);
  acc.y = fma_bf16_hi(p0, xp[0], acc.y);
  acc.x = fma_bf16_lo(p1, xp[1], acc.x);
  acc.y = fma_bf16_hi(p1, xp[1], acc.y);
  acc.x = fma_bf16_lo(p2, xp[2], acc.x);
  acc.y = fma_bf16_hi(p2, xp[2], acc.y);
  acc.x = fma_bf16_lo(p3, xp[3], acc.x);
  acc.y = fma_bf16_hi(p3, xp[3], acc.y);
}

// Warp-specialized streaming GEMV. Warps [0, C) consume, warp C produces (bulk copies).
// RS output rows per stage, NS stages, P row partitions, DOT: 0 = fp32 magic + FFMA2,
// 1 = bf16 magic pairs + mixed-precision FMA. blockDim = P * G + 32.
template <int RS, int NS, int P, int DOT, bool NORM, bool ADD, bool PAIRED>
__global__ void __launch_bounds__(P * 128 + 32 > 416 ? P * 128 + 32 : 416, 1) w4a16_stream(StreamArgs a, int max_rows) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[NS];
  __shared__ __align__(8) uint64_t empty[NS];
  constexpr int H = PAIRED ? 2 : 1;  // weight-row blocks per stage (gate, up)
  constexpr int RP = RS / P;         // rows per partition per stage
  constexpr int NV = RP * H;         // values reduced per lane per stage
  static_assert(RS % P == 0 && (NV & (NV - 1)) == 0 && NV <= 32, "bad tile");
  __shared__ float ssum[32];
  __shared__ int failed;

  const int K = a.k, G = K >> 5;
  const int consumers = P * G, cwarps = consumers >> 5;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool producer = tid >= consumers;
  const int part = producer ? 0 : tid / G, g = producer ? 0 : tid - part * G;
  const int wpp = G >> 5;  // warps per partition
  const size_t row_bytes = (size_t)K >> 1, srow = (size_t)G * 2, zrow = (size_t)(G >> 1);
  const bool zeros = a.qzeros != nullptr;
  const size_t stage_rows_bytes = row_bytes + srow + (zeros ? zrow : 0);
  const size_t stage_bytes = (size_t)RS * H * stage_rows_bytes;

  const int n_out = PAIRED ? a.n / 2 : a.n;
  const int units = n_out >> 1;
  const int u0 = (int)((long)blockIdx.x * units / gridDim.x), u1 = (int)((long)(blockIdx.x + 1) * units / gridDim.x);
  const int r0 = u0 * 2, r1 = u1 * 2, nrows = r1 - r0;
  const int stages = (nrows + RS - 1) / RS;
  float* partial = reinterpret_cast<float*>(smem + (size_t)NS * stage_bytes);  // [cwarps][max_rows][H]

  auto codes_at = [&](int slot) { return smem + (size_t)slot * stage_bytes; };
  auto scales_at = [&](int slot) { return codes_at(slot) + (size_t)RS * H * row_bytes; };
  auto zeros_at = [&](int slot) { return scales_at(slot) + (size_t)RS * H * srow; };
  auto issue = [&](int st) {
    const int slot = st % NS;
    const int rows = min(RS, nrows - st * RS);
    mbar_expect_tx(&full[slot], (unsigned)(rows * H * stage_rows_bytes));
#pragma unroll
    for (int h = 0; h < H; ++h) {
      const size_t row = (size_t)r0 + (size_t)st * RS + (size_t)h * n_out;
      bulk_copy(codes_at(slot) + (size_t)h * RS * row_bytes, a.qweight + row * row_bytes,
                (unsigned)(rows * row_bytes), &full[slot]);
      bulk_copy(scales_at(slot) + (size_t)h * RS * srow, reinterpret_cast<const uint8_t*>(a.scales) + row * srow,
                (unsigned)(rows * srow), &full[slot]);
      if (zeros)
        bulk_copy(zeros_at(slot) + (size_t)h * RS * zrow, a.qzeros + row * zrow, (unsigned)(rows * zrow),
                  &full[slot]);
    }
  };

  if (tid == consumers) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], cwarps);
    }
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // weights never depend on the previous kernel: start streaming before the PDL wait
    for (int st = 0; st < NS && st < stages; ++st) issue(st);
  }
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
      if (st < stages) {  // consumers stopped early: drain what is still in flight
        atomicExch(&g_error_word, 1);
        for (int d = st - NS; d < st; ++d)
          if (d >= 0) mbar_wait_bounded(&full[d % NS], (unsigned)((d / NS) & 1));
      }
    }
    return;
  }

  pdl_wait();
  pdl_trigger();

  // Activation of this thread's group, optionally add + RMSNorm (kernels.py:57-59,76-82).
  float xv[32];
  {
    const uint4* xp = reinterpret_cast<const uint4*>(a.x + (size_t)g * 32);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = xp[q];
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) { xv[8 * q + 2 * i] = bf16_lo(ww[i]); xv[8 * q + 2 * i + 1] = bf16_hi(ww[i]); }
    }
    if (ADD) {
      const uint4* rp = reinterpret_cast<const uint4*>(a.residual + (size_t)g * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = rp[q];
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float& lo = xv[8 * q + 2 * i];
          float& hi = xv[8 * q + 2 * i + 1];
          lo = round_bf16(lo + bf16_lo(ww[i]));
          hi = round_bf16(hi + bf16_hi(ww[i]));
          __nv_bfloat162 pr = __floats2bfloat162_rn(lo, hi);
          o[i] = *reinterpret_cast<uint32_t*>(&pr);
        }
        if (a.summed && blockIdx.x == 0 && part == 0)
          reinterpret_cast<uint4*>(a.summed + (size_t)g * 32)[q] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    if (NORM) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) ss += xv[i] * xv[i];
      ss = warp_sum(part == 0 ? ss : 0.f);
      if (lane == 0) ssum[warp] = ss;
      named_sync(1, consumers);
      float tot = 0.f;
      for (int w = 0; w < wpp; ++w) tot += ssum[w];
      const float inv = 1.0f / sqrtf(tot / (float)K + a.eps);
      const uint4* wp = reinterpret_cast<const uint4*>(a.norm_w + (size_t)g * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = wp[q];
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xv[8 * q + 2 * i] = round_bf16(round_bf16(xv[8 * q + 2 * i] * inv) * bf16_lo(ww[i]));
          xv[8 * q + 2 * i + 1] = round_bf16(round_bf16(xv[8 * q + 2 * i + 1] * inv) * bf16_hi(ww[i]));
        }
      }
    }
  }
  float ev = 0.f, od = 0.f;
#pragma unroll
  for (int i = 0; i < 32; i += 2) { ev += xv[i]; od += xv[i + 1]; }
  const float xsum = ev + od;
  // DOT 0: fp32 magic (128 + q even k, 2048 + q odd k); DOT 1: bf16 pairs, 128 + q everywhere.
  const float2 c0 = DOT == 0 ? make_float2(-128.f * ev, -2048.f * od) : make_float2(-128.f * xsum, 0.f);
  uint32_t xpair[16];  // DOT 1: (x[8w + i], x[8w + i + 4]) as bf16x2, exact (x is bf16)
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 pr = __floats2bfloat162_rn(xv[8 * w + i], xv[8 * w + i + 4]);
      xpair[4 * w + i] = *reinterpret_cast<uint32_t*>(&pr);
    }

  bool ok = true;
  for (int st = 0; st < stages; ++st) {
    const int slot = st % NS;
    const unsigned parity = (unsigned)((st / NS) & 1);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[slot], parity))) { ok = false; break; }
    const int rows = min(RS, nrows - st * RS);
    const uint8_t* cb = codes_at(slot);
    const __nv_bfloat16* sb = reinterpret_cast<const __nv_bfloat16*>(scales_at(slot));
    const uint8_t* zb = zeros_at(slot);
    float acc[NV];
#pragma unroll
    for (int j = 0; j < RP; ++j) {
      const int i = j * P + part;
#pragma unroll
      for (int h = 0; h < H; ++h) {
        float v = 0.f;
        if (i < rows) {
          const int rr = h * RS + i;
          const uint4 w = *reinterpret_cast<const uint4*>(cb + (size_t)rr * row_bytes + (size_t)g * 16);
          const float s = bf16f(sb[(size_t)rr * G + g]);
          float z = 8.f;
          if (zeros) z = (float)((zb[(size_t)rr * (G >> 1) + (g >> 1)] >> ((g & 1) << 2)) & 15u);
          float2 d0 = c0, d1 = make_float2(0.f, 0.f);
          if (DOT == 0) {
            dot_word(w.x, xv + 0, d0);
            dot_word(w.y, xv + 8, d1);
            dot_word(w.z, xv + 16, d0);
            dot_word(w.w, xv + 24, d1);
          } else {
            dot_word_mixed<DOT == 2>(w.x, xpair + 0, d0);
            dot_word_mixed<DOT == 2>(w.y, xpair + 4, d1);
            dot_word_mixed<DOT == 2>(w.z, xpair + 8, d0);
            dot_word_mixed<DOT == 2>(w.w, xpair + 12, d1);
          }
          v = s * fmaf(-z, xsum, (d0.x + d1.x) + (d0.y + d1.y));
        }
        acc[j * H + h] = v;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);  // stage slot may be refilled
    const float tot = butterfly<NV>(acc, lane);
    constexpr int dup = 32 / NV;
    if ((lane & (dup - 1)) == 0) {
      const int v = row_of<NV>(lane), j = v / H, h = v - j * H;
      const int i = j * P + part;
      if (i < rows) partial[((size_t)warp * max_rows + st * RS + i) * H + h] = tot;
    }
  }
  if (!__all_sync(0xffffffffu, ok)) ok = false;
  if (!ok && lane == 0) failed = 1;
  named_sync(1, consumers);
  if (failed) {
    if (tid == 0) atomicExch(&g_error_word, 1);
    return;
  }
  for (int i = tid; i < nrows; i += consumers) {
    const int p = i % P;
    float vals[H];
#pragma unroll
    for (int h = 0; h < H; ++h) {
      float sacc = 0.f;
      for (int w = 0; w < wpp; ++w) sacc += partial[((size_t)(p * wpp + w) * max_rows + i) * H + h];
      vals[h] = sacc;
    }
    float out = vals[0];
    if (PAIRED) {  // dp4a_packing.py:86-89
      const float gate = round_bf16(vals[0]), up = round_bf16(vals[H - 1]);
      out = round_bf16(gate / (1.0f + expf(-gate))) * up;
    }
    a.y[(size_t)r0 + i] = to_bf16(out);
  }
}

size_t stream_smem(int rs, int ns, bool paired, int k, bool zeros, int cwarps, int max_rows) {
  const size_t G = (size_t)k / 32;
  const int h = paired ? 2 : 1;
  return (size_t)ns * rs * h * ((size_t)k / 2 + 2 * G + (zeros ? G / 2 : 0)) +
         (size_t)cwarps * max_rows * h * sizeof(float);
}

// Tuning knobs read once from the environment (defaults are the measured best):
// MT_W4_DOT = 0 (fp32 magic + FFMA2), 1 (bf16 pairs + mixed FMA), 2 (as 1, multiply-high
// shifts); MT_W4_PARTS = row partitions per CTA for K <= 4096 (2 or 4).
static int env_int(const char* name, int dflt) {
  const char* e = getenv(name);
  return (e && e[0] >= '0' && e[0] <= '9') ? atoi(e) : dflt;
}
static int stream_dot_mode() {
  static int mode = -1;
  if (mode < 0) mode = env_int("MT_W4_DOT", 1);
  return mode;
}
static int stream_parts() {
  static int parts = -1;
  if (parts < 0) parts = env_int("MT_W4_PARTS", 4) == 2 ? 2 : 4;
  return parts;
}

template <int RS, int NS, int P, int DOT, bool NORM, bool ADD, bool PAIRED>
static cudaError_t go_dot(const StreamArgs& a, cudaStream_t s, int flags) {
  const int n_out = PAIRED ? a.n / 2 : a.n;
  int blocks = sm_count();
  if (blocks > n_out / 2) blocks = n_out / 2;
  const int units = n_out / 2;
  const int max_rows = 2 * ((units + blocks - 1) / blocks);
  const int cwarps = P * (a.k / 32) / 32;
  const size_t smem = stream_smem(RS, NS, PAIRED, a.k, a.qzeros != nullptr, cwarps, max_rows);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  return launch(w4a16_stream<RS, NS, P, DOT, NORM, ADD, PAIRED>, dim3(blocks), dim3(P * (a.k / 32) + 32), smem,
                s, flags, a, max_rows);
}

template <int RS, int NS, int P, bool NORM, bool ADD, bool PAIRED>
static cudaError_t go(const StreamArgs& a, cudaStream_t s, int flags) {
  switch (stream_dot_mode()) {
    case 0: return go_dot<RS, NS, P, 0, NORM, ADD, PAIRED>(a, s, flags);
    case 2: return go_dot<RS, NS, P, 2, NORM, ADD, PAIRED>(a, s, flags);
    default: return go_dot<RS, NS, P, 1, NORM, ADD, PAIRED>(a, s, flags);
  }
}

template <bool NORM, bool ADD>
static cudaError_t go_k(const StreamArgs& a, bool paired, cudaStream_t s, int flags) {
  const int G = a.k / 32;
  if (G > 128) {  // wide K (down projection): one partition of G consumer threads
    return paired ? go<8, 2, 1, NORM, ADD, true>(a, s, flags) : go<8, 2, 1, NORM, ADD, false>(a, s, flags);
  }
  if (stream_parts() == 4)
    return paired ? go<8, 3, 4, NORM, ADD, true>(a, s, flags) : go<16, 3, 4, NORM, ADD, false>(a, s, flags);
  return paired ? go<8, 3, 2, NORM, ADD, true>(a, s, flags) : go<16, 3, 2, NORM, ADD, false>(a, s, flags);
}

// Batch-1 entry used by mt_w4a16_linear when the shape fits this kernel.
bool stream_supported(int batch, int n, int k, int mode) {
  const int G = k / 32;
  if (batch != 1 || G % 32 || G > 384) return false;
  const int n_out = (mode & 4) ? n / 2 : n;
  if (n_out % 2) return false;
  return true;
}

cudaError_t stream_launch(const void* x, const void* residual, const void* norm_w, float eps, void* summed,
                          const void* qweight, const void* scales, const void* qzeros, void* y, int n, int k,
                          int mode, int flags, cudaStream_t s) {
  StreamArgs a;
  a.x = (const __nv_bfloat16*)x;
  a.residual = (const __nv_bfloat16*)residual;
  a.norm_w = (const __nv_bfloat16*)norm_w;
  a.summed = (__nv_bfloat16*)summed;
  a.qweight = (const uint8_t*)qweight;
  a.scales = (const __nv_bfloat16*)scales;
  a.qzeros = (const uint8_t*)qzeros;
  a.y = (__nv_bfloat16*)y;
  a.n = n;
  a.k = k;
  a.eps = eps;
  const bool paired = mode & 4;
  if (mode & 2) return go_k<true, true>(a, paired, s, flags);
  if (mode & 1) return go_k<true, false>(a, paired, s, flags);
  return go_k<false, false>(a, paired, s, flags);
}

}  // namespace mt

using namespace mt;

// Diagnostic read of the library's error word on the current device (1 after a kernel
// abandoned a bounded wait); optionally clears it. Synchronous, unlike every other call.
namespace mt {
cudaError_t heads_error_word(int* value, bool clear);
}

MT_API int mt_read_error_word(int* value, int clear) {
  if (!value) return kBadArgument;
  cudaError_t e = cudaMemcpyFromSymbol(value, g_error_word, sizeof(int));
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_error_word, &zero, sizeof(int));
  }
  if (e == cudaSuccess) e = heads_error_word(value, clear != 0);
  return (int)e;
}
