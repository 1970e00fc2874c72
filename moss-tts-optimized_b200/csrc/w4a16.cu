// W4A16 G32 quantized linear for batch-1..8 decode on B200 (sm_100a).
//
// Weight format (the reference's calibrated export byte layout,
// src/moss_tts/calibration.py:190-191, generalised with GPTQ zero points):
//   qweight uint8 [N, K/2]   code k of row n in nibble (k & 1) of byte k/2
//                            (== int32 [N, K/8] with element 8i+j in nibble j)
//   scales  bf16  [N, K/32]  one scale per group of 32 along K
//   qzeros  uint8 [N, K/64]  one 4-bit zero point per group, two per byte,
//                            or null for the symmetric export (z = 8)
//   W[n, k] = bf16((q - z) * s)        (exact fp32 product, one RNE rounding)
//
// GEMV design (HBM bound: 0.5 B of codes per weight, ~1 FLOP per byte):
//   * one warp owns R output rows (2R weight rows when the gate/up pair is
//     fused); lane l of chunk c owns group g = 32c + l, so each warp-wide 16-byte
//     load pulls 512 contiguous bytes of a row: one full group per lane;
//   * the activation lives in shared memory as fp32, transposed to
//     [8 quads][G groups] float4 so the 32 lanes read consecutive 16-byte words
//     (bank-conflict free), reused by all rows of the CTA;
//   * nibbles become floats with one LOP3 each ("magic number" dequantization:
//     a nibble OR-ed into the mantissa of 128.0 or 2048.0 at the bit that is worth
//     1 gives M + q); the per-group constant sum of M * x is folded into the
//     accumulator's initial value, the zero point is applied per group as
//     z * sum(x), and the scale once per group: acc += s * (sum x (q) - z sum x);
//   * products accumulate with Blackwell's packed FFMA2 (fma.rn.f32x2) in fp32;
//   * lanes reduce with warp shuffles; the fused epilogue applies
//     bf16(silu(bf16 gate)) * bf16 up (src/moss_tts/_runtime/dp4a_packing.py:85-89).
//   * optional prologue: bf16 residual add + Qwen3 RMSNorm of the activation,
//     recomputed per CTA (src/moss_tts/_runtime/dp4a_norm_projection.py:48-117).
// The scale is applied after the integer-valued dot product of each group, so
// the result equals dequantize-then-matmul up to fp32 rounding (the dequantized
// bf16 weights themselves are produced bit-exactly by mt_dequant_w4).
#include "common.cuh"

namespace mt {

struct W4Args {
  const __nv_bfloat16* x;         // [B, K] activation (pre-norm input when NORM)
  const __nv_bfloat16* residual;  // [B, K] added before the norm (ADD)
  const __nv_bfloat16* norm_w;    // [K] RMSNorm weight (NORM)
  __nv_bfloat16* summed;          // [B, K] receives bf16(x + residual) (ADD, optional)
  const uint8_t* qweight;         // [N, K/2]
  const __nv_bfloat16* scales;    // [N, K/32]
  const uint8_t* qzeros;          // [N, K/64] or null (z = 8)
  __nv_bfloat16* y;               // [B, N] or [B, N/2] when PAIRED
  int batch, n, k;
  float eps;
};

__device__ __forceinline__ float magic_lo(uint32_t w) {  // nibble at bits 16..19 -> 128 + q
  return __uint_as_float((w & 0x000F0000u) | 0x43000000u);
}
__device__ __forceinline__ float magic_hi(uint32_t w) {  // nibble at bits 12..15 -> 2048 + q
  return __uint_as_float((w & 0x0000F000u) | 0x45000000u);
}

// acc.x += sum over even j of x[8i+j] * (128 + q_j); acc.y over odd j with 2048.
__device__ __forceinline__ void dot_word(uint32_t w, float4 xa, float4 xb, float2& acc) {
  const uint32_t r8 = __funnelshift_r(w, w, 8);
  const uint32_t r16 = __byte_perm(w, w, 0x1032);
  const uint32_t r24 = __funnelshift_r(w, w, 24);
  acc = __ffma2_rn(make_float2(magic_lo(r16), magic_hi(r24)), make_float2(xa.x, xa.y), acc);
  acc = __ffma2_rn(make_float2(magic_lo(r24), magic_hi(w)), make_float2(xa.z, xa.w), acc);
  acc = __ffma2_rn(make_float2(magic_lo(w), magic_hi(r8)), make_float2(xb.x, xb.y), acc);
  acc = __ffma2_rn(make_float2(magic_lo(r8), magic_hi(r16)), make_float2(xb.z, xb.w), acc);
}

__device__ __forceinline__ float zero_point(const uint8_t* qzeros, size_t row, int gpr, int g) {
  if (!qzeros) return 8.f;
  const uint32_t b = qzeros[row * (size_t)(gpr >> 1) + (g >> 1)];
  return (float)((b >> ((g & 1) << 2)) & 15u);
}

// Stage the activation rows into shared memory (fp32, [b][quad j][group g]) with
// the optional add + RMSNorm, and the per-group correction terms.
template <int B, bool NORM, bool ADD>
__device__ __forceinline__ void stage_activation(const W4Args& a, float4* xs, float2* corr,
                                                 float* xsum, float* red) {
  const int K = a.k, G = K >> 5, slots = 8 * G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = blockDim.x >> 5;
  for (int b = 0; b < B; ++b) {
    const bool live = b < a.batch;
    float ss = 0.f;
    for (int s = tid; s < slots; s += blockDim.x) {
      const int g = s >> 3, j = s & 7;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (live) {
        const uint2 xr = *reinterpret_cast<const uint2*>(a.x + (size_t)b * K + 4 * s);
        v = make_float4(bf16_lo(xr.x), bf16_hi(xr.x), bf16_lo(xr.y), bf16_hi(xr.y));
        if (ADD) {
          const uint2 rr = *reinterpret_cast<const uint2*>(a.residual + (size_t)b * K + 4 * s);
          v.x = round_bf16(v.x + bf16_lo(rr.x));
          v.y = round_bf16(v.y + bf16_hi(rr.x));
          v.z = round_bf16(v.z + bf16_lo(rr.y));
          v.w = round_bf16(v.w + bf16_hi(rr.y));
          if (a.summed && blockIdx.x == 0) {
            __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
            uint2 o;
            o.x = *reinterpret_cast<uint32_t*>(&lo);
            o.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(a.summed + (size_t)b * K + 4 * s) = o;
          }
        }
      }
      if (NORM) ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      xs[(b * 8 + j) * G + g] = v;
    }
    if (NORM) {
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float tot = 0.f;
      for (int w = 0; w < nwarp; ++w) tot += red[w];
      __syncthreads();
      const float inv = 1.0f / sqrtf(tot / (float)K + a.eps);
      for (int s = tid; s < slots; s += blockDim.x) {
        const int g = s >> 3, j = s & 7;
        float4 v = xs[(b * 8 + j) * G + g];
        const uint2 wr = *reinterpret_cast<const uint2*>(a.norm_w + 4 * s);
        // Qwen3 order: normalized value rounded to bf16, times weight, rounded again
        // (src/moss_tts/_runtime/kernels.py:57-59).
        v.x = round_bf16(round_bf16(v.x * inv) * bf16_lo(wr.x));
        v.y = round_bf16(round_bf16(v.y * inv) * bf16_hi(wr.x));
        v.z = round_bf16(round_bf16(v.z * inv) * bf16_lo(wr.y));
        v.w = round_bf16(round_bf16(v.w * inv) * bf16_hi(wr.y));
        if (!live) v = make_float4(0.f, 0.f, 0.f, 0.f);
        xs[(b * 8 + j) * G + g] = v;
      }
    }
  }
  __syncthreads();
  // Corrections: eight consecutive slots form one group; reduce with shuffles.
  for (int b = 0; b < B; ++b) {
    for (int s = tid; s < slots; s += blockDim.x) {
      const int g = s >> 3, j = s & 7;
      const float4 v = xs[(b * 8 + j) * G + g];
      float ev = v.x + v.z, od = v.y + v.w;
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        ev += __shfl_xor_sync(0xffffffffu, ev, o);
        od += __shfl_xor_sync(0xffffffffu, od, o);
      }
      if (j == 0) {
        corr[b * G + g] = make_float2(-128.f * ev, -2048.f * od);
        xsum[b * G + g] = ev + od;
      }
    }
  }
  __syncthreads();
}

template <int B, int R, bool NORM, bool ADD, bool PAIRED>
__global__ void __launch_bounds__(256, B == 1 ? 2 : 1) w4a16_gemv(W4Args a) {
  extern __shared__ __align__(16) float4 smem[];
  __shared__ float red[32];
  const int K = a.k, G = K >> 5;
  float4* xs = smem;
  float2* corr = reinterpret_cast<float2*>(xs + B * 8 * G);
  float* xsum = reinterpret_cast<float*>(corr + B * G);

  constexpr int RR = PAIRED ? 2 * R : R;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
  const int n_out = PAIRED ? a.n / 2 : a.n;
  const int tasks = n_out / R;
  // Tasks are dealt round-robin over CTAs first so every SM gets a similar share.
  const int gw = warp * gridDim.x + blockIdx.x, tw = gridDim.x * nwarp;
  const size_t row_bytes = (size_t)K >> 1;

  // Weights never depend on the previous kernel: start pulling this warp's first
  // task into L2 before waiting on the predecessor.
  if (lane == 0 && gw < tasks) {
#pragma unroll
    for (int h = 0; h < (PAIRED ? 2 : 1); ++h) {
      const size_t row = (size_t)gw * R + (size_t)h * n_out;
      prefetch_l2_bulk(a.qweight + row * row_bytes, (uint32_t)(R * row_bytes));
    }
  }
  pdl_wait();
  pdl_trigger();
  stage_activation<B, NORM, ADD>(a, xs, corr, xsum, red);

  const int chunks = (G + 31) >> 5;
  for (int t = gw; t < tasks; t += tw) {
    size_t rows[RR];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      rows[i] = (size_t)t * R + i;
      if (PAIRED) rows[R + i] = rows[i] + n_out;
    }
    float acc[B][RR];
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
      for (int r = 0; r < RR; ++r) acc[b][r] = 0.f;

    uint4 wn[RR];
    float sn[RR], zn[RR];
    auto fetch = [&](int g, uint4* w, float* s, float* z) {
#pragma unroll
      for (int r = 0; r < RR; ++r) {
        w[r] = ld_stream_v4(a.qweight + rows[r] * row_bytes + (size_t)g * 16);
        s[r] = bf16f(a.scales[rows[r] * G + g]);
        z[r] = zero_point(a.qzeros, rows[r], G, g);
      }
    };
    if (lane < G) fetch(lane, wn, sn, zn);
    for (int c = 0; c < chunks; ++c) {
      const int g = (c << 5) + lane;
      uint4 w[RR];
      float s[RR], z[RR];
#pragma unroll
      for (int r = 0; r < RR; ++r) { w[r] = wn[r]; s[r] = sn[r]; z[r] = zn[r]; }
      if (c + 1 < chunks && g + 32 < G) fetch(g + 32, wn, sn, zn);
      if (g < G) {
#pragma unroll
        for (int b = 0; b < B; ++b) {
          float4 xv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[j] = xs[(b * 8 + j) * G + g];
          const float2 c0 = corr[b * G + g];
          const float sx = xsum[b * G + g];
#pragma unroll
          for (int r = 0; r < RR; ++r) {
            float2 d = c0;
            dot_word(w[r].x, xv[0], xv[1], d);
            dot_word(w[r].y, xv[2], xv[3], d);
            dot_word(w[r].z, xv[4], xv[5], d);
            dot_word(w[r].w, xv[6], xv[7], d);
            acc[b][r] = fmaf(s[r], fmaf(-z[r], sx, d.x + d.y), acc[b][r]);
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
      for (int r = 0; r < RR; ++r) acc[b][r] = warp_sum(acc[b][r]);
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b >= a.batch) break;
#pragma unroll
        for (int i = 0; i < R; ++i) {
          float v = acc[b][i];
          if (PAIRED) {
            const float gate = round_bf16(v), up = round_bf16(acc[b][R + i]);
            const float act = round_bf16(gate / (1.0f + expf(-gate)));
            v = act * up;
          }
          a.y[(size_t)b * n_out + rows[i]] = to_bf16(v);
        }
      }
    }
  }
}

// Bit-exact dequantization: one thread per 8-code word -> 16 bytes of bf16.
__global__ void dequant_w4(const uint32_t* __restrict__ qw, const __nv_bfloat16* __restrict__ scales,
                           const uint8_t* __restrict__ qzeros, __nv_bfloat16* __restrict__ out,
                           int n, int k) {
  const int wpr = k >> 3, gpr = k >> 5;
  const size_t words = (size_t)n * wpr;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < words;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / wpr;
    const int wi = (int)(i - row * wpr), g = wi >> 2;
    const float s = bf16f(scales[row * gpr + g]);
    const float z = zero_point(qzeros, row, gpr, g);
    const uint32_t w = qw[i];
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = ((float)((w >> (8 * j)) & 15u) - z) * s;
      const float hi = ((float)((w >> (8 * j + 4)) & 15u) - z) * s;
      __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
      o[j] = *reinterpret_cast<uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(out + i * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

static size_t w4_smem_bytes(int b, int k) { return (size_t)b * (k / 32) * (8 * 16 + 8 + 4); }

template <int B, int R, bool NORM, bool ADD, bool PAIRED>
static cudaError_t launch_w4(const W4Args& a, cudaStream_t stream, int flags) {
  const int n_out = PAIRED ? a.n / 2 : a.n;
  const int tasks = n_out / R;
  const size_t smem = w4_smem_bytes(B, a.k);
  const int per_sm = (B > 1 || smem > 100 * 1024) ? 1 : 2;
  int blocks = sm_count() * per_sm;
  if (blocks > tasks) blocks = tasks;
  return launch(w4a16_gemv<B, R, NORM, ADD, PAIRED>, dim3(blocks), dim3(256), smem, stream, flags, a);
}

template <int B, bool NORM, bool ADD>
static cudaError_t dispatch_paired(const W4Args& a, bool paired, cudaStream_t s, int flags) {
  return paired ? launch_w4<B, 2, NORM, ADD, true>(a, s, flags) : launch_w4<B, 4, NORM, ADD, false>(a, s, flags);
}

template <int B>
static cudaError_t dispatch_mode(const W4Args& a, int mode, cudaStream_t s, int flags) {
  const bool paired = mode & 4;
  if (mode & 2) return dispatch_paired<B, true, true>(a, paired, s, flags);
  if (mode & 1) return dispatch_paired<B, true, false>(a, paired, s, flags);
  return dispatch_paired<B, false, false>(a, paired, s, flags);
}

}  // namespace mt

using namespace mt;

// Replaces the reference's G32 quantized projections: int4_dp4a
// (src/moss_tts/_runtime/int4_dp4a.py:56-74), dp4a_packing.linear / project
// (dp4a_packing.py:94-125, paired gate/up + SiLU at :85-89) and the fused
// residual/RMSNorm prologue of dp4a_norm_projection.linear (:99-117), as W4A16.
MT_API int mt_w4a16_linear(const void* x, const void* residual, const void* norm_w, float eps,
                           void* summed, const void* qweight, const void* scales, const void* qzeros,
                           void* y, int batch, int n, int k, int group, int mode, int flags,
                           void* stream) {
  const bool paired = mode & 4;
  if (!x || !qweight || !scales || !y || group != 32 || batch < 1 || batch > 8 || k < 128 ||
      k % 128 || n < 4 || n % (paired ? 8 : 4) || (mode & ~7))
    return kBadArgument;
  if ((mode & 2) && (!(mode & 1) || !residual)) return kBadArgument;
  if ((mode & 1) && !norm_w) return kBadArgument;
  if (!aligned(x, 8) || !aligned(qweight, 16) || (residual && !aligned(residual, 8)) ||
      (summed && !aligned(summed, 8)) || (norm_w && !aligned(norm_w, 8)) || !aligned(scales, 2))
    return kBadArgument;
  // Rows per launch: the whole batch when its staged activations fit in shared memory,
  // otherwise chunks of it (each chunk streams the weights again).
  int chunk = batch;
  auto padded = [](int b) { return b == 1 ? 1 : b == 2 ? 2 : b <= 4 ? 4 : 8; };
  while (chunk > 1 && w4_smem_bytes(padded(chunk), k) > 200 * 1024) chunk = (chunk + 1) / 2;
  if (w4_smem_bytes(1, k) > 200 * 1024) return kBadArgument;
  const int n_out = paired ? n / 2 : n;
  cudaStream_t s = (cudaStream_t)stream;
  for (int b0 = 0; b0 < batch; b0 += chunk) {
    W4Args a;
    a.x = (const __nv_bfloat16*)x + (size_t)b0 * k;
    a.residual = residual ? (const __nv_bfloat16*)residual + (size_t)b0 * k : nullptr;
    a.norm_w = (const __nv_bfloat16*)norm_w;
    a.summed = summed ? (__nv_bfloat16*)summed + (size_t)b0 * k : nullptr;
    a.qweight = (const uint8_t*)qweight;
    a.scales = (const __nv_bfloat16*)scales;
    a.qzeros = (const uint8_t*)qzeros;
    a.y = (__nv_bfloat16*)y + (size_t)b0 * n_out;
    a.batch = batch - b0 < chunk ? batch - b0 : chunk;
    a.n = n;
    a.k = k;
    a.eps = eps;
    cudaError_t e;
    switch (padded(a.batch)) {
      case 1: e = dispatch_mode<1>(a, mode, s, flags & kFlagPdl); break;
      case 2: e = dispatch_mode<2>(a, mode, s, flags & kFlagPdl); break;
      case 4: e = dispatch_mode<4>(a, mode, s, flags & kFlagPdl); break;
      default: e = dispatch_mode<8>(a, mode, s, flags & kFlagPdl); break;
    }
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

// Replaces calibrated_backend.unpack_signed + calibrated_quant.dequantize
// (src/moss_tts/_runtime/calibrated_backend.py:8-13, calibrated_quant.py:41-42),
// generalised to per-group zero points: out[n, k] = bf16((q - z) * s).
MT_API int mt_dequant_w4(const void* qweight, const void* scales, const void* qzeros, void* out,
                         int n, int k, int group, void* stream) {
  if (!qweight || !scales || !out || group != 32 || n < 1 || k < 64 || k % 64) return kBadArgument;
  if (!aligned(qweight, 4) || !aligned(out, 16)) return kBadArgument;
  const size_t words = (size_t)n * (k / 8);
  size_t blocks = (words + 255) / 256;
  const size_t cap = (size_t)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  dequant_w4<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      (const uint32_t*)qweight, (const __nv_bfloat16*)scales, (const uint8_t*)qzeros,
      (__nv_bfloat16*)out, n, k);
  return (int)cudaGetLastError();
}
