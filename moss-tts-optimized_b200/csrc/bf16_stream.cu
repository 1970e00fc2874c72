// bf16-weight decode GEMV streamed through shared memory (sm_100a): the batch-1
// projections of the BF16 preset — linear_decode (src/moss_tts/_runtime/kernels.py:93-108)
// and the paired gate/up + SiLU GEMV (fused_mlp.py:7-30) — with the optional residual add
// + RMSNorm prologue of add_rmsnorm (kernels.py:69-90).
//
// One persistent CTA per SM owns a balanced contiguous range of output rows. A producer
// warp streams RS-row stages into a three-deep ring with cp.async.bulk (one copy per stage,
// or two for the fused pair: the stage's gate rows and the matching up rows), full/empty
// mbarriers and bounded waits; the first stages are issued before griddepcontrol.wait, so
// the weight stream of a kernel starts while its predecessor finishes. 512 consumer threads
// own fixed 8-element column chunks (thread t: chunks t + 512 j), keep their (normalised)
// activation in registers and read conflict-free 16-byte words of each staged row. Row sums
// are reduced inside the warp per stage (transposed butterfly) and across warps once, at
// the end, in a fixed order, so results are deterministic.
#include "stream_pipeline.cuh"

namespace mt {

__device__ int g_bf16_error;  // set when a bounded wait expired (read through mt_read_error_word)

using namespace pipe;

struct Bf16StreamArgs {
  const __nv_bfloat16* x;         // [K]
  const __nv_bfloat16* residual;  // [K] (ADD)
  const __nv_bfloat16* norm_w;    // [K] (NORM)
  __nv_bfloat16* summed;          // [K] (ADD, optional)
  const __nv_bfloat16* w;         // [N, K]
  __nv_bfloat16* y;               // [N] or [N/2] (PAIRED)
  int n, k;
  float eps;
  int unit0, units;  // output rows [unit0, unit0 + units) handled by this launch
};

constexpr int kBfConsumers = 512;
constexpr int kBfStages = 3;
constexpr int kBfStageBytes = 64 * 1024;
constexpr int kBfMaxRows = 512;  // partial rows per CTA and launch (64 B of shared memory each)

template <int RS, int KC, bool NORM, bool ADD, bool PAIRED>
__global__ void __launch_bounds__(kBfConsumers + 32, 1) bf16_stream(Bf16StreamArgs a, int max_rows) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kBfStages];
  __shared__ __align__(8) uint64_t empty[kBfStages];
  __shared__ float ssum[kBfConsumers / 32];
  __shared__ int failed;
  constexpr int U = PAIRED ? RS / 2 : RS;  // output rows per stage
  constexpr int kWarps = kBfConsumers / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = a.k, E = K >> 3;
  const size_t row_bytes = (size_t)K * 2, stage_bytes = (size_t)RS * row_bytes;
  const int n_out = PAIRED ? a.n / 2 : a.n;
  const int u0 = a.unit0 + (int)((long)blockIdx.x * a.units / gridDim.x);
  const int nunits = a.unit0 + (int)((long)(blockIdx.x + 1) * a.units / gridDim.x) - u0;
  const int stages = (nunits + U - 1) / U;
  float* partial = reinterpret_cast<float*>(smem + (size_t)kBfStages * stage_bytes);  // [kWarps][max_rows]
  const uint8_t* wb = reinterpret_cast<const uint8_t*>(a.w);

  auto issue = [&](int st) {
    const int slot = st % kBfStages, cnt = min(U, nunits - st * U), g = u0 + st * U;
    uint8_t* dst = smem + (size_t)slot * stage_bytes;
    const unsigned bytes = (unsigned)(cnt * row_bytes);
    mbar_expect_tx(&full[slot], PAIRED ? 2 * bytes : bytes);
    bulk_copy(dst, wb + (size_t)g * row_bytes, bytes, &full[slot]);
    if (PAIRED) bulk_copy(dst + (size_t)U * row_bytes, wb + (size_t)(n_out + g) * row_bytes, bytes, &full[slot]);
  };

  if (tid == kBfConsumers) {
#pragma unroll
    for (int s = 0; s < kBfStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int st = 0; st < kBfStages && st < stages; ++st) issue(st);
  }
  __syncthreads();

  if (tid >= kBfConsumers) {  // producer warp
    pdl_trigger();
    if (lane == 0) {
      int st = kBfStages;
      for (; st < stages; ++st) {
        const int slot = st % kBfStages;
        if (!mbar_wait_bounded(&empty[slot], (unsigned)(((st / kBfStages) - 1) & 1))) break;
        issue(st);
      }
      if (st < stages) {  // abandoned: record it and let the copies in flight land
        atomicExch(&g_bf16_error, 1);
        for (int d = st - kBfStages; d < st; ++d)
          if (d >= 0) mbar_wait_bounded(&full[d % kBfStages], (unsigned)((d / kBfStages) & 1));
      }
    }
    return;
  }

  pdl_wait();
  pdl_trigger();

  // Activation chunks in registers: optional bf16 residual add, RMSNorm with the
  // reference's rounding points (bf16(x * inv) then bf16(. * w)).
  float xv[KC][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < KC; ++j) {
    const int e = tid + kBfConsumers * j;
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[j][i] = 0.f;
    if (e < E) {
      const uint4 xr = reinterpret_cast<const uint4*>(a.x)[e];
      const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) { xv[j][2 * i] = bf16_lo(xw[i]); xv[j][2 * i + 1] = bf16_hi(xw[i]); }
      if (ADD) {
        const uint4 rr = reinterpret_cast<const uint4*>(a.residual)[e];
        const uint32_t rw[4] = {rr.x, rr.y, rr.z, rr.w};
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xv[j][2 * i] = round_bf16(xv[j][2 * i] + bf16_lo(rw[i]));
          xv[j][2 * i + 1] = round_bf16(xv[j][2 * i + 1] + bf16_hi(rw[i]));
          __nv_bfloat162 p = __floats2bfloat162_rn(xv[j][2 * i], xv[j][2 * i + 1]);
          o[i] = *reinterpret_cast<uint32_t*>(&p);
        }
        if (a.summed && blockIdx.x == 0) reinterpret_cast<uint4*>(a.summed)[e] = make_uint4(o[0], o[1], o[2], o[3]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += xv[j][i] * xv[j][i];
    }
  }
  if (NORM) {
    ss = warp_sum(ss);
    if (lane == 0) ssum[warp] = ss;
    named_sync(1, kBfConsumers);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tot += ssum[w];
    const float inv = 1.0f / sqrtf(tot / (float)K + a.eps);
#pragma unroll
    for (int j = 0; j < KC; ++j) {
      const int e = tid + kBfConsumers * j;
      if (e < E) {
        const uint4 wr = reinterpret_cast<const uint4*>(a.norm_w)[e];
        const uint32_t ww[4] = {wr.x, wr.y, wr.z, wr.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xv[j][2 * i] = round_bf16(round_bf16(xv[j][2 * i] * inv) * bf16_lo(ww[i]));
          xv[j][2 * i + 1] = round_bf16(round_bf16(xv[j][2 * i + 1] * inv) * bf16_hi(ww[i]));
        }
      }
    }
  }

  bool ok = true;
  for (int st = 0; st < stages; ++st) {
    const int slot = st % kBfStages;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[slot], (unsigned)((st / kBfStages) & 1)))) {
      ok = false;
      break;
    }
    const int cnt = min(U, nunits - st * U);
    const uint8_t* base = smem + (size_t)slot * stage_bytes;
    float acc[RS];
#pragma unroll
    for (int i = 0; i < RS; ++i) {
      float2 d = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const int e = tid + kBfConsumers * j;
        if ((i % U) < cnt && e < E) {
          const uint4 w = *reinterpret_cast<const uint4*>(base + (size_t)i * row_bytes + (size_t)e * 16);
          d = __ffma2_rn(make_float2(bf16_lo(w.x), bf16_hi(w.x)), make_float2(xv[j][0], xv[j][1]), d);
          d = __ffma2_rn(make_float2(bf16_lo(w.y), bf16_hi(w.y)), make_float2(xv[j][2], xv[j][3]), d);
          d = __ffma2_rn(make_float2(bf16_lo(w.z), bf16_hi(w.z)), make_float2(xv[j][4], xv[j][5]), d);
          d = __ffma2_rn(make_float2(bf16_lo(w.w), bf16_hi(w.w)), make_float2(xv[j][6], xv[j][7]), d);
        }
      }
      acc[i] = d.x + d.y;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    const float tot = butterfly<RS>(acc, lane);
    constexpr int dup = 32 / RS;
    if ((lane & (dup - 1)) == 0) {
      const int i = row_of<RS>(lane);
      if ((i % U) < cnt) partial[(size_t)warp * max_rows + st * RS + i] = tot;
    }
  }
  if (!ok) failed = 1;
  named_sync(1, kBfConsumers);
  if (failed) {
    if (tid == 0) atomicExch(&g_bf16_error, 1);
    return;
  }
  for (int u = tid; u < nunits; u += kBfConsumers) {
    const int p = (u / U) * RS + u % U;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += partial[(size_t)w * max_rows + p];
    if (PAIRED) {  // fused_mlp.py:18-23: bf16 gate and up, bf16 SiLU, product rounded once
      float up = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) up += partial[(size_t)w * max_rows + p + U];
      const float gate = round_bf16(v);
      v = round_bf16(gate / (1.0f + expf(-gate))) * round_bf16(up);
    }
    a.y[u0 + u] = to_bf16(v);
  }
}

template <int RS, int KC>
static cudaError_t bf16_stream_mode(const Bf16StreamArgs& a, int mode, int blocks, int max_rows, size_t smem,
                                    cudaStream_t s, int flags) {
  const dim3 grid(blocks), block(kBfConsumers + 32);
  switch (mode) {
    case 0: return launch(bf16_stream<RS, KC, false, false, false>, grid, block, smem, s, flags, a, max_rows);
    case 1: return launch(bf16_stream<RS, KC, true, false, false>, grid, block, smem, s, flags, a, max_rows);
    case 3: return launch(bf16_stream<RS, KC, true, true, false>, grid, block, smem, s, flags, a, max_rows);
    case 4: return launch(bf16_stream<RS, KC, false, false, true>, grid, block, smem, s, flags, a, max_rows);
    case 5: return launch(bf16_stream<RS, KC, true, false, true>, grid, block, smem, s, flags, a, max_rows);
    case 7: return launch(bf16_stream<RS, KC, true, true, true>, grid, block, smem, s, flags, a, max_rows);
    default: return cudaErrorInvalidValue;
  }
}

// Batch-1 dispatch of mt_bf16_linear. Returns false (nothing launched) for shapes the
// streaming kernel does not take: K above 12288 or not a multiple of 8.
bool bf16_stream_linear(const Bf16StreamArgs& args, int mode, int flags, cudaStream_t s, cudaError_t* err) {
  const int K = args.k;
  if (K < 8 || K % 8 || K > 3 * kBfConsumers * 8) return false;
  const size_t row_bytes = (size_t)K * 2;
  int rs = 32;
  while (rs > 2 && (size_t)rs * row_bytes > kBfStageBytes) rs >>= 1;
  const int kc = (K / 8 + kBfConsumers - 1) / kBfConsumers;
  // (RS, KC) pairs that the shape rule above produces
  if (!((kc == 1 && rs >= 8) || (kc == 2 && rs == 4) || (kc == 3 && rs == 2))) return false;
  const bool paired = mode & 4;
  const int U = paired ? rs / 2 : rs;
  const int n_out = paired ? args.n / 2 : args.n;
  const int sms = sm_count();
  const int per_launch = sms * (kBfMaxRows / rs) * U;  // output rows one launch can hold
  *err = cudaSuccess;
  for (int u0 = 0; u0 < n_out; u0 += per_launch) {
    Bf16StreamArgs a = args;
    a.unit0 = u0;
    a.units = n_out - u0 < per_launch ? n_out - u0 : per_launch;
    const int blocks = a.units < sms ? a.units : sms;
    const int max_units = (a.units + blocks - 1) / blocks;
    const int max_rows = ((max_units + U - 1) / U) * rs;
    const size_t smem = (size_t)kBfStages * rs * row_bytes + (size_t)(kBfConsumers / 32) * max_rows * sizeof(float);
    if (smem > 227 * 1024) { *err = cudaErrorInvalidValue; return true; }
    if (u0 > 0) a.summed = nullptr;  // the first launch already wrote the sum
    switch (rs) {
      case 32: *err = bf16_stream_mode<32, 1>(a, mode, blocks, max_rows, smem, s, flags); break;
      case 16: *err = bf16_stream_mode<16, 1>(a, mode, blocks, max_rows, smem, s, flags); break;
      case 8: *err = bf16_stream_mode<8, 1>(a, mode, blocks, max_rows, smem, s, flags); break;
      case 4: *err = bf16_stream_mode<4, 2>(a, mode, blocks, max_rows, smem, s, flags); break;
      default: *err = bf16_stream_mode<2, 3>(a, mode, blocks, max_rows, smem, s, flags); break;
    }
    if (*err != cudaSuccess) return true;
  }
  return true;
}

cudaError_t bf16_error_word(int* value, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_bf16_error, sizeof(int));
  if (e != cudaSuccess) return e;
  *value |= v;
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_bf16_error, &zero, sizeof(int));
  }
  return e;
}

}  // namespace mt
