// Offline G32 calibration helpers (sm_100a): the static per-group scales of the reference's
// calibrated export (src/moss_tts/_runtime/calibrated_quant.py:36-38),
//   scale[n][g] = bf16(max(max_{k in g} |W[n][k]|, 1e-8) / 7),
// computed with one fp32 division and one round to nearest even, as the reference's
// `.float() ... / 7` then `.bfloat16()` does.
#include <cuda_fp16.h>

#include "common.cuh"

namespace mt {

template <typename T>
__device__ __forceinline__ float load_f(const T* p);
template <>
__device__ __forceinline__ float load_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float load_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_f<__half>(const __half* p) { return __half2float(*p); }

// One warp per (row, group): lane l reads element l of the group (coalesced), warp max.
template <typename T>
__global__ void static_scales_kernel(const T* __restrict__ w, __nv_bfloat16* __restrict__ out, long long groups,
                                     int k) {
  const long long gid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gid >= groups) return;
  const int lane = threadIdx.x & 31;
  const long long row = gid / (k / 32), g = gid - row * (k / 32);
  float m = fabsf(load_f<T>(w + row * k + g * 32 + lane));
  m = warp_max(m);
  if (lane == 0) out[gid] = __float2bfloat16_rn(fmaxf(m, 1e-8f) / 7.0f);
}

}  // namespace mt

using namespace mt;

// Static G32 scales of a weight matrix w [n, k] (dtype 0 bf16, 1 fp32, 2 fp16) into out bf16
// [n, k / 32]. Replaces calibrated_quant.static_scales (src/moss_tts/_runtime/calibrated_quant.py:36-38).
MT_API int mt_static_scales(const void* w, int dtype, void* out, int n, int k, void* stream) {
  if (!w || !out || n < 1 || k < 32 || k % 32 || dtype < 0 || dtype > 2) return kBadArgument;
  const long long groups = (long long)n * (k / 32);
  const unsigned warps = 8;
  const unsigned ctas = (unsigned)((groups + warps - 1) / warps);
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == 0)
    static_scales_kernel<__nv_bfloat16><<<ctas, warps * 32, 0, s>>>((const __nv_bfloat16*)w, (__nv_bfloat16*)out, groups, k);
  else if (dtype == 1)
    static_scales_kernel<float><<<ctas, warps * 32, 0, s>>>((const float*)w, (__nv_bfloat16*)out, groups, k);
  else
    static_scales_kernel<__half><<<ctas, warps * 32, 0, s>>>((const __half*)w, (__nv_bfloat16*)out, groups, k);
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// GPTQ block solver: the column loop of calibrated_quant.gptq (src/moss_tts/_runtime/
// calibrated_quant.py:46-85; the reference runs it as one Triton _column launch per column,
// calibrated_quant.py:15-33). Rows are independent inside a block of columns, so one launch
// handles a whole block: CTA b owns kRows weight rows, keeps their block of the (permuted,
// fp32) weights in shared memory and steps through the block's columns:
//   code  = rint(w / s) clamped to [-7, 7]            (round half to even, as torch .round())
//   q     = float(bf16(code * s))
//   err   = (w - q) / hinv[c][c]
//   w[:, j] -= err * hinv[c][j]   for j >= c           (a product, then a difference)
// every operation rounded on its own (no fused multiply-add), in the reference's order. The
// caller applies the block's errors to the columns after it (errors @ hinv, a plain matmul).
namespace mt {
namespace gptq {
constexpr int kRows = 16;      // weight rows per CTA
constexpr int kThreads = 128;  // one thread per column of a block of up to 128 columns

__global__ void __launch_bounds__(kThreads) block_kernel(float* __restrict__ w, float* __restrict__ errors,
                                                         int8_t* __restrict__ codes,
                                                         const __nv_bfloat16* __restrict__ scales,
                                                         const float* __restrict__ hinv,
                                                         const long long* __restrict__ perm, int start, int cols,
                                                         int n, int k, int group) {
  __shared__ float tile[kRows][kThreads + 1];
  __shared__ float err[kRows];
  const int r0 = blockIdx.x * kRows, j = threadIdx.x;
  const int rows = min(kRows, n - r0);
  for (int r = 0; r < rows; ++r) tile[r][j] = j < cols ? w[(size_t)(r0 + r) * cols + j] : 0.f;
  __syncthreads();
  for (int c = 0; c < cols; ++c) {
    const float* hrow = hinv + (size_t)(start + c) * k + start;
    if (j < rows) {
      const int r = j;
      const long long orig = perm[start + c];
      const float s = __bfloat162float(scales[(size_t)(r0 + r) * (k / group) + orig / group]);
      const float value = tile[r][c];
      float code = rintf(__fdiv_rn(value, s));
      code = fminf(fmaxf(code, -7.f), 7.f);
      const float q = __bfloat162float(__float2bfloat16_rn(__fmul_rn(code, s)));
      const float e = __fdiv_rn(__fsub_rn(value, q), hrow[c]);
      codes[(size_t)(r0 + r) * k + orig] = (int8_t)code;
      errors[(size_t)(r0 + r) * cols + c] = e;
      err[r] = e;
    }
    __syncthreads();
    if (j >= c && j < cols) {
      const float h = hrow[j];
      for (int r = 0; r < rows; ++r) tile[r][j] = __fsub_rn(tile[r][j], __fmul_rn(err[r], h));
    }
    __syncthreads();
  }
  for (int r = 0; r < rows; ++r)
    if (j < cols) w[(size_t)(r0 + r) * cols + j] = tile[r][j];
}
}  // namespace gptq
}  // namespace mt

// One block of GPTQ columns [start, start + cols) (cols <= 128) for n weight rows: w fp32 [n, cols]
// (the block of the permuted weights, updated in place), errors fp32 [n, cols] (out), codes int8
// [n, k] (written at the permuted columns' original positions), scales bf16 [n, k / group],
// hinv fp32 [k, k] (upper Cholesky factor of the inverse Hessian, permuted), perm int64 [k].
// Replaces the per-column _column launches of calibrated_quant.gptq (calibrated_quant.py:15-33, 67-80).
MT_API int mt_gptq_block(void* w, void* errors, void* codes, const void* scales, const void* hinv, const void* perm,
                         int start, int cols, int n, int k, int group, void* stream) {
  if (!w || !errors || !codes || !scales || !hinv || !perm || n < 1 || k < 1 || cols < 1 ||
      cols > mt::gptq::kThreads || start < 0 || start + cols > k || group < 1 || k % group)
    return kBadArgument;
  const unsigned ctas = (unsigned)((n + mt::gptq::kRows - 1) / mt::gptq::kRows);
  mt::gptq::block_kernel<<<ctas, mt::gptq::kThreads, 0, (cudaStream_t)stream>>>(
      (float*)w, (float*)errors, (int8_t*)codes, (const __nv_bfloat16*)scales, (const float*)hinv,
      (const long long*)perm, start, cols, n, k, group);
  return (int)cudaGetLastError();
}
