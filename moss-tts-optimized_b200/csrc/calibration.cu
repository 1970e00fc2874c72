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
