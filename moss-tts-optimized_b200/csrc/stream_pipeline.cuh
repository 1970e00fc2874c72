// Shared pieces of the bulk-copy streaming kernels (sm_100a): mbarrier waits with an
// iteration bound, 1-D bulk global->shared copies completing on an mbarrier, named
// barriers and a transposed warp reduction.
#pragma once
#include "common.cuh"

namespace mt {
namespace pipe {

static constexpr long kSpinLimit = 1L << 22;

static __device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
static __device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
static __device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
static __device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps (up to
// `hint_ns`) instead of spinning, so waiting warps do not take issue slots from working ones.
static __device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, unsigned parity, unsigned hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Longest wait for one pipeline phase before a kernel gives up (its copies or its partner
// warps are stuck): far above any healthy wait, short enough to return control.
static constexpr unsigned long long kWaitDeadlineNs = 200ull * 1000 * 1000;

static __device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (long i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait_sleep(bar, parity, 2000)) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > kWaitDeadlineNs) return false;
  }
  return false;
}
static __device__ __forceinline__ void bulk_copy(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Transposed warp reduction of N (power of two <= 32) per-lane values: afterwards lane l
// holds the warp-wide sum of value index row_of<N>(l).
template <int N>
__device__ __forceinline__ float butterfly(float (&v)[N], int lane) {
  int n = N;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      const bool upper = lane & o;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        if (i < n / 2) {
          const float send = upper ? v[i] : v[i + n / 2];
          const float keep = upper ? v[i + n / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      n >>= 1;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
  return v[0];
}
template <int N>
__device__ __forceinline__ int row_of(int lane) {
  int r = 0, n = N;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      r = r * 2 + ((lane & o) ? 1 : 0);
      n >>= 1;
    }
  }
  return r;
}


static __device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
static __device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

}  // namespace pipe
}  // namespace mt
