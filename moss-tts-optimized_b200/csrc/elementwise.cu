// Small decode-step operators for B200 (sm_100a): RMSNorm, add + RMSNorm,
// SiLU * up and the 33-channel embedding sum, plus library-wide helpers.
// Rounding points follow src/moss_tts/_runtime/kernels.py exactly (cited per kernel).
#include "common.cuh"

namespace mt {

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// One CTA per row. RMSNorm (kernels.py:50-59) or add + RMSNorm (kernels.py:69-90).
__global__ void __launch_bounds__(256) rmsnorm_rows(const __nv_bfloat16* __restrict__ x,
                                                    const __nv_bfloat16* __restrict__ residual,
                                                    const __nv_bfloat16* __restrict__ w,
                                                    __nv_bfloat16* __restrict__ summed,
                                                    __nv_bfloat16* __restrict__ y, int n, float eps) {
  extern __shared__ float buf[];
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const __nv_bfloat16* xr = x + (size_t)row * n;
  float ss = 0.f;
  for (int i = tid; i < n; i += blockDim.x) {
    float v = bf16f(xr[i]);
    if (residual) {
      v = round_bf16(v + bf16f(residual[(size_t)row * n + i]));
      if (summed) summed[(size_t)row * n + i] = to_bf16(v);
    }
    buf[i] = v;
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / (float)n + eps);
  for (int i = tid; i < n; i += blockDim.x)
    y[(size_t)row * n + i] = to_bf16(round_bf16(buf[i] * inv) * bf16f(w[i]));
}

// The same for rows of n % 8 == 0 elements (<= 256 * 8 * J): every thread issues all of its
// 16-byte loads up front (x and residual) and keeps the row in registers, so a row costs one
// memory round trip instead of one per element sweep.
template <int J>
__global__ void __launch_bounds__(256) rmsnorm_rows_v8(const __nv_bfloat16* __restrict__ x,
                                                       const __nv_bfloat16* __restrict__ residual,
                                                       const __nv_bfloat16* __restrict__ w,
                                                       __nv_bfloat16* __restrict__ summed,
                                                       __nv_bfloat16* __restrict__ y, int n, float eps) {
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x, E = n >> 3;
  pdl_wait();
  pdl_trigger();
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * n);
  const uint4* rr = residual ? reinterpret_cast<const uint4*>(residual + (size_t)row * n) : nullptr;
  uint4 xv[J], rv[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int e = tid + 256 * j;
    xv[j] = e < E ? xr[e] : make_uint4(0, 0, 0, 0);
    rv[j] = (rr && e < E) ? rr[e] : make_uint4(0, 0, 0, 0);
  }
  float v[J][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const uint32_t xw[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w}, rw[4] = {rv[j].x, rv[j].y, rv[j].z, rv[j].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[j][2 * i] = bf16_lo(xw[i]);
      v[j][2 * i + 1] = bf16_hi(xw[i]);
      if (residual) {
        v[j][2 * i] = round_bf16(v[j][2 * i] + bf16_lo(rw[i]));
        v[j][2 * i + 1] = round_bf16(v[j][2 * i + 1] + bf16_hi(rw[i]));
      }
      ss += v[j][2 * i] * v[j][2 * i] + v[j][2 * i + 1] * v[j][2 * i + 1];
    }
    const int e = tid + 256 * j;
    if (residual && summed && e < E) {
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 p = __floats2bfloat162_rn(v[j][2 * i], v[j][2 * i + 1]);
        o[i] = *reinterpret_cast<uint32_t*>(&p);
      }
      reinterpret_cast<uint4*>(summed + (size_t)row * n)[e] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / (float)n + eps);
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int e = tid + 256 * j;
    if (e >= E) continue;
    const uint4 wv = reinterpret_cast<const uint4*>(w)[e];
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a0 = round_bf16(round_bf16(v[j][2 * i] * inv) * bf16_lo(ww[i]));
      const float a1 = round_bf16(round_bf16(v[j][2 * i + 1] * inv) * bf16_hi(ww[i]));
      __nv_bfloat162 p = __floats2bfloat162_rn(a0, a1);
      o[i] = *reinterpret_cast<uint32_t*>(&p);
    }
    reinterpret_cast<uint4*>(y + (size_t)row * n)[e] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Device-side advance of `batch` decode steps (first_audio_graph._advance,
// src/moss_tts/_runtime/first_audio_graph.py:14-27): control int64 [ids batch*n_ids | positions
// batch | audio_length batch | delay_length batch] takes next_ids [batch, n_ids] as its ids,
// positions and audio lengths advance by one, and a sequence whose text token is the delay slot
// starts its delay count, which then advances by one per step.
__global__ void __launch_bounds__(256) decode_advance(int64_t* __restrict__ control,
                                                      const int64_t* __restrict__ next_ids, int n_ids, int batch,
                                                      int delay_slot_id) {
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x;
  for (int i = tid; i < batch * n_ids; i += blockDim.x) control[i] = next_ids[i];
  for (int b = tid; b < batch; b += blockDim.x) {
    int64_t* pos = control + (size_t)batch * n_ids;
    pos[b] += 1;                       // position
    pos[batch + b] += 1;               // audio_length
    int64_t d = pos[2 * batch + b];    // delay_length
    if (d < 0 && next_ids[(size_t)b * n_ids] == delay_slot_id) d = 0;
    if (d >= 0) d += 1;
    pos[2 * batch + b] = d;
  }
}

// SiLU(gate) rounded to bf16, times up (kernels.py:123-139); x is [rows, 2n].
__global__ void silu_mul_rows(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                              int rows, int n) {
  pdl_wait();
  pdl_trigger();
  const size_t total = (size_t)rows * n;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / n, c = i - r * n;
    const float g = bf16f(x[r * 2 * n + c]), u = bf16f(x[r * 2 * n + n + c]);
    y[i] = to_bf16(round_bf16(g / (1.0f + expf(-g))) * u);
  }
}

// The same for n % 8 == 0 and 16-byte aligned rows: one thread per 8 outputs (16-byte loads
// of the gate and up halves, one 16-byte store), rows split in n / 8 chunks.
__global__ void silu_mul_rows_v8(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int rows,
                                 int n) {
  pdl_wait();
  pdl_trigger();
  const int chunks = n / 8;
  const size_t total = (size_t)rows * chunks;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / chunks, c = (i - r * chunks) * 8;
    const uint4 gw = *reinterpret_cast<const uint4*>(x + r * 2 * n + c);
    const uint4 uw = *reinterpret_cast<const uint4*>(x + r * 2 * n + n + c);
    const uint32_t ga[4] = {gw.x, gw.y, gw.z, gw.w}, ua[4] = {uw.x, uw.y, uw.z, uw.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g0 = bf16_lo(ga[k]), g1 = bf16_hi(ga[k]);
      __nv_bfloat162 pr = __floats2bfloat162_rn(round_bf16(g0 / (1.0f + expf(-g0))) * bf16_lo(ua[k]),
                                                round_bf16(g1 / (1.0f + expf(-g1))) * bf16_hi(ua[k]));
      o[k] = *reinterpret_cast<uint32_t*>(&pr);
    }
    *reinterpret_cast<uint4*>(y + r * n + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Text embedding plus the n_vq audio embeddings with a bf16 rounding after every
// sequential addition (kernels.py:7-26). Each thread owns 8 hidden dims; the rows it
// adds are fetched in batches ahead of the (order-preserving) additions.
constexpr int kEmbBatch = 11;

__device__ __forceinline__ int64_t clamp_id(int64_t c, int limit, int* status) {
  if (c < 0 || c >= limit) {  // never read outside the table
    if (status) atomicExch(status, 2);
    return 0;
  }
  return c;
}

__global__ void __launch_bounds__(64) embedding_sum_rows(const int64_t* __restrict__ ids,
                                                         const __nv_bfloat16* __restrict__ text,
                                                         const __nv_bfloat16* __restrict__ audio,
                                                         __nv_bfloat16* __restrict__ out, int h, int vocab,
                                                         int audio_vocab, int n_vq, int* status) {
  const int t = blockIdx.y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;  // 8-element slot
  pdl_wait();
  pdl_trigger();
  if (e * 8 >= h) return;
  const int64_t* row = ids + (size_t)t * (n_vq + 1);
  const int64_t tok = clamp_id(row[0], vocab, status);
  const uint4 tv = *reinterpret_cast<const uint4*>(text + (size_t)tok * h + 8 * e);
  float v[8];
  const uint32_t tw[4] = {tv.x, tv.y, tv.z, tv.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) { v[2 * i] = bf16_lo(tw[i]); v[2 * i + 1] = bf16_hi(tw[i]); }
  for (int q0 = 0; q0 < n_vq; q0 += kEmbBatch) {
    uint4 rows[kEmbBatch];
#pragma unroll
    for (int j = 0; j < kEmbBatch; ++j) {
      const int q = q0 + j;
      if (q < n_vq) {
        const int64_t c = clamp_id(row[q + 1], audio_vocab, status);
        rows[j] = *reinterpret_cast<const uint4*>(audio + ((size_t)q * audio_vocab + c) * h + 8 * e);
      }
    }
#pragma unroll
    for (int j = 0; j < kEmbBatch; ++j) {
      if (q0 + j < n_vq) {
        const uint32_t aw[4] = {rows[j].x, rows[j].y, rows[j].z, rows[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[2 * i] = round_bf16(v[2 * i] + bf16_lo(aw[i]));
          v[2 * i + 1] = round_bf16(v[2 * i + 1] + bf16_hi(aw[i]));
        }
      }
    }
  }
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    o[i] = *reinterpret_cast<uint32_t*>(&p);
  }
  *reinterpret_cast<uint4*>(out + (size_t)t * h + 8 * e) = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace mt

using namespace mt;

MT_API int mt_abi_version(void) { return 1; }

// rmsnorm(x, weight, eps) (src/moss_tts/_runtime/kernels.py:62) when residual is null;
// add_rmsnorm(x, residual, weight, eps) -> (summed, normalized) (kernels.py:85) otherwise.
MT_API int mt_rmsnorm(const void* x, const void* residual, const void* weight, void* summed, void* y,
                      int rows, int n, float eps, int flags, void* stream) {
  if (!x || !weight || !y || rows < 1 || n < 1 || n > 16384) return kBadArgument;
  const bool vec = n % 8 == 0 && aligned(x, 16) && aligned(weight, 16) && aligned(y, 16) &&
                   (!residual || aligned(residual, 16)) && (!summed || aligned(summed, 16));
  if (vec) {
    auto k = n <= 256 * 8 * 2 ? rmsnorm_rows_v8<2> : rmsnorm_rows_v8<8>;
    return launch(k, dim3(rows), dim3(256), 0, (cudaStream_t)stream, flags, (const __nv_bfloat16*)x,
                  (const __nv_bfloat16*)residual, (const __nv_bfloat16*)weight, (__nv_bfloat16*)summed,
                  (__nv_bfloat16*)y, n, eps);
  }
  return launch(rmsnorm_rows, dim3(rows), dim3(256), (size_t)n * 4, (cudaStream_t)stream, flags,
                (const __nv_bfloat16*)x, (const __nv_bfloat16*)residual, (const __nv_bfloat16*)weight,
                (__nv_bfloat16*)summed, (__nv_bfloat16*)y, n, eps);
}

// silu_mul(x) (src/moss_tts/_runtime/kernels.py:132): x [rows, 2n] -> y [rows, n].
MT_API int mt_silu_mul(const void* x, void* y, int rows, int n, int flags, void* stream) {
  if (!x || !y || rows < 1 || n < 1) return kBadArgument;
  const size_t cap = (size_t)sm_count() * 8;
  if (n % 8 == 0 && aligned(x, 16) && aligned(y, 16)) {
    size_t blocks = ((size_t)rows * (n / 8) + 255) / 256;
    if (blocks > cap) blocks = cap;
    return launch(silu_mul_rows_v8, dim3((unsigned)blocks), dim3(256), 0, (cudaStream_t)stream, flags,
                  (const __nv_bfloat16*)x, (__nv_bfloat16*)y, rows, n);
  }
  const size_t total = (size_t)rows * n;
  size_t blocks = (total + 255) / 256;
  if (blocks > cap) blocks = cap;
  return launch(silu_mul_rows, dim3((unsigned)blocks), dim3(256), 0, (cudaStream_t)stream, flags,
                (const __nv_bfloat16*)x, (__nv_bfloat16*)y, rows, n);
}

// embedding_sum(ids, text_weight, audio_weight) (src/moss_tts/_runtime/kernels.py:21):
// ids int64 [tokens, 1 + n_vq], text [vocab, h], audio [n_vq, audio_vocab, h] -> out [tokens, h].
MT_API int mt_embedding_sum(const void* ids, const void* text, const void* audio, void* out,
                            int tokens, int h, int vocab, int audio_vocab, int n_vq, void* status,
                            int flags, void* stream) {
  if (!ids || !text || !audio || !out || tokens < 1 || h < 8 || h % 8 || vocab < 1 ||
      audio_vocab < 1 || n_vq < 0)
    return kBadArgument;
  if (!aligned(text, 16) || !aligned(audio, 16) || !aligned(out, 16) || !aligned(ids, 8))
    return kBadArgument;
  const dim3 grid((h / 8 + 63) / 64, tokens);
  return launch(embedding_sum_rows, grid, dim3(64), 0, (cudaStream_t)stream, flags,
                (const int64_t*)ids, (const __nv_bfloat16*)text, (const __nv_bfloat16*)audio,
                (__nv_bfloat16*)out, h, vocab, audio_vocab, n_vq, (int*)status);
}

// Device-side state advance after a decode step, for `batch` sequences (one launch instead of
// the reference's handful of tensor operations in first_audio_graph._advance,
// src/moss_tts/_runtime/first_audio_graph.py:14-27). control int64
// [ids batch*n_ids | positions batch | audio_length batch | delay_length batch].
MT_API int mt_decode_advance(void* control, const void* next_ids, int n_ids, int batch, int delay_slot_id,
                             int flags, void* stream) {
  if (!control || !next_ids || n_ids < 1 || batch < 1 || batch > 65536) return kBadArgument;
  return launch(decode_advance, dim3(1), dim3(256), 0, (cudaStream_t)stream, flags, (int64_t*)control,
                (const int64_t*)next_ids, n_ids, batch, delay_slot_id);
}
