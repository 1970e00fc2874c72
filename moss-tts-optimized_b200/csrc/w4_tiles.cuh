// Packed W4 slice blocks of the batch-1 tensor-core GEMV (sm_100a): geometry of the packed
// layout (written by mt_w4a16_pack) and the consumer-side dequantise-and-dot of one block,
// shared by the one-projection kernel (w4a16_stream.cu) and the persistent decode-step kernel
// (decode_persistent.cu). The layout and the arithmetic are described in w4a16_stream.cu.
#pragma once
#include <cuda_fp16.h>

#include "stream_pipeline.cuh"

namespace mt {

constexpr int kSliceCols = 256;   // input columns per slice block
constexpr int kSliceMax = 64;     // slices of the largest K (16384)
constexpr int kCodeBytes = 2048;  // 16 rows x 128 bytes
constexpr int kScaleBytes = 256;  // 16 rows x 8 groups x bf16
constexpr int kZeroBytes = 64;    // 16 rows x 8 groups x 4 bits

struct PackGeom {
  int n_out, rt, tiles, slices, block_b;
  long long blocks;
  PackGeom(int n, int k, bool zeros, bool paired) {
    n_out = paired ? n / 2 : n;
    rt = paired ? 8 : 16;
    tiles = (n_out + rt - 1) / rt;
    slices = k / kSliceCols;
    block_b = kCodeBytes + kScaleBytes + (zeros ? kZeroBytes : 0);
    blocks = (long long)tiles * slices;
  }
  size_t packed_bytes() const { return (size_t)blocks * block_b; }
  static constexpr int kMaxCtas = 1024;  // workspace capacity: one slot per CTA boundary
  static constexpr int kSlotFloats = 32;  // per slot side: 16 tile rows x up to 2 activation rows
  static size_t workspace_bytes() { return (size_t)kMaxCtas * (2 * kSlotFloats * sizeof(float) + sizeof(int)); }
};

// Weight row held at tile row tr (0..15) of tile t, or -1 for padding past the last row.
__host__ __device__ inline long long tile_row(int t, int tr, int n_out, bool paired) {
  if (paired) {
    const int o = t * 8 + (tr & 7);
    return o < n_out ? (long long)o + (tr >= 8 ? n_out : 0) : -1;
  }
  const int o = t * 16 + tr;
  return o < n_out ? o : -1;
}

// Codes as fp16 subnormals: (w & 0x000F000F) is the fp16 pair (q_j, q_{j+4}) * 2^-24 and
// (w & 0x00F000F0) the pair 16 (q_{j+1}, q_{j+5}) * 2^-24, exactly (the tensor cores keep
// fp16 subnormal operands). The matching activation slots carry x c and x c / 16.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// y row of tile row pair (gate = v, up = u) or plain row v (kernels.py / dp4a_packing.py:86-89).
template <bool PAIRED>
__device__ __forceinline__ float finish_row(float v, float u) {
  if (!PAIRED) return v;
  const float gate = round_bf16(v), up = round_bf16(u);
  return round_bf16(gate / (1.0f + expf(-gate))) * up;
}

// Consumer-side dot product of one slice block (16 rows x 256 columns) against the B
// fragments of its slice: returns the block's contribution to rows r (va) and r + 8 (vb),
// already summed over the lane quad (lanes with c == 0 hold the row totals).
struct BlockRegs {
  uint4 c0, c1, c2, c3;  // codes: row r (c0, c1) and row r + 8 (c2, c3)
  uint2 sw;              // scales: (s[r][2c], s[r][2c+1]) | (s[r+8][2c], s[r+8][2c+1])
  uint32_t zz;           // zero points: groups 2c | 2c+1 of row r (low byte) and r + 8
};

__device__ __forceinline__ BlockRegs load_block(const uint8_t* blk, int lane, bool zeros) {
  BlockRegs b;
  b.c0 = *reinterpret_cast<const uint4*>(blk + lane * 16);
  b.c1 = *reinterpret_cast<const uint4*>(blk + 512 + lane * 16);
  b.c2 = *reinterpret_cast<const uint4*>(blk + 1024 + lane * 16);
  b.c3 = *reinterpret_cast<const uint4*>(blk + 1536 + lane * 16);
  b.sw = *reinterpret_cast<const uint2*>(blk + kCodeBytes + lane * 8);
  b.zz = zeros ? (uint32_t)*reinterpret_cast<const uint16_t*>(blk + kCodeBytes + kScaleBytes + lane * 2) : 0x8888u;
  return b;
}

// NACC independent accumulators: the 17 mma of a block form NACC dependency chains (mma.sync
// has a long latency; the chains let one warp keep several in flight).
template <int NACC = 2>
__device__ __forceinline__ void block_dot(const BlockRegs& bk, const uint32_t (&bl)[16], const uint32_t (&bh)[16],
                                          uint32_t bz0, uint32_t bz1, float& va, float& vb) {
  const uint32_t wa[8] = {bk.c0.x, bk.c0.y, bk.c0.z, bk.c0.w, bk.c1.x, bk.c1.y, bk.c1.z, bk.c1.w};
  const uint32_t wb[8] = {bk.c2.x, bk.c2.y, bk.c2.z, bk.c2.w, bk.c3.x, bk.c3.y, bk.c3.z, bk.c3.w};
  float d[NACC][4] = {};
  // zero points: A = (z[r][2c], 16 z[r][2c+1]) (and row r + 8) as fp16 subnormals against
  // B = -(c sum x) of groups 2c / 2c + 1 split into fp16 hi and lo parts
  const uint32_t za = __byte_perm(bk.zz, 0, 0x4040) & 0x00F0000Fu, zb = __byte_perm(bk.zz, 0, 0x4141) & 0x00F0000Fu;
  mma_f16(d[NACC - 1], za, zb, za, zb, bz0, bz1);
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const uint32_t* bsel = u < 4 ? bl : bh;
    const int bi = (u & 3) * 4;
    const uint32_t sa = wa[u] >> 8, sb = wb[u] >> 8;
    mma_f16(d[(2 * u) % NACC], wa[u] & 0x000F000Fu, wb[u] & 0x000F000Fu, wa[u] & 0x00F000F0u, wb[u] & 0x00F000F0u,
            bsel[bi], bsel[bi + 1]);
    mma_f16(d[(2 * u + 1) % NACC], sa & 0x000F000Fu, sb & 0x000F000Fu, sa & 0x00F000F0u, sb & 0x00F000F0u,
            bsel[bi + 2], bsel[bi + 3]);
  }
#pragma unroll
  for (int i = 1; i < NACC; ++i) {
    d[0][0] += d[i][0];
    d[0][1] += d[i][1];
    d[0][2] += d[i][2];
    d[0][3] += d[i][3];
  }
  // column 2c = group 2c (element 0: row r, element 2: row r + 8), column 2c + 1 = group 2c + 1
  va = fmaf(__uint_as_float(bk.sw.x & 0xFFFF0000u), d[0][1], __uint_as_float(bk.sw.x << 16) * d[0][0]);
  vb = fmaf(__uint_as_float(bk.sw.y & 0xFFFF0000u), d[0][3], __uint_as_float(bk.sw.y << 16) * d[0][2]);
  va += __shfl_xor_sync(0xffffffffu, va, 1);
  vb += __shfl_xor_sync(0xffffffffu, vb, 1);
  va += __shfl_xor_sync(0xffffffffu, va, 2);
  vb += __shfl_xor_sync(0xffffffffu, vb, 2);
}

// Two activation rows per mma: the one-row B operand uses only column 2c + h of k-slot c (group
// 2c + h); with one accumulator per group instead (group 2c: mmas 0-7, group 2c + 1: mmas 8-15)
// column 2c + b of k-slot c can carry activation row b. The zero-point mma runs once per
// accumulator, its B holding -(c_b sum x_b) of that group only. Returns, summed over the lane
// quad, rows r (va[b]) and r + 8 (vb[b]) of activation rows b = 0, 1.
__device__ __forceinline__ void block_dot_rows2(const BlockRegs& bk, const uint32_t (&bl)[16], const uint32_t (&bh)[16],
                                                uint32_t bzl0, uint32_t bzl1, uint32_t bzh0, uint32_t bzh1,
                                                float (&va)[2], float (&vb)[2]) {
  const uint32_t wa[8] = {bk.c0.x, bk.c0.y, bk.c0.z, bk.c0.w, bk.c1.x, bk.c1.y, bk.c1.z, bk.c1.w};
  const uint32_t wb[8] = {bk.c2.x, bk.c2.y, bk.c2.z, bk.c2.w, bk.c3.x, bk.c3.y, bk.c3.z, bk.c3.w};
  float dl[4] = {}, dh[4] = {};
  const uint32_t za = __byte_perm(bk.zz, 0, 0x4040) & 0x00F0000Fu, zb = __byte_perm(bk.zz, 0, 0x4141) & 0x00F0000Fu;
  mma_f16(dl, za, zb, za, zb, bzl0, bzl1);
  mma_f16(dh, za, zb, za, zb, bzh0, bzh1);
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    float (&d)[4] = u < 4 ? dl : dh;
    const uint32_t* bsel = u < 4 ? bl : bh;
    const int bi = (u & 3) * 4;
    const uint32_t sa = wa[u] >> 8, sb = wb[u] >> 8;
    mma_f16(d, wa[u] & 0x000F000Fu, wb[u] & 0x000F000Fu, wa[u] & 0x00F000F0u, wb[u] & 0x00F000F0u, bsel[bi],
            bsel[bi + 1]);
    mma_f16(d, sa & 0x000F000Fu, sb & 0x000F000Fu, sa & 0x00F000F0u, sb & 0x00F000F0u, bsel[bi + 2], bsel[bi + 3]);
  }
  // element 0 / 1: row r, activation row 0 / 1; element 2 / 3: row r + 8
  const float sl_a = __uint_as_float(bk.sw.x << 16), sh_a = __uint_as_float(bk.sw.x & 0xFFFF0000u);
  const float sl_b = __uint_as_float(bk.sw.y << 16), sh_b = __uint_as_float(bk.sw.y & 0xFFFF0000u);
  va[0] = fmaf(sh_a, dh[0], sl_a * dl[0]);
  va[1] = fmaf(sh_a, dh[1], sl_a * dl[1]);
  vb[0] = fmaf(sh_b, dh[2], sl_b * dl[2]);
  vb[1] = fmaf(sh_b, dh[3], sl_b * dl[3]);
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    va[0] += __shfl_xor_sync(0xffffffffu, va[0], o);
    va[1] += __shfl_xor_sync(0xffffffffu, va[1], o);
    vb[0] += __shfl_xor_sync(0xffffffffu, vb[0], o);
    vb[1] += __shfl_xor_sync(0xffffffffu, vb[1], o);
  }
}

constexpr int kWarps = 16;  // consumer warps per CTA

}  // namespace mt
