// W4A16 G32 skinny GEMM on the fifth-generation tensor cores (sm_100a): the batched decode
// projections y[B, N] = x[B, K] . W^T, B = 9..128, with W = bf16((q - z) * s), the
// reference's dequantize-then-matmul (src/moss_tts/_runtime/calibrated_quant.py:41-42 and
// the projection of dp4a_packing.py:94-125), with fp32 accumulation; optional fused gate/up
// pair with bf16(silu(bf16 gate)) * bf16 up (fused_mlp.py:18-23).
//
// Batch-1..8 decode streams weights far below the tensor-core crossover and stays on the
// CUDA-core / mma.sync GEMV kernels; at B >= 16 one weight byte feeds 4B multiply-adds and
// only tcgen05 keeps the dequantised stream fed at HBM speed. Design:
//
// * A tile is 128 weight rows (the 128 TMEM lanes). One persistent CTA per SM owns a
//   balanced contiguous range of the (tile, 256-wide K chunk) work list, so every SM streams
//   the same number of weight bytes; a range cuts at most two tiles (its first and last).
// * Two loader warps fill two shared-memory rings with TMA loads: the code ring holds the
//   chunk's 4-bit codes (128 rows x 128 bytes, 128-byte swizzle), scales and zero points and
//   is released by the dequantisation group as soon as it has read them; the activation ring
//   holds the activation chunk (B x 256 bf16 in four 64-column boxes with the 128-byte
//   swizzle: the canonical K-major SWIZZLE_128B operand layout; rows past B read as zeros) and
//   is released by the MMAs. Separate rings keep up to eight code chunks in flight even when
//   the activation chunks are large (32 KB at B = 64). The code loads do not depend on the
//   previous kernel and start before griddepcontrol.wait.
// * The dequantised weights never touch shared memory: sixteen dequantisation warps in two
//   groups taking alternate chunks (so one group computes while the other waits; in a group
//   warp w owns TMEM lanes 32 (w % 4) .. +31, one weight row per thread, and one half of the
//   chunk's K) read their row's codes from the stage (conflict-free thanks to the swizzle), their
//   scales and zero points from L1-cached loads issued three chunks ahead, turn each code pair
//   into an exact bf16 pair (bf16(128 + q) by bit insertion, minus bf16(128 + z) exactly,
//   times the bf16 scale with one round to nearest: the oracle's bf16((q - z) * s) bit for
//   bit) and store them into one of two or three TMEM slots with tcgen05.st; each K half of a
//   slot has its own full / empty barrier pair, so the two MMA warps run independently.
// * Two MMA warps issue tcgen05.mma.kind::f16 with A in TMEM and B in shared memory: warp i
//   the 8 K steps of half i of every chunk, into its own fp32 accumulator D_i[128, B] in TMEM
//   (one thread issues at most one MMA per ~70 cycles whatever N, so a single issuer paced
//   the kernel at small batches). Up to 32 batch columns each warp double-buffers its
//   accumulator per tile segment. tcgen05.commit frees the TMEM slot half and the activation
//   stage and hands finished accumulators to four epilogue warps, which read D_0 + D_1 with
//   tcgen05.ld.
// * A tile cut between CTAs is finished by the last contributor (ticket), which sums the
//   contributions in CTA order, so results are deterministic.
// Every mbarrier wait is bounded; an expired wait sets an error word and the kernel still
// drains, releases its TMEM and returns.
#include <cuda.h>
#include <string.h>
#include <cudaTypedefs.h>

#include "stream_pipeline.cuh"

namespace mt {

__device__ int g_gemm_error;  // set when a bounded wait expired (read through mt_read_error_word)

namespace tc {

using namespace pipe;

constexpr int kTileM = 128;        // weight rows per tile = TMEM lanes
constexpr int kChunk = 256;        // K elements per pipeline stage
constexpr int kMaxSlots = 3;       // TMEM A slots (3 when the batch fits 64 columns, else 2)
constexpr int kMaxStages = 8;      // shared-memory stages per ring (codes; activations)
constexpr int kDequantWarps = 16;  // two groups of 8 (alternate chunks); lane quarter w % 4, K half (w / 4) % 2
constexpr int kMmaWarp = 16;       // warps 16 and 17 issue the MMAs of K halves 0 and 1
constexpr int kMmaWarps = 2;
constexpr int kEpiWarp0 = 18;      // warps 18..21 read the accumulators
constexpr int kCodeWarp = 22;      // TMA loads of the 4-bit codes
constexpr int kActWarp = 23;       // TMA loads of the activation chunks
constexpr int kThreads = 24 * 32;
constexpr int kMaxBatch = 128;
constexpr int kMaxTiles = 4096;    // 128-row tiles per projection (n <= 524288)
constexpr int kSlotCols = kChunk / 2;  // TMEM columns of one A slot (two bf16 per column)
constexpr uint32_t kCodeBytes = kTileM * kChunk / 2;  // codes of one chunk of one tile
constexpr uint32_t kScaleOff = kCodeBytes;            // [128 rows][8 bf16 scales]
constexpr uint32_t kZeroOff = kScaleOff + kTileM * 16;  // [128 rows][16 zero-point bytes (4 chunks)]
constexpr uint32_t kXOff = kZeroOff + kTileM * 16;      // activation boxes (1024-byte aligned)
// Packed layout (mt_w4a16_gemm_pack): one contiguous block per (tile, K chunk), tile-major, so a
// CTA's work range is one contiguous byte range and each stage is one bulk copy.
constexpr uint32_t kPackedZeroOff = kScaleOff + kTileM * 16;  // [128 rows][4 zero-point bytes]
constexpr uint32_t kPackedBlock = kPackedZeroOff + kTileM * 4;  // 18,944 bytes
constexpr uint32_t kPackedXOff = (kPackedBlock + 1023) / 1024 * 1024;
constexpr int kTmemCols = 512;

struct GemmArgs {
  const __nv_bfloat16* x;        // [batch, K]
  const uint8_t* qweight;        // [N, K/2]
  const __nv_bfloat16* scales;   // [N, K/32]
  const uint8_t* qzeros;         // [N, K/64] or null (z = 8)
  __nv_bfloat16* y;              // [batch, N] or [batch, N/2] (paired)
  float* partial;                // [2 * grid][batch][128] contributions to cut tiles
  unsigned* tickets;             // [tiles], zero on entry and exit
  int batch, n, k, n_mma, tiles, chunks, cstages, xstages;  // code and activation ring stages
  int zt;             // zero points arrive by TMA with the codes ((k / 64) % 16 == 0), else per thread
  const uint8_t* packed;  // packed layout: [tiles * chunks][kPackedBlock] (PACKED kernels)
  int d_cols, nbuf, slots;  // accumulator columns (32, 64 or 128), buffers per MMA warp, TMEM A slots
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// One lane of a converged warp (PTX elect.sync): the issuing lane of a warp-uniform loop.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(pred));
  return pred != 0;
}
// Bounded wait for a phase that is usually far off: back off between polls so that waiting
// warps leave the issue slots to the dequantisation warps.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t* bar, unsigned parity) {
  for (long i = 0; i < (1L << 22); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(64);
  }
  return false;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// D[128, N] (+)= A[128, 16] (TMEM) . B[N, 16]^T (shared memory descriptor), bf16 in, fp32 out.
__device__ __forceinline__ void mma_ts(uint32_t d_taddr, uint32_t a_taddr, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n}" ::"r"(d_taddr),
      "r"(a_taddr), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8 rows x 16 bytes;
// `lbo` = byte distance between the two K-adjacent core matrices of one K=16 step, `sbo` =
// byte distance between 8-row groups; bit 46 = descriptor version of sm_100.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
// K-major, 128-byte swizzle (layout type 2): rows of 64 bf16 (128 bytes), 8-row atoms of
// 1024 bytes at a stride of 1024; a K=16 step inside the atom advances the start by 32 bytes.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return smem_desc(addr, 16, 1024) | (2ull << 61);
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

struct RowLoads {
  uint32_t z;     // two zero-point bytes (low nibble first), when they do not arrive by TMA
};

__device__ __forceinline__ int range_start(int b, long work, int ctas) { return (int)((long)b * work / ctas); }
// The CTA whose work range holds item w.
__device__ __forceinline__ int owner_of(int w, long work, int ctas) {
  int b = (int)((long)w * ctas / work);
  while (b + 1 < ctas && range_start(b + 1, work, ctas) <= w) ++b;
  while (b > 0 && range_start(b, work, ctas) > w) --b;
  return b;
}

template <bool PAIRED, bool PACKED>
__global__ void __launch_bounds__(kThreads, 1)
    w4a16_gemm_tc(GemmArgs a, const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                  const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap zmap) {
  // dynamic shared memory, from the first 1024-byte boundary: [cstages] x codes [128][128 B]
  // (128-byte swizzle) with scales and zero points, [xstages] x activations [4][n_mma][64]
  // bf16 (128-byte swizzle), then [16][64] f32 for the paired epilogue
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[2][kMaxSlots];    // K half of a dequantised chunk in TMEM slot
  __shared__ __align__(8) uint64_t aempty[2][kMaxSlots];  // that half's MMAs done with the TMEM slot
  __shared__ __align__(8) uint64_t wfull[kMaxStages];   // codes landed
  __shared__ __align__(8) uint64_t cempty[kMaxStages];  // dequantisation group done with the codes
  __shared__ __align__(8) uint64_t xfull[kMaxStages];   // activations landed
  __shared__ __align__(8) uint64_t xempty[kMaxStages];  // MMAs done with the activations
  __shared__ __align__(8) uint64_t dfull[2];
  __shared__ __align__(8) uint64_t dfree[2];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;
  __shared__ unsigned last_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = a.k, n_mma = a.n_mma, B = a.batch, chunks = a.chunks, ctas = gridDim.x;
  const int ncs = a.cstages, nxs = a.xstages;
  const int n_out = PAIRED ? a.n / 2 : a.n;
  const long work = (long)a.tiles * chunks;
  const int w0 = range_start(blockIdx.x, work, ctas), w1 = range_start(blockIdx.x + 1, work, ctas);
  const int nwork = w1 - w0;
  const int t_first = w0 / chunks;
  const int nseg = nwork > 0 ? (w1 - 1) / chunks - t_first + 1 : 0;
  const int nslot = a.slots, nbuf = a.nbuf, a_col0 = kMmaWarps * nbuf * a.d_cols;
  const uint32_t x_bytes = (uint32_t)n_mma * kChunk * 2, x_box = (uint32_t)n_mma * 128;  // 64-column boxes
  constexpr uint32_t kCodeStage = PACKED ? kPackedXOff : kXOff;  // 1024-byte multiples
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* xring = smem + (size_t)ncs * kCodeStage;
  float* exch = reinterpret_cast<float*>(xring + (size_t)nxs * x_bytes);

  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    if (lane == 0) {
      for (int i = 0; i < kMaxSlots; ++i)
        for (int hh = 0; hh < 2; ++hh) {
          mbar_init(&full[hh][i], kDequantWarps / 4 * 32);  // the lanes of one K half of a group
          mbar_init(&aempty[hh][i], 1);
        }
      for (int i = 0; i < kMaxStages; ++i) {
        mbar_init(&wfull[i], 1);
        mbar_init(&cempty[i], kDequantWarps / 2 * 32);
        mbar_init(&xfull[i], 1);
        mbar_init(&xempty[i], kMmaWarps);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&dfull[i], kMmaWarps);
        mbar_init(&dfree[i], 128);
      }
      abort_s = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;
  pdl_trigger();

  if (warp < kDequantWarps) {
    // Two groups of eight warps take alternate chunks (group g: chunks g, g + 2, ...), so one
    // group dequantises while the other waits on its barriers; in a group, warp w covers TMEM
    // lane quarter w % 4 (one weight row per thread) and half (w / 4) % 2 of the chunk's K.
    const int q = warp & 3, h = (warp >> 2) & 1, grp = warp >> 3, m = 32 * q + lane;
    // scales and zero points: L1-cached loads two of the group's chunks ahead
    auto load = [&](int j, RowLoads& r) {
      if (j < nwork) {
        const int w = w0 + j, tile = w / chunks, c = w - tile * chunks;
        const int row = PAIRED ? (m < 64 ? tile * 64 + m : n_out + tile * 64 + (m - 64)) : tile * kTileM + m;
        if (!PACKED && a.qzeros && !a.zt)
          r.z = (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(a.qzeros + (size_t)row * (K / 64) + c * 4 + h * 2));
      }
    };
    // weights are never written by a predecessor: no dependency wait before streaming them
    const uint32_t t_lane = (uint32_t)(32 * q) << 16;
    const int sw = m & 7;  // 128-byte swizzle of row m: 16-byte piece p sits at p ^ sw
    const uint32_t code_off = (uint32_t)m * 128;

    // this group's chunks are grp, grp + 2, ...: TMEM slot and code stage of the next one, and
    // the phase parities, kept as counters (no runtime division in the loop)
    int slot = grp, spar = 0, st = grp, cpar = 0;
    auto process = [&](int j, const RowLoads& r) {
      bool ok = true;
      if (j >= nslot) {  // the MMAs of chunk j - nslot have released this TMEM slot
        ok = mbar_wait_bounded(&aempty[h][slot], (unsigned)(spar ^ 1));
        tc_fence_after();
      }
      ok = mbar_wait_bounded(&wfull[st], (unsigned)cpar) && ok;
      if (!ok) abort_s = 1;
      const uint8_t* stage = smem + st * kCodeStage;
      const uint8_t* cs = stage + code_off;
      const uint2 sc = *reinterpret_cast<const uint2*>(stage + kScaleOff + m * 16 + h * 8);
      uint32_t zpair = 0x8888u;
      if (PACKED)
        zpair = *reinterpret_cast<const uint16_t*>(stage + kPackedZeroOff + m * 4 + h * 2);
      else if (a.qzeros)
        zpair = a.zt ? (uint32_t)*reinterpret_cast<const uint16_t*>(stage + kZeroOff + m * 16 +
                                                                   (((w0 + j) % chunks) * 4 & 15) + h * 2)
                     : r.z;
      const uint32_t ta = tmem + t_lane + (uint32_t)(a_col0 + slot * kSlotCols + h * 64);
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // 64 codes -> 32 bf16 pairs, twice
        const int p0 = 4 * h + 2 * half;
        const uint4 c0 = *reinterpret_cast<const uint4*>(cs + ((p0 ^ sw) << 4));
        const uint4 c1 = *reinterpret_cast<const uint4*>(cs + (((p0 + 1) ^ sw) << 4));
        const uint32_t zb = (zpair >> (8 * half)) & 0xFF;
        const uint32_t zz0 = (0x4300u + (zb & 0xF)) * 0x10001u, zz1 = (0x4300u + (zb >> 4)) * 0x10001u;
        const uint32_t sp = half ? sc.y : sc.x;
        const uint32_t s0 = (sp & 0xFFFFu) * 0x10001u, s1 = (sp >> 16) * 0x10001u;
        const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        uint32_t v[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // code word i holds k = 8i .. 8i + 7
          const uint32_t u = cw[i];
          const uint32_t zz = i < 4 ? zz0 : zz1, ss = i < 4 ? s0 : s1;
          if (PACKED) {
            // packed words hold k = 8i + 2b in nibble b and k = 8i + 2b + 1 in nibble b + 4
            // (mt_w4a16_gemm_pack), so one shift and mask give the pair: no byte permute
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const uint32_t t = ((u >> (4 * b)) & 0x000F000Fu) | 0x43004300u;
              v[4 * i + b] = bf16x2_mul(bf16x2_sub(t, zz), ss);
            }
          } else {
            const uint32_t hi = u >> 4;  // GPTQ words: byte b holds k = 8i + 2b (low), + 1 (high)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const uint32_t t = (prmt(u, hi, 0x0400u + 0x0101u * b) & 0x000F000Fu) | 0x43004300u;
              v[4 * i + b] = bf16x2_mul(bf16x2_sub(t, zz), ss);
            }
          }
        }
        __syncwarp();
        tmem_st16(ta + 32 * half, v);
        tmem_st16(ta + 32 * half + 16, v + 16);
      }
      mbar_arrive(&cempty[st]);  // codes, scales and zero points consumed: the stage may refill
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&full[h][slot]);
      slot += 2;  // nslot, ncs >= 2: at most one wrap
      if (slot >= nslot) {
        slot -= nslot;
        spar ^= 1;
      }
      st += 2;
      if (st >= ncs) {
        st -= ncs;
        cpar ^= 1;
      }
    };
    RowLoads buf[3];
    load(grp, buf[0]);
    load(grp + 2, buf[1]);
#pragma unroll 1
    for (int j = grp; j < nwork; j += 6) {
      load(j + 4, buf[2]);
      process(j, buf[0]);
      if (j + 2 < nwork) {
        load(j + 6, buf[0]);
        process(j + 2, buf[1]);
      }
      if (j + 4 < nwork) {
        load(j + 8, buf[1]);
        process(j + 4, buf[2]);
      }
    }
  } else if (warp < kMmaWarp + kMmaWarps) {
    // MMA warp i: the 8 K steps of half i of every chunk into its own accumulator (the epilogue
    // adds the two); two issuing warps because one thread issues at most one tcgen05.mma per
    // ~70 cycles whatever N, and 16 per chunk would pace the kernel. Warp-uniform loop; one
    // elected lane issues the MMAs and commits.
    const int i = warp - kMmaWarp;
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n_mma >> 3) << 17) |
                           ((uint32_t)(kTileM >> 4) << 24);
    const uint32_t b0 = smem_u32(xring);
    // ring positions, parities and the chunk index inside the tile kept as counters
    int seg = -1, buf = 0, c = w0 % chunks, slot = 0, spar = 0, st = 0, xpar = 0;
    uint32_t d = tmem;
    for (int j = 0; j < nwork; ++j) {
      const bool first = j == 0 || c == 0, last = j == nwork - 1 || c == chunks - 1;
      if (first) {
        ++seg;
        buf = nbuf == 2 ? (seg & 1) : 0;
        if (seg >= nbuf) {  // the epilogue must have read this buffer's previous segment
          if (!mbar_wait_bounded(&dfree[buf], (unsigned)(((seg / nbuf) - 1) & 1))) abort_s = 1;
          tc_fence_after();
        }
        d = tmem + (uint32_t)((i * nbuf + buf) * a.d_cols);
      }
      const bool ok = mbar_wait_bounded(&xfull[st], (unsigned)xpar) &&
                      mbar_wait_bounded(&full[i][slot], (unsigned)spar);
      tc_fence_after();
      if (!ok) abort_s = 1;
      const uint32_t a_col = tmem + (uint32_t)(a_col0 + slot * kSlotCols);
      const uint32_t x0 = b0 + st * x_bytes;
      __syncwarp();
      if (elect_one()) {
        if (ok && !abort_s) {
#pragma unroll
          for (int u = 0; u < kChunk / 32; ++u) {
            const int kk = (kChunk / 32) * i + u;
            mma_ts(d, a_col + kk * 8, smem_desc_sw128(x0 + (kk >> 2) * x_box + (kk & 3) * 32), idesc,
                   (first && u == 0) ? 0u : 1u);
          }
        }
        mma_commit(&aempty[i][slot]);
        mma_commit(&xempty[st]);
        if (last) mma_commit(&dfull[buf]);
      }
      __syncwarp();
      if (++c == chunks) c = 0;
      if (++slot == nslot) {
        slot = 0;
        spar ^= 1;
      }
      if (++st == nxs) {
        st = 0;
        xpar ^= 1;
      }
    }
  } else if (warp == kCodeWarp || warp == kActWarp) {
    // codes (independent of the previous kernel) and activations; warp-uniform loops, one
    // elected lane issues each stage's TMA loads
    const bool codes = warp == kCodeWarp;
    if (!codes) pdl_wait();
    const int ns = codes ? ncs : nxs;
    uint64_t* empty = codes ? cempty : xempty;
    int st = 0, par = 0, tile = w0 / chunks, c = w0 - tile * chunks;  // counters, no division in the loop
    for (int j = 0; j < nwork; ++j) {
      if (j >= ns && !mbar_wait_idle(&empty[st], (unsigned)(par ^ 1))) abort_s = 1;
      const int w = w0 + j;
      const uint32_t base = codes ? smem_u32(smem) + st * kCodeStage : smem_u32(xring) + st * x_bytes;
      __syncwarp();
      if (elect_one()) {
        if (codes && PACKED) {
          mbar_expect_tx(&wfull[st], kPackedBlock);
          bulk_copy(smem + st * kCodeStage, a.packed + (size_t)w * kPackedBlock, kPackedBlock, &wfull[st]);
        } else if (codes) {
          const int r0 = PAIRED ? tile * 64 : tile * kTileM, r1 = PAIRED ? n_out + tile * 64 : r0 + 64;
          mbar_expect_tx(&wfull[st], kZeroOff + (a.zt ? kTileM * 16 : 0));
          tma_load_2d(base, &wmap, c * (kChunk / 2), r0, &wfull[st]);
          tma_load_2d(base + kCodeBytes / 2, &wmap, c * (kChunk / 2), r1, &wfull[st]);
          tma_load_2d(base + kScaleOff, &smap, c * 8, r0, &wfull[st]);
          tma_load_2d(base + kScaleOff + 64 * 16, &smap, c * 8, r1, &wfull[st]);
          if (a.zt) {
            tma_load_2d(base + kZeroOff, &zmap, (c * 4) & ~15, r0, &wfull[st]);
            tma_load_2d(base + kZeroOff + 64 * 16, &zmap, (c * 4) & ~15, r1, &wfull[st]);
          }
        } else {
          mbar_expect_tx(&xfull[st], x_bytes);
#pragma unroll
          for (int bx = 0; bx < kChunk / 64; ++bx)
            tma_load_2d(base + bx * x_box, &xmap, c * kChunk + 64 * bx, 0, &xfull[st]);
        }
      }
      __syncwarp();
      if (++st == ns) {
        st = 0;
        par ^= 1;
      }
      if (++c == chunks) {
        c = 0;
        ++tile;
      }
    }
  } else {
    // Epilogue warps: lane quarter warp % 4; e = 0..127 indexes the named barrier group.
    const int q = warp & 3, m = 32 * q + lane, e = tid - kEpiWarp0 * 32;
    const uint32_t t_lane = (uint32_t)(32 * q) << 16;
    pdl_wait();
    auto emit = [&](int tile, int cb, const float* v) {
      if (PAIRED) {  // fused_mlp.py:18-23: rows < 64 gate, rows >= 64 the matching up rows
        if (m >= 64)
#pragma unroll
          for (int t = 0; t < 16; ++t) exch[t * 64 + (m - 64)] = v[t];
        named_sync(1, 128);
        if (m < 64) {
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            if (cb + t < B) {
              const float gate = round_bf16(v[t]), up = round_bf16(exch[t * 64 + m]);
              a.y[(size_t)(cb + t) * n_out + tile * 64 + m] = to_bf16(round_bf16(gate / (1.0f + expf(-gate))) * up);
            }
          }
        }
        named_sync(1, 128);
      } else {
#pragma unroll
        for (int t = 0; t < 16; ++t)
          if (cb + t < B) a.y[(size_t)(cb + t) * n_out + tile * kTileM + m] = to_bf16(v[t]);
      }
    };
    for (int s = 0; s < nseg; ++s) {
      const int tile = t_first + s;
      const int ca = max(w0, tile * chunks) - tile * chunks, ce = min(w1, (tile + 1) * chunks) - tile * chunks;
      const bool whole = ca == 0 && ce == chunks;
      if (!mbar_wait_idle(&dfull[s % nbuf], (unsigned)((s / nbuf) & 1))) abort_s = 1;
      tc_fence_after();
      // the two MMA warps' accumulators of this segment (K halves 0 and 1)
      const uint32_t d = tmem + t_lane + (uint32_t)((s % nbuf) * a.d_cols);
      const uint32_t d1 = d + (uint32_t)(nbuf * a.d_cols);
      float* mine = a.partial + (size_t)(2 * blockIdx.x + (s == 0 ? 0 : 1)) * B * kTileM;
      for (int cb = 0; cb < n_mma; cb += 16) {
        float v[16], v1[16];
        __syncwarp();
        tmem_ld16(d + (uint32_t)cb, v);
        tmem_ld16(d1 + (uint32_t)cb, v1);
#pragma unroll
        for (int t = 0; t < 16; ++t) v[t] += v1[t];
        if (whole) {
          emit(tile, cb, v);
        } else {
#pragma unroll
          for (int t = 0; t < 16; ++t)
            if (cb + t < B) mine[(size_t)(cb + t) * kTileM + m] = v[t];
        }
      }
      tc_fence_before();
      mbar_arrive(&dfree[s % nbuf]);
      if (whole) continue;
      // A cut tile: the last contributor sums the contributions in CTA order.
      const int b_first = owner_of(tile * chunks, work, ctas), b_last = owner_of(tile * chunks + chunks - 1, work, ctas);
      __threadfence();
      named_sync(1, 128);
      if (e == 0) last_s = atomicAdd(a.tickets + tile, 1u) == (unsigned)(b_last - b_first) ? 1u : 0u;
      named_sync(1, 128);
      if (last_s) {
        __threadfence();
        for (int cb = 0; cb < n_mma; cb += 16) {
          float v[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) v[t] = 0.f;
          for (int b = b_first; b <= b_last; ++b) {
            const int slot = 2 * b + (range_start(b, work, ctas) / chunks == tile ? 0 : 1);
            const float* src = a.partial + (size_t)slot * B * kTileM;
#pragma unroll
            for (int t = 0; t < 16; ++t)
              if (cb + t < B) v[t] += __ldcg(src + (size_t)(cb + t) * kTileM + m);
          }
          emit(tile, cb, v);
        }
        if (e == 0) a.tickets[tile] = 0u;
      }
      named_sync(1, 128);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (abort_s && tid == 0) atomicExch(&g_gemm_error, 1);
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Load-time repack of a GPTQ-layout projection into the packed layout: per (tile, chunk) the
// 128 rows' codes (16-byte pieces pre-swizzled as the 128-byte TMA swizzle would place them;
// in every 32-bit word the codes of k = 0, 2, 4, 6 in nibbles 0-3 and of k = 1, 3, 5, 7 in
// nibbles 4-7, so the dequantisation takes a pair with one shift and mask), their 8 scales
// and 4 zero-point bytes (0x88 = zero point 8 without zero points). One thread per (tile,
// chunk, row).
template <bool PAIRED>
__global__ void __launch_bounds__(256) w4a16_gemm_pack_kernel(const uint8_t* __restrict__ qweight,
                                                              const __nv_bfloat16* __restrict__ scales,
                                                              const uint8_t* __restrict__ qzeros,
                                                              uint8_t* __restrict__ out, int n, int k, int tiles,
                                                              int chunks) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)tiles * chunks * kTileM) return;
  const int m = (int)(idx & (kTileM - 1));
  const long tcw = idx >> 7;
  const int tile = (int)(tcw / chunks), c = (int)(tcw % chunks);
  const int n_out = PAIRED ? n / 2 : n;
  const int row = PAIRED ? (m < 64 ? tile * 64 + m : n_out + tile * 64 + (m - 64)) : tile * kTileM + m;
  uint8_t* blk = out + tcw * kPackedBlock;
  const uint4* src = reinterpret_cast<const uint4*>(qweight + (size_t)row * (k / 2) + (size_t)c * (kChunk / 2));
  uint4* dst = reinterpret_cast<uint4*>(blk + (size_t)m * (kChunk / 2));
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    // each 32-bit word: the even-k codes into nibbles 0-3, the odd-k codes into nibbles 4-7
    uint4 q = src[p];
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t e = w[i] & 0x0F0F0F0Fu, o = (w[i] >> 4) & 0x0F0F0F0Fu;
      const uint32_t e16 = (e & 0xFu) | ((e >> 4) & 0xF0u) | ((e >> 8) & 0xF00u) | ((e >> 12) & 0xF000u);
      const uint32_t o16 = (o & 0xFu) | ((o >> 4) & 0xF0u) | ((o >> 8) & 0xF00u) | ((o >> 12) & 0xF000u);
      w[i] = e16 | (o16 << 16);
    }
    dst[p ^ (m & 7)] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  *reinterpret_cast<uint4*>(blk + kScaleOff + m * 16) =
      *reinterpret_cast<const uint4*>(scales + (size_t)row * (k / 32) + (size_t)c * 8);
  *reinterpret_cast<uint32_t*>(blk + kPackedZeroOff + m * 4) =
      qzeros ? *reinterpret_cast<const uint32_t*>(qzeros + (size_t)row * (k / 64) + (size_t)c * 4) : 0x88888888u;
}

struct Plan {
  int tiles, chunks, n_mma, ctas, cstages, xstages, d_cols, nbuf, slots;
  size_t smem, partial_bytes, ticket_bytes;
};

static bool make_plan(int batch, int n, int k, int mode, Plan* p, bool packed = false) {
  const bool paired = mode & 4;
  if (batch < 1 || batch > kMaxBatch || k < kChunk || k % kChunk || n < kTileM || n % kTileM) return false;
  p->tiles = paired ? (n / 2) / 64 : n / kTileM;
  p->chunks = k / kChunk;
  p->n_mma = (batch + 15) / 16 * 16;
  // two MMA warps, each with its own accumulator per buffer: double-buffered up to 32 columns
  // (3 A slots either way up to 64 columns, 2 at 128)
  p->d_cols = p->n_mma <= 32 ? 32 : p->n_mma <= 64 ? 64 : 128;
  p->nbuf = p->d_cols <= 32 ? 2 : 1;
  p->slots = (kTmemCols - kMmaWarps * p->nbuf * p->d_cols) / kSlotCols;
  if (p->slots > kMaxSlots) p->slots = kMaxSlots;
  const long work = (long)p->tiles * p->chunks;
  p->ctas = (int)(work < sm_count() ? work : sm_count());
  // activation stages: up to four in at most ~45 % of the budget (two at least); the code
  // ring takes the rest, up to eight stages
  const size_t cstage = packed ? kPackedXOff : kXOff, xstage = (size_t)p->n_mma * kChunk * 2,
               fixed = 1024 + 16 * 64 * sizeof(float), budget = 220 * 1024 - fixed;
  p->xstages = (int)(budget * 45 / 100 / xstage);
  if (p->xstages > 4) p->xstages = 4;
  if (p->xstages < 2) p->xstages = 2;
  p->cstages = (int)((budget - p->xstages * xstage) / cstage);
  if (p->cstages > kMaxStages) p->cstages = kMaxStages;
  if (p->cstages < 2) return false;
  p->smem = fixed + (size_t)p->cstages * cstage + (size_t)p->xstages * xstage;
  // a fixed ticket region, so that calls of different shapes can share one workspace: one
  // call's partials never overlap another call's tickets
  if (p->tiles > kMaxTiles) return false;
  p->ticket_bytes = (size_t)kMaxTiles * sizeof(unsigned);
  p->partial_bytes = (size_t)2 * p->ctas * batch * kTileM * sizeof(float);
  return true;
}

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && fn)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return encode;
}

// TMA map of the 4-bit codes qweight [n, k/2] bytes: boxes of 128 bytes (one K chunk) x 64 rows
// with the 128-byte swizzle.
static bool code_map(CUtensorMap* map, const void* qweight, int n, int k) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)k / 2, (cuuint64_t)n};
  const cuuint64_t strides[1] = {(cuuint64_t)k / 2};
  const cuuint32_t box[2] = {kChunk / 2, 64};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(qweight), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// TMA map of a per-row table (scales [n, cols] bf16 or zero points [n, cols] bytes): boxes of
// `box` elements (16 bytes) x 64 rows, no swizzle.
static bool row_map(CUtensorMap* map, const void* base, CUtensorMapDataType type, int n, int cols, int elem,
                    int box_cols) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)n};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * elem};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, 64};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// TMA map of the activations x [batch, k] bf16: boxes of 64 columns x n_mma rows with the
// 128-byte swizzle; rows past `batch` are out of bounds and read as zeros.
static bool activation_map(CUtensorMap* map, const void* x, int batch, int k, int n_mma) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)batch};
  const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)n_mma};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc

cudaError_t gemm_error_word(int* value, bool clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int));
  if (e != cudaSuccess) return e;
  *value |= v;
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof(int));
  }
  return e;
}

}  // namespace mt

using namespace mt;

// Workspace bytes of mt_w4a16_gemm on the current device for this shape: a fixed 16 KB ticket
// region, then the contributions to tiles cut between CTAs. Calls of different shapes may
// share one workspace of the largest size when they are ordered on one stream. The workspace must be zero-filled once; calls leave the tickets zero.
MT_API int mt_w4a16_gemm_workspace(int batch, int n, int k, int mode, long long* bytes) {
  tc::Plan p;
  if (!bytes || (mode & ~4) || !tc::make_plan(batch, n, k, mode, &p)) return kBadArgument;
  *bytes = (long long)(p.ticket_bytes + p.partial_bytes);
  return 0;
}

// Batched W4A16 G32 projection on tcgen05 tensor cores: y[b, :] = bf16(x[b, :] . W^T) for
// b < batch (1..128; meant for 16 and up), W = bf16((q - z) * s) from the GPTQ layout
// (qweight uint8 [n, k/2], scales bf16 [n, k/32], qzeros uint8 [n, k/64] or NULL for z = 8).
// mode 0, or MT_LINEAR_PAIRED (rows [0, n/2) gate, [n/2, n) up; y has n/2 columns).
// Requires n % 128 == 0, k % 256 == 0, 16-byte aligned x / qweight / y.
MT_API int mt_w4a16_gemm(const void* x, const void* qweight, const void* scales, const void* qzeros, void* y,
                         int batch, int n, int k, int mode, void* workspace, int flags, void* stream) {
  tc::Plan p;
  if (!x || !qweight || !scales || !y || !workspace || (mode & ~4) || !tc::make_plan(batch, n, k, mode, &p))
    return kBadArgument;
  if (!aligned(x, 16) || !aligned(qweight, 16) || !aligned(scales, 16) || (qzeros && !aligned(qzeros, 16)) ||
      !aligned(workspace, 256))
    return kBadArgument;
  tc::GemmArgs a;
  a.x = (const __nv_bfloat16*)x;
  a.packed = nullptr;
  a.qweight = (const uint8_t*)qweight;
  a.scales = (const __nv_bfloat16*)scales;
  a.qzeros = (const uint8_t*)qzeros;
  a.y = (__nv_bfloat16*)y;
  a.tickets = (unsigned*)workspace;
  a.partial = (float*)((uint8_t*)workspace + p.ticket_bytes);
  a.batch = batch;
  a.n = n;
  a.k = k;
  a.n_mma = p.n_mma;
  a.tiles = p.tiles;
  a.chunks = p.chunks;
  a.cstages = p.cstages;
  a.xstages = p.xstages;
  a.d_cols = p.d_cols;
  a.nbuf = p.nbuf;
  a.slots = p.slots;
  a.zt = qzeros && (k / 64) % 16 == 0;
  alignas(64) CUtensorMap xmap, wmap, smap, zmap;
  memset(&zmap, 0, sizeof(zmap));
  if (!tc::activation_map(&xmap, x, batch, k, p.n_mma) || !tc::code_map(&wmap, qweight, n, k) ||
      !tc::row_map(&smap, scales, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, n, k / 32, 2, 8) ||
      (a.zt && !tc::row_map(&zmap, qzeros, CU_TENSOR_MAP_DATA_TYPE_UINT8, n, k / 64, 1, 16)))
    return (int)cudaErrorNotSupported;
  const dim3 grid(p.ctas), block(tc::kThreads);
  cudaStream_t s = (cudaStream_t)stream;
  if (mode & 4) return (int)launch(tc::w4a16_gemm_tc<true, false>, grid, block, p.smem, s, flags & kFlagPdl, a, xmap, wmap, smap, zmap);
  return (int)launch(tc::w4a16_gemm_tc<false, false>, grid, block, p.smem, s, flags & kFlagPdl, a, xmap, wmap, smap, zmap);
}

// Bytes of the packed layout of an [n, k] projection for mt_w4a16_gemm_packed (mode as
// mt_w4a16_gemm): 18,944 bytes per 128-row tile and 256-column chunk.
MT_API int mt_w4a16_gemm_pack_size(int n, int k, int mode, long long* bytes) {
  tc::Plan p;
  if (!bytes || (mode & ~4) || !tc::make_plan(1, n, k, mode, &p, true)) return kBadArgument;
  *bytes = (long long)p.tiles * p.chunks * tc::kPackedBlock;
  return 0;
}

// Load-time repack of a GPTQ-layout projection (qweight uint8 [n, k/2], scales bf16 [n, k/32],
// qzeros uint8 [n, k/64] or NULL) into `packed` (mt_w4a16_gemm_pack_size bytes, 16-byte
// aligned): each (tile, chunk) of the batched GEMM becomes one contiguous block, so the kernel
// fetches it with one bulk copy instead of hundreds of row pieces. Same role as the
// reference's load-time install_packing (src/moss_tts/_runtime/dp4a_packing.py:128-160).
MT_API int mt_w4a16_gemm_pack(const void* qweight, const void* scales, const void* qzeros, int n, int k, int mode,
                              void* packed, void* stream) {
  tc::Plan p;
  if (!qweight || !scales || !packed || (mode & ~4) || !tc::make_plan(1, n, k, mode, &p, true)) return kBadArgument;
  if (!aligned(qweight, 16) || !aligned(scales, 16) || (qzeros && !aligned(qzeros, 4)) || !aligned(packed, 16))
    return kBadArgument;
  const long threads = (long)p.tiles * p.chunks * tc::kTileM;
  const dim3 grid((unsigned)((threads + 255) / 256));
  auto k_ = (mode & 4) ? tc::w4a16_gemm_pack_kernel<true> : tc::w4a16_gemm_pack_kernel<false>;
  return (int)launch(k_, grid, dim3(256), 0, (cudaStream_t)stream, 0, (const uint8_t*)qweight,
                     (const __nv_bfloat16*)scales, (const uint8_t*)qzeros, (uint8_t*)packed, n, k, p.tiles, p.chunks);
}

// mt_w4a16_gemm over the packed layout (mt_w4a16_gemm_pack): same arguments and results, the
// weights given as `packed`; the workspace is the one of mt_w4a16_gemm_workspace.
MT_API int mt_w4a16_gemm_packed(const void* x, const void* packed, void* y, int batch, int n, int k, int mode,
                                void* workspace, int flags, void* stream) {
  tc::Plan p;
  if (!x || !packed || !y || !workspace || (mode & ~4) || !tc::make_plan(batch, n, k, mode, &p, true))
    return kBadArgument;
  if (!aligned(x, 16) || !aligned(packed, 16) || !aligned(workspace, 256)) return kBadArgument;
  tc::GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.x = (const __nv_bfloat16*)x;
  a.packed = (const uint8_t*)packed;
  a.y = (__nv_bfloat16*)y;
  a.tickets = (unsigned*)workspace;
  a.partial = (float*)((uint8_t*)workspace + p.ticket_bytes);
  a.batch = batch;
  a.n = n;
  a.k = k;
  a.n_mma = p.n_mma;
  a.tiles = p.tiles;
  a.chunks = p.chunks;
  a.cstages = p.cstages;
  a.xstages = p.xstages;
  a.d_cols = p.d_cols;
  a.nbuf = p.nbuf;
  a.slots = p.slots;
  alignas(64) CUtensorMap xmap, none;
  memset(&none, 0, sizeof(none));
  if (!tc::activation_map(&xmap, x, batch, k, p.n_mma)) return (int)cudaErrorNotSupported;
  const dim3 grid(p.ctas), block(tc::kThreads);
  cudaStream_t s = (cudaStream_t)stream;
  if (mode & 4)
    return (int)launch(tc::w4a16_gemm_tc<true, true>, grid, block, p.smem, s, flags & kFlagPdl, a, xmap, none, none,
                       none);
  return (int)launch(tc::w4a16_gemm_tc<false, true>, grid, block, p.smem, s, flags & kFlagPdl, a, xmap, none, none,
                     none);
}
