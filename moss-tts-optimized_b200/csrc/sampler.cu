// On-device top-k / top-p sampling of a decode step's next ids (sm_100a).
//
// The non-greedy half of FastLLM._decode (src/moss_tts/_runtime/llm.py:280-287) with the
// reference's sampler sample_topk (llm.py:10-19) for every channel of every sequence:
//   text:  sample_topk(text logits [n_text], 1.5, 2, 1.0) -> index into the audio-phase id table
//   audio: sample_topk(codebook logits [vocab], 1.7, 25, 0.8) per codebook
// followed by the delay-pattern masks (llm.py:281-286), as mt_heads_select does for greedy.
// sample_topk: x = float(logit) / T; the top k of x (sorted, descending); probabilities =
// softmax over those k; an entry is removed when the cumulative probability before it
// (cumsum - p, as the reference computes it) exceeds top_p; one draw from the kept entries in
// proportion to their probabilities (torch.multinomial). T <= 0 is argmax (first index on ties).
//
// One CTA of 128 threads per (channel, sequence). The row (at most 1024 logits) lives in
// registers, 8 per thread; the top k are found in k rounds of a block-wide 64-bit max over
// (order-preserving value bits, ~index) keys, so equal values keep ascending index order. The
// draw is one uniform from Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers:
// as easy as 1, 2, 3", SC'11), keyed by the sequence's 64-bit seed with counter (channel,
// position low, position high, 0): a function of (seed, position, channel) only, so graph
// replays, batch composition and launch order do not change a sequence's samples.
#include "common.cuh"

namespace mt {

constexpr int kSampleThreads = 128;
constexpr int kSamplePerThread = 8;  // vocab <= 1024
constexpr int kMaxTopK = 64;

struct SampleArgs {
  const __nv_bfloat16* text_logits;   // [batch, n_text]
  const __nv_bfloat16* audio_logits;  // [batch, n_cb * V]
  const int64_t* text_ids;            // [n_text]
  const int64_t* position;            // [batch]
  const int64_t* audio_length;        // [batch]
  const int64_t* delay_length;        // [batch]
  const uint64_t* seed;               // [batch]
  int64_t* next_ids;                  // [batch, 1 + n_vq]
  int n_text, n_cb, V, cb_offset, n_vq;
  int delay_slot_id, audio_end_id, pad_code, text_owner;
  float temp[2], top_p[2];  // [0] text, [1] audio
  int top_k[2];
};

// Philox4x32 with 10 rounds: per round (hi0, lo0) = M0 * c0, (hi1, lo1) = M1 * c2 (32 x 32 -> 64),
// c = (hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0); the key advances by the Weyl constants between
// rounds. Constants are the published Philox4x32 multipliers and key increments.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

__device__ __forceinline__ unsigned long long sample_key(float v, int idx) {
  return ((unsigned long long)ordered_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(kSampleThreads) heads_sample(SampleArgs a) {
  __shared__ unsigned long long warp_best[2][kSampleThreads / 32];
  __shared__ float topv[kMaxTopK];
  __shared__ int topi[kMaxTopK];
  const int b = blockIdx.y, c = (int)blockIdx.x - 1;  // c < 0: the text channel
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  pdl_trigger();
  int64_t* out = a.next_ids + (size_t)b * (1 + a.n_vq);
  if (c < 0) {  // channels owned by other tensor-parallel shards are summed in as zeros
    for (int ch = tid; ch < a.n_vq; ch += blockDim.x)
      if (ch < a.cb_offset || ch >= a.cb_offset + a.n_cb) out[1 + ch] = 0;
    if (!a.text_owner) {
      if (tid == 0) out[0] = 0;
      return;
    }
  }
  const int sel = c < 0 ? 0 : 1;
  const int len = c < 0 ? a.n_text : a.V;
  const float T = a.temp[sel];
  const bool greedy = !(T > 0.f);
  const int k = greedy ? 1 : min(a.top_k[sel], len);
  const __nv_bfloat16* src =
      c < 0 ? a.text_logits + (size_t)b * a.n_text : a.audio_logits + ((size_t)b * a.n_cb + c) * a.V;
  float val[kSamplePerThread];
#pragma unroll
  for (int j = 0; j < kSamplePerThread; ++j) {
    const int i = tid + j * kSampleThreads;
    val[j] = 0.f;
    if (i < len) val[j] = greedy ? bf16f(src[i]) : __fdiv_rn(bf16f(src[i]), T);
  }
  uint32_t taken = 0;  // bit j: val[j] already selected
  for (int r = 0; r < k; ++r) {
    unsigned long long best = 0ull;
#pragma unroll
    for (int j = 0; j < kSamplePerThread; ++j) {
      const int i = tid + j * kSampleThreads;
      if (i < len && !(taken >> j & 1u)) {
        const unsigned long long key = sample_key(val[j], i);
        best = key > best ? key : best;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) warp_best[r & 1][warp] = best;
    __syncthreads();  // the other buffer is rewritten only after the next barrier
#pragma unroll
    for (int w = 0; w < kSampleThreads / 32; ++w) best = warp_best[r & 1][w] > best ? warp_best[r & 1][w] : best;
    const int idx = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    if (idx % kSampleThreads == tid) {  // the owner records the value and retires it
      const int j = idx / kSampleThreads;
#pragma unroll
      for (int jj = 0; jj < kSamplePerThread; ++jj)
        if (jj == j) {
          topv[r] = val[jj];
          taken |= 1u << jj;
        }
      topi[r] = idx;
    }
  }
  __syncthreads();
  if (tid != 0) return;
  int pick = topi[0];
  if (!greedy) {
    // softmax over the k values (fp32, max subtracted), then the top-p cut on cumsum - p
    float p[kMaxTopK];
    float sum = 0.f;
    for (int i = 0; i < k; ++i) {
      p[i] = expf(topv[i] - topv[0]);
      sum += p[i];
    }
    float cum = 0.f, kept = 0.f;
    for (int i = 0; i < k; ++i) {
      p[i] = p[i] / sum;
      cum += p[i];
      if (cum - p[i] > a.top_p[sel]) p[i] = 0.f;
      kept += p[i];
    }
    const uint64_t s = a.seed[b];
    const uint64_t pos = (uint64_t)a.position[b];
    const uint4 rnd = philox4x32_10(make_uint4((uint32_t)(c + 1), (uint32_t)pos, (uint32_t)(pos >> 32), 0u),
                                    make_uint2((uint32_t)s, (uint32_t)(s >> 32)));
    const float u = (float)(rnd.x >> 8) * 0x1.0p-24f;  // [0, 1) in 2^-24 steps
    const float target = u * kept;
    float acc = 0.f;
    int last = 0;
    for (int i = 0; i < k; ++i) {
      if (p[i] <= 0.f) continue;
      last = i;
      acc += p[i];
      if (acc > target) break;
    }
    pick = topi[last];
  }
  const int64_t delay = a.delay_length[b], alen = a.audio_length[b];
  if (c < 0) {  // llm.py:281-283
    int64_t tok = a.text_ids[(pick >= 0 && pick < a.n_text) ? pick : 0];
    if (delay >= 0) tok = a.delay_slot_id;
    if (delay == 32) tok = a.audio_end_id;
    out[0] = tok;
  } else {  // llm.py:284-286
    const int ch = a.cb_offset + c;
    const bool valid = ch < alen && (delay < 0 || ch >= delay);
    out[1 + ch] = valid ? (int64_t)pick : (int64_t)a.pad_code;
  }
}

}  // namespace mt

using namespace mt;

// Sampled next ids for `batch` sequences from their head logits (the non-greedy half of
// FastLLM._decode, src/moss_tts/_runtime/llm.py:280-287, with sample_topk, llm.py:10-19).
// Temperatures <= 0 select the argmax. next_ids [batch, 1 + n_vq]: this shard's codebooks,
// zeros for the others; the text token when text_owner != 0, else zero.
MT_API int mt_heads_sample(const void* text_logits, const void* audio_logits, const void* text_ids,
                           const void* position, const void* audio_length, const void* delay_length,
                           const void* seed, void* next_ids, int batch, int n_text, int n_cb, int vocab,
                           int cb_offset, int n_vq, int delay_slot_id, int audio_end_id, int pad_code,
                           int text_owner, float text_temperature, int text_top_k, float text_top_p,
                           float audio_temperature, int audio_top_k, float audio_top_p, int flags,
                           void* stream) {
  if (!position || !audio_length || !delay_length || !seed || !next_ids || batch < 1 || batch > 65535 ||
      n_cb < 0 || vocab < 1 || vocab > kSampleThreads * kSamplePerThread || cb_offset < 0 ||
      cb_offset + n_cb > n_vq || (n_cb > 0 && !audio_logits))
    return kBadArgument;
  if (text_owner && (!text_logits || !text_ids || n_text < 1 || n_text > kSampleThreads * kSamplePerThread))
    return kBadArgument;
  if (text_top_k < 1 || text_top_k > kMaxTopK || audio_top_k < 1 || audio_top_k > kMaxTopK) return kBadArgument;
  SampleArgs a;
  a.text_logits = (const __nv_bfloat16*)text_logits;
  a.audio_logits = (const __nv_bfloat16*)audio_logits;
  a.text_ids = (const int64_t*)text_ids;
  a.position = (const int64_t*)position;
  a.audio_length = (const int64_t*)audio_length;
  a.delay_length = (const int64_t*)delay_length;
  a.seed = (const uint64_t*)seed;
  a.next_ids = (int64_t*)next_ids;
  a.n_text = n_text;
  a.n_cb = n_cb;
  a.V = vocab;
  a.cb_offset = cb_offset;
  a.n_vq = n_vq;
  a.delay_slot_id = delay_slot_id;
  a.audio_end_id = audio_end_id;
  a.pad_code = pad_code;
  a.text_owner = text_owner;
  a.temp[0] = text_temperature;
  a.temp[1] = audio_temperature;
  a.top_k[0] = text_top_k;
  a.top_k[1] = audio_top_k;
  a.top_p[0] = text_top_p;
  a.top_p[1] = audio_top_p;
  return (int)launch(heads_sample, dim3(1 + n_cb, batch), dim3(kSampleThreads), 0, (cudaStream_t)stream,
                     flags & kFlagPdl, a);
}
