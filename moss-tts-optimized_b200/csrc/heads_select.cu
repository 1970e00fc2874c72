// Greedy token selection for a batch of decode steps from precomputed head logits (sm_100a).
//
// The batched decode step computes its text and audio logits with one plain bf16 GEMM each
// (as the reference's F.linear heads, src/moss_tts/_runtime/llm.py:271-274); this kernel
// does the rest of FastLLM._decode with greedy sampling for every sequence: argmax per
// codebook with torch.argmax's first-index tie rule (llm.py:11-12), the text token through
// the audio-phase id table, and the delay-pattern masks (llm.py:280-286), each sequence with
// its own audio and delay lengths. One CTA per (channel, sequence): a 64-bit max over
// (order-preserving bf16 logit bits, ~index) keys.
#include "common.cuh"

namespace mt {

struct SelectArgs {
  const __nv_bfloat16* text_logits;   // [batch, n_text]
  const __nv_bfloat16* audio_logits;  // [batch, n_cb * V]
  const int64_t* text_ids;            // [n_text]
  const int64_t* audio_length;        // [batch]
  const int64_t* delay_length;        // [batch]
  int64_t* next_ids;                  // [batch, 1 + n_vq]
  int n_text, n_cb, V, cb_offset, n_vq;
  int delay_slot_id, audio_end_id, pad_code, text_owner;
};

__device__ __forceinline__ unsigned long long select_key(float v, int idx) {
  return ((unsigned long long)ordered_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(256) heads_select(SelectArgs a) {
  __shared__ unsigned long long warp_best[8];
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
  const int len = c < 0 ? a.n_text : a.V;
  const __nv_bfloat16* src =
      c < 0 ? a.text_logits + (size_t)b * a.n_text : a.audio_logits + ((size_t)b * a.n_cb + c) * a.V;
  unsigned long long best = 0ull;
  for (int i = tid; i < len; i += blockDim.x) {
    const unsigned long long k = select_key(bf16f(src[i]), i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if (lane == 0) warp_best[warp] = best;
  __syncthreads();
  if (tid != 0) return;
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = warp_best[w] > best ? warp_best[w] : best;
  const int idx = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
  const int64_t delay = a.delay_length[b], alen = a.audio_length[b];
  if (c < 0) {  // llm.py:280-283
    int64_t tok = a.text_ids[(idx >= 0 && idx < a.n_text) ? idx : 0];
    if (delay >= 0) tok = a.delay_slot_id;
    if (delay == 32) tok = a.audio_end_id;
    out[0] = tok;
  } else {  // llm.py:284-286
    const int ch = a.cb_offset + c;
    const bool valid = ch < alen && (delay < 0 || ch >= delay);
    out[1 + ch] = valid ? (int64_t)idx : (int64_t)a.pad_code;
  }
}

}  // namespace mt

using namespace mt;

// Greedy selection for `batch` sequences from their head logits. Replaces the sampling half of
// FastLLM._decode with greedy=True (src/moss_tts/_runtime/llm.py:276-287) for a batch: writes
// next_ids [batch, 1 + n_vq] (this shard's codebooks, zeros for the others; the text token
// when text_owner != 0, else zero).
MT_API int mt_heads_select(const void* text_logits, const void* audio_logits, const void* text_ids,
                           const void* audio_length, const void* delay_length, void* next_ids, int batch,
                           int n_text, int n_cb, int vocab, int cb_offset, int n_vq, int delay_slot_id,
                           int audio_end_id, int pad_code, int text_owner, int flags, void* stream) {
  if (!audio_length || !delay_length || !next_ids || batch < 1 || batch > 65535 || n_cb < 0 || vocab < 1 ||
      cb_offset < 0 || cb_offset + n_cb > n_vq || (n_cb > 0 && !audio_logits))
    return kBadArgument;
  if (text_owner && (!text_logits || !text_ids || n_text < 1)) return kBadArgument;
  SelectArgs a;
  a.text_logits = (const __nv_bfloat16*)text_logits;
  a.audio_logits = (const __nv_bfloat16*)audio_logits;
  a.text_ids = (const int64_t*)text_ids;
  a.audio_length = (const int64_t*)audio_length;
  a.delay_length = (const int64_t*)delay_length;
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
  return (int)launch(heads_select, dim3(1 + n_cb, batch), dim3(256), 0, (cudaStream_t)stream, flags & kFlagPdl, a);
}
