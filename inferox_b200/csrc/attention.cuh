// Attention kernels over the device-resident KV cache.
#pragma once
#include "common.cuh"

namespace ifx {

struct DecodeAttnArgs {
  const float *qkv;       // [H*hd | G*hd | G*hd] f32 projections of the new token
  __half *kc, *vc;        // this layer's caches [G][max_seq][hd]
  const int *pos;         // device: cache length before this token (= its position)
  float *part_o;          // [G][NS][grp][hd]
  float2 *part_ml;        // [G][NS][grp] (running max, running sum)
  int *counters;          // [G], zero between launches
  float *attn_out;        // [H*hd]
  float *zero_ptr;        // buffer zeroed by this kernel (may be null)
  int zero_n;
  int H, G, hd, max_seq, ns;
  int rope_compat;        // 1: RoPE at position 0 (identity), forward.rs:371-372
  int rope_dim;
  float rope_base;
  int *err;
  // batched decode (gridDim.z = sequences): sequence b reads qkv + b * qkv_stride,
  // its caches at kc/vc + b * kv_seq_stride, its position pos[b], and uses its
  // own partials, counters and output row (attn_out + b * H * hd)
  int64_t qkv_stride = 0, kv_seq_stride = 0;
  int batch = 1;
  // when set, row b's cache and position are those of sequence slot[b]
  // (a step over a subset of a batch's sequences); workspace rows stay b
  const int *slot = nullptr;
  // paged cache (no reference counterpart: cache pages shared by the
  // sequences of a batch): when set, split s of sequence q covers the
  // page_rows positions of its page page_table[q * max_pages + s], which
  // holds, for every layer and kv head, page_rows consecutive rows; kc / vc
  // then point at the layer's rows in page 0 ([G][page_rows][hd]) and
  // kv_seq_stride is unused
  const int *page_table = nullptr;
  int page_rows = 0, max_pages = 0;
  int64_t page_stride = 0;  // elements per page (all layers and kv heads)
};

ifx_status decode_attention(const DecodeAttnArgs &a, cudaStream_t st, bool pdl);
int decode_attention_smem(int grp, int hd, int max_seq, int ns);

// Causal attention inside one prefill chunk (forward.rs:255-305): q/k/v rows
// of the chunk only, position t attends to 0..=t of the chunk.
struct PrefillAttnArgs {
  const float *q;   // [n][H*hd]
  const float *k;   // [n][G*hd]
  const float *v;   // [n][G*hd]
  float *out;       // [n][H*hd]
  int n, H, G, hd;
  int causal = 1;   // 0: every row attends to every key (Model::forward, forward.rs:100-150)
  // when set (a causal prefill into a KV cache): this layer's cache, whose
  // rows start .. start + n - 1 already hold the chunk's K/V (f16, columns
  // swizzled by position); the streamed kernel reads its K/V tiles there.
  // Paged caches as in DecodeAttnArgs (kc / vc at the layer's rows of page
  // 0, page p of the sequence at page_table[p]).
  const __half *kc = nullptr, *vc = nullptr;
  int start = 0, max_seq = 0;
  const int *page_table = nullptr;
  int page_rows = 0;
  int64_t page_stride = 0;
  int *err = nullptr;
};
ifx_status prefill_attention(const PrefillAttnArgs &a, cudaStream_t st);

}  // namespace ifx
