// Paged fp16 KV cache and RoPE + GQA attention kernels.
#pragma once
#include "common.cuh"

namespace n730 {

// One layer's paged KV: pages of `page_size` positions, layout
// k_pages/v_pages [num_pages][n_kv][page_size][head_dim] fp16.  A sequence's
// position p lives in page block_table[b * max_pages + p / page_size].
struct KVLayer {
  __half* k_pages;
  __half* v_pages;
};

struct AttnDims {
  int n_heads, n_kv, head_dim;
  int page_size, max_pages;   // per sequence
  float scale;                // 1/sqrt(head_dim)
};

// Decode: one new token per sequence.  qkv [B][ld_qkv] holds q|k|v (biases
// added, RoPE not yet applied); positions are seq_lens[b].  Writes the RoPE'd
// k and v into the cache and attn_out [B][n_heads*head_dim].  No global
// workspace: the context splits of a (sequence, KV head) form one thread-block
// cluster and merge through distributed shared memory.
struct DecodeAttnArgs {
  const float* qkv; int ld_qkv;
  const float* cos_t; const float* sin_t;   // [max_pos][head_dim/2]
  const int* seq_lens;                       // [B]
  const int* block_table;                    // [B][max_pages]
  KVLayer kv;
  AttnDims d;
  float* out;
  int batch;
  int pdl;
};
int attn_decode_launch(const DecodeAttnArgs& a, cudaStream_t st);

// Prefill of T tokens of sequence b at positions [pos0, pos0+T): applies RoPE
// to q (in place in qkv) and k, writes k/v into the cache.
struct KVWriteArgs {
  float* qkv; int ld_qkv;
  const float* cos_t; const float* sin_t;
  const int* block_table;  // row of sequence b
  KVLayer kv;
  AttnDims d;
  int T, pos0;
  int pdl;
};
int kv_write_launch(const KVWriteArgs& a, cudaStream_t st);

// Causal attention of T queries (q RoPE'd, in qkv) against cache positions
// [0, pos0+T); query t sees keys <= pos0+t.  out [T][n_heads*head_dim].
struct PrefillAttnArgs {
  const float* qkv; int ld_qkv;
  const int* block_table;
  KVLayer kv;
  AttnDims d;
  int T, pos0;
  float* out;
  int pdl;
};
int attn_prefill_launch(const PrefillAttnArgs& a, cudaStream_t st);

}  // namespace n730
