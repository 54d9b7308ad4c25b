#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace air {

// Which keys each query row sees.
struct AttnRows {
  const int* row_seq;        // [R] block-table row of each query row (null: r)
  const int* ctx_len;        // [R] keys [0, ctx) are candidates (causal bound)
  const int* tree_base;      // [R] first position of the speculative tree region (null: none)
  const unsigned long long* tree_mask;  // [R] ancestor bitmask over tree positions
  int window;                // sliding window (0 = none)
  float softcap;             // > 0: scaled scores s -> softcap * tanh(s / softcap) (Gemma-2 style)
};

struct AttnArgs {
  const float* q;            // [R, n_heads, head_dim] (RoPE applied, unscaled)
  const void* kv;            // layer [num_blocks, 2, n_kv, block_size, row]: head_dim bf16, or
                             // (kv_fp8) head_dim E4M3 codes + f32 scale + 12 B padding
  int kv_fp8;
  const int* block_tables;   // [n_seqs, max_blocks]
  int max_blocks;
  AttnRows rows;
  int n_rows, n_heads, n_kv, head_dim, block_size;
  int64_t num_blocks;
  int n_splits, split_tokens;
  float scale;
  float* part_o;             // [R, n_heads, n_splits, head_dim] scratch (n_splits > 1)
  float2* part_ml;           // [R, n_heads, n_splits]
  float* out;                // [R, n_heads, head_dim] fp32
  int8_t* out_q;             // optional Q8A of out
  void* out_bf16;            // optional bf16 copy of out (written by the split merge)
  float2* out_ds;
  int* err;
};

bool launch_paged_attention(const AttnArgs& a, cudaStream_t st);
// tensor-core main pass (head_dim 128, group <= 8); false if the shape is not covered
bool launch_paged_attention_mma(const AttnArgs& a, cudaStream_t st);
// query-tiled prefill pass (head_dim 128, no tree rows, one split, no Q8A output): 16 query
// rows of one KV head per CTA share every K/V tile; false if the shape is not covered
bool launch_prefill_attention(const AttnArgs& a, cudaStream_t st);

}  // namespace air
