#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "kernels.h"

namespace air {

struct RopeKvArgs {
  const float2* rope_cs;   // [max_pos, rot_dim/2]
  const int* positions;    // [T]
  const int64_t* slots;    // [T]
  void* kv_cache;          // layer [num_blocks, 2, n_kv, block_size, head_dim] bf16
  float* q_out;            // [T, n_heads, head_dim]
  int n_heads, n_kv, head_dim, block_size, rot_dim;
  int64_t num_blocks;
  int* err;
  const float* bias;       // optional [(n_heads + 2 n_kv) * head_dim] q|k|v bias, added before RoPE
  int kv_fp8;              // 1: the pool rows are E4M3 codes + f32 scale (kv_f8.cuh)
};

void launch_embed(int fmt, const void* table, const void* scales, int64_t row_bytes, int K,
                  const int* ids, int n, int64_t vocab, float* out_f32, void* out_bf16, float mult,
                  int* err, cudaStream_t st);
void launch_dequant(int fmt, const void* w, const void* scales, int64_t row_bytes, int N, int K,
                    void* out, cudaStream_t st);
void launch_rope_kv(const void* qkv, bool bf16_in, int T, const RopeKvArgs& a, cudaStream_t st);
void launch_swiglu(const void* gu, bool bf16_in, int T, int F, int64_t ld_in, int64_t up_off,
                   int64_t ld_out, void* out_bf16, float* out_f32, int act, cudaStream_t st);
void launch_residual_add(float* resid, const void* y, bool bf16_in, int64_t n, cudaStream_t st);

}  // namespace air
