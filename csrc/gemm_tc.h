#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>
#include "kernels.h"

namespace air {

// kGemmPeerPush: the output is a tensor-parallel partial, stored from the epilogue into the
// peer receive buffers (PeerPush protocol, comm.h) instead of `out`.
// kGemmQkvRope: the output rows are [q heads | k heads | v heads] of head_dim 128 (one head per
// 128-row tile); the epilogue adds the optional bias, applies NeoX RoPE to q and k, writes q
// (fp32) and k, v into the paged KV cache (bf16) instead of `out`.
enum GemmMode : int { kGemmStoreF32 = 0, kGemmStoreBF16 = 1, kGemmResidualF32 = 2, kGemmPeerPush = 3,
                      kGemmQkvRope = 4 };

struct GemmRope {
  const float2* cs;        // [max_pos, rot_dim / 2] (cos, sin)
  const int* positions;    // [T]
  const int64_t* slots;    // [T] paged-cache slot (block * block_size + offset); < 0 = skip
  void* kv;                // layer [num_blocks, 2, n_kv, block_size, 128] bf16
  float* q_out;            // [T, n_heads, 128]
  const float* bias;       // optional [(n_heads + 2 n_kv) * 128]
  int n_heads, n_kv, block_size, rot_dim;
  int64_t num_blocks;
};

struct GemmArgs {
  int N, K, T;          // weight rows, reduction length, tokens
  int mode;             // GemmMode
  void* out;            // [T, ldo] (f32 or bf16)
  int64_t ldo;
  int splits;           // split-K factor (1 = none)
  float* ws;            // split-K partials: gemm_q_workspace_floats() floats
  int* counters;        // gemm_q_counters() ints, zero before first use (self-resetting)
  int* err;
  long long* dbg;
  const uint8_t* wq;    // weight base (filled by launch_gemm_q)
  int wsplit;           // raw weight tile copy split into this many bulk copies (filled in)
  const int* row_count; // optional device count of valid token rows: token tiles at or past it
                        // exit at once (routed-expert GEMMs launched for a capacity)
  PeerPush push;        // kGemmPeerPush destinations
  const void* wscales;  // Q8_0: f16 block scales [N, K/32] (the codes are the weight pointer)
  GemmRope rope;        // kGemmQkvRope
       // optional per-phase clock64 stamps of CTA (0,0,0) (profiling aid)
};

int gemm_q_token_tile(int T);
int gemm_q_splits(int N, int K, int T, int fmt);
size_t gemm_q_workspace_floats(int N, int K, int T, int fmt, int splits);
size_t gemm_q_counters(int N, int T);
// Returns nullptr on success, else an error message (nothing was launched).
const char* launch_gemm_q(int fmt, const void* w, int64_t w_row_bytes, const void* x, int64_t ldx,
                          const GemmArgs& a, cudaStream_t st);

}  // namespace air
