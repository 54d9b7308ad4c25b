#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>
#include "kernels.h"

namespace air {

// kGemmPeerPush: the output is a tensor-parallel partial, stored from the epilogue into the
// peer receive buffers (PeerPush protocol, comm.h) instead of `out`.
enum GemmMode : int { kGemmStoreF32 = 0, kGemmStoreBF16 = 1, kGemmResidualF32 = 2, kGemmPeerPush = 3 };

constexpr int kGemmMaxGroups = 8;


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
  // Grouped launch (routed experts): blockIdx.y = group * tiles_per_group + token tile; group g
  // reads weight g (wq_g / wscales_g / its tensor maps) and rows [g * group_rows, + group_rows)
  // of x and out, limited by row_count[g]. groups == 0: one weight, rows [0, T).
  int groups, group_rows, tiles_per_group;
  const uint8_t* wq_g[kGemmMaxGroups];
  const void* wscales_g[kGemmMaxGroups];
       // optional per-phase clock64 stamps of CTA (0,0,0) (profiling aid)
};

int gemm_q_token_tile(int T);
int gemm_q_splits(int N, int K, int T, int fmt);
size_t gemm_q_workspace_floats(int N, int K, int T, int fmt, int splits);
size_t gemm_q_counters(int N, int T);
// Grouped launch: G <= kGemmMaxGroups weights of one shape, x [G * rows, K], out [G * rows, N];
// row_count[g] (device) limits group g. Store modes only.
const char* launch_gemm_q_grouped(int fmt, const void* const* w, const void* const* scales, int G,
                                  int64_t w_row_bytes, const void* x, int64_t ldx, int rows, const GemmArgs& a,
                                  cudaStream_t st);
// Returns nullptr on success, else an error message (nothing was launched).
const char* launch_gemm_q(int fmt, const void* w, int64_t w_row_bytes, const void* x, int64_t ldx,
                          const GemmArgs& a, cudaStream_t st);

}  // namespace air
