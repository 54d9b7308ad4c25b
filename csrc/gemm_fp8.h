#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace air {

// W8A8 FP8 GEMM (tcgen05 kind::f8f6f4): out[T, N] (op)= (sx * qx) @ (sw * qw)^T with E4M3
// codes, one f32 weight multiplier per row and 128-wide K block, one f32 scale per token.
struct GemmF8Args {
  int N, K, T;
  int mode;                 // kGemmStoreF32 / kGemmStoreBF16 / kGemmResidualF32 (gemm_tc.h)
  const void* wq;           // [N, w_row_bytes] E4M3 codes
  int64_t w_row_bytes;
  const float* wscale;      // [N, K/128]
  const void* xq;           // [T, K] E4M3 codes (row stride K)
  const float* xscale;      // [T]
  void* out;                // [T, ldo]
  int64_t ldo;
  int splits;
  float* ws;                // gemm_fp8_workspace_floats() floats when splits > 1
  int* counters;            // gemm_fp8_counters() ints, zero before first use (self-resetting)
  int* err;                 // required: bounded waits report here
};

int gemm_fp8_token_tile(int T);
int gemm_fp8_splits(int N, int K, int T);
size_t gemm_fp8_workspace_floats(int N, int T, int splits);
size_t gemm_fp8_counters(int N, int T);
// Both return nullptr on success, else an error message (nothing was launched).
const char* launch_gemm_fp8(const GemmF8Args& a, cudaStream_t st);
// x bf16 [T, K] (row stride ldx elements) -> xq E4M3 [T, K], xs f32 [T] (row amax / 448)
const char* launch_quant_fp8_rows(const void* x, int64_t ldx, int T, int K, void* xq, float* xs, cudaStream_t st);

}  // namespace air
