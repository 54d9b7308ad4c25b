#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include "kernels.h"

namespace air {

struct GemvTiledScratch {
  float* ws;        // split-K partials: gemv_tiled_workspace_floats() floats
  int* counters;    // gemv_tiled_counters() ints, zero before first use (self-resetting)
  int wsplit = 0;   // bulk copies per 18 KB slab (0: launch_gemv_tiled picks)
  int early_trigger = -1;   // release a dependent launch before the epilogue (-1: AIR_PDL_EARLY, default on)
};

int gemv_tiled_splits(int N, int K, int mode);
size_t gemv_tiled_workspace_floats(int N, int splits, int mode);
size_t gemv_tiled_counters(int N);
// nullptr on success, else an error message (nothing launched).
const char* launch_gemv_tiled(const GemvWeight& w, int N, int K, int B, const int8_t* xq,
                              const float2* xds, const GemvEpiParams& ep, const GemvTiledScratch& sc,
                              int splits, cudaStream_t st);

}  // namespace air
