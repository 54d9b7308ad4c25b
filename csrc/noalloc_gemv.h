// Allocation-free C entry point for the Q4_K decode GEMV.
//
// This entry point has no counterpart in the reference implementation; it exists for
// callers that must not allocate device memory: code running inside an allocator-free
// runtime (a custom memory manager that owns all of HBM, a plugin host that forbids
// cudaMalloc, real-time or embedded loops where an allocation could block or fail).
// It runs the same tiled Q4_K GEMV kernel as the library path (air_rs._C.gemv), but its
// split-K workspace and tile counters live in a fixed device array inside this library
// instead of a caller- or torch-allocated buffer.
//
// Limits and rules:
//   * The scratch is AIR_NOALLOC_SCRATCH_BYTES (4 MiB) per GPU, reserved on every GPU that
//     loads the library until the process exits. It holds a header of tile counters and the
//     split-K partials; the number of splits is lowered until the partials fit, so any K
//     works, and the only size limit is N <= AIR_NOALLOC_MAX_N (16383 row tiles of 128):
//     larger N is rejected with AIR_NOALLOC_TOO_LARGE.
//   * The first call on a device looks up the array's device address (cudaGetSymbolAddress)
//     with that device current; make that first call before any stream capture.
//   * All calls share the one array and it keeps the previous call's contents; the call
//     clears the parts that must start at zero. Calls whose kernels overlap on the GPU
//     (different streams without ordering) race on the array: serialise them.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define AIR_NOALLOC_SCRATCH_BYTES (4u << 20)
#define AIR_NOALLOC_MAX_N (16383 * 128)

enum AirNoAllocStatus {
  AIR_NOALLOC_OK = 0,
  AIR_NOALLOC_BAD_ARGUMENT = 1,   // null pointer (err included), B outside [1, 8], K not a multiple of 256, N <= 0
  AIR_NOALLOC_TOO_LARGE = 2,      // N > AIR_NOALLOC_MAX_N
  AIR_NOALLOC_SETUP_FAILED = 3,   // cudaGetDevice / cudaGetSymbolAddress failed
  AIR_NOALLOC_LAUNCH_FAILED = 4,  // the kernel launch (or the counter clear) was rejected
};

#ifdef __cplusplus
extern "C" {
#endif

// out[b, n] = sum_k x[b, k] * W[n, k] for b < B (B <= 8), written as fp32 with row stride N.
//   w_tiled : Q4_K weight in the tiled device layout [ceil(N/128)][K/256][128][144 B]
//   xq, xds : activations quantised per 32 (int8 [B, K] and float2 (d, d*sum) [B, K/32])
//   err     : required device int; receives a nonzero code if a bounded wait in the kernel
//             gave up (the output is then incomplete). It is never cleared by the call.
// Enqueues work on `stream` and returns without synchronising.
int air_gemv_q4k_noalloc(const void* w_tiled, int N, int K, int B, const int8_t* xq, const void* xds,
                         float* out, int* err, cudaStream_t stream);

// Human-readable text for a status code.
const char* air_noalloc_status_string(int status);

#ifdef __cplusplus
}
#endif
