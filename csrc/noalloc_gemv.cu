// Allocation-free Q4_K decode GEMV entry point (see noalloc_gemv.h for the contract).
// No counterpart in the reference implementation.
#include <mutex>

#include "noalloc_gemv.h"
#include "gemv_tiled.h"
#include "kernels.h"

namespace {

// The only scratch this entry point uses: [err word + tile counters | split-K partials].
static __device__ __align__(256) unsigned char g_noalloc_scratch[AIR_NOALLOC_SCRATCH_BYTES];

constexpr size_t kHeaderBytes = 64 * 1024;              // err word + up to 16383 tile counters
constexpr size_t kMaxCounters = kHeaderBytes / sizeof(int) - 1;
constexpr int kMaxDevices = 64;

// Device address of g_noalloc_scratch per device. In host code the symbol name is only a
// host-side stand-in, so the address must be looked up on each device it is used on.
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_mu;

int scratch_for_current_device(unsigned char** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AIR_NOALLOC_SETUP_FAILED;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return AIR_NOALLOC_SETUP_FAILED;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_ptr[dev]);
  return AIR_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int air_gemv_q4k_noalloc(
    const void* w_tiled, int N, int K, int B, const int8_t* xq, const void* xds, float* out, int* err,
    cudaStream_t stream) {
  if (!w_tiled || !xq || !xds || !out || !err || N <= 0 || K <= 0 || K % 256 != 0 || B < 1 || B > 8)
    return AIR_NOALLOC_BAD_ARGUMENT;
  // grid cap: as many CTAs as the static array has split-K partial slots for
  const int per_cta = (int)(air::gemv_tiled_workspace_floats(N, 1, air::kEpiStore) * sizeof(float));
  const int fit = (int)((AIR_NOALLOC_SCRATCH_BYTES - kHeaderBytes) / per_cta);
  int splits = air::gemv_tiled_splits(N, K, air::kEpiStore);
  splits = splits < fit ? splits : fit;
  const size_t counters = air::gemv_tiled_counters(N);
  // The split count above is capped to what the array holds, so the partials always fit;
  // the one real limit is the tile-counter header (N <= AIR_NOALLOC_MAX_N).
  if (counters > kMaxCounters) return AIR_NOALLOC_TOO_LARGE;

  unsigned char* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch);
  if (st != AIR_NOALLOC_OK) return st;
  int* cnt = reinterpret_cast<int*>(scratch) + 1;
  float* ws = reinterpret_cast<float*>(scratch + kHeaderBytes);
  // The counters must start at zero; a previous call that gave up early could have left
  // them raised. The caller's err word is left alone (it accumulates across calls).
  if (cudaMemsetAsync(scratch, 0, (counters + 1) * sizeof(int), stream) != cudaSuccess) {
    cudaGetLastError();
    return AIR_NOALLOC_LAUNCH_FAILED;
  }

  air::GemvWeight w{air::kFmtQ4K, w_tiled, nullptr, (int64_t)(K / 256) * 144};
  air::GemvEpiParams ep{};
  ep.mode = air::kEpiStore;
  ep.out_f32 = out;
  ep.ld_out = N;
  ep.err = err;
  air::GemvTiledScratch sc{ws, cnt};
  const char* e = air::launch_gemv_tiled(w, N, K, B, xq, static_cast<const float2*>(xds), ep, sc, splits, stream);
  if (e != nullptr || cudaGetLastError() != cudaSuccess) return AIR_NOALLOC_LAUNCH_FAILED;
  return AIR_NOALLOC_OK;
}

extern "C" __attribute__((visibility("default"))) const char* air_noalloc_status_string(int status) {
  switch (status) {
    case AIR_NOALLOC_OK: return "ok";
    case AIR_NOALLOC_BAD_ARGUMENT: return "bad argument (null pointer, err included; B not in [1, 8]; K not a multiple of 256; or N <= 0)";
    case AIR_NOALLOC_TOO_LARGE: return "N above 2,097,024 (16383 tiles of 128 rows): more tile counters than the static array's header holds";
    case AIR_NOALLOC_SETUP_FAILED: return "could not resolve the scratch array's device address on the current device";
    case AIR_NOALLOC_LAUNCH_FAILED: return "kernel launch or scratch clear failed";
    default: return "unknown status";
  }
}
