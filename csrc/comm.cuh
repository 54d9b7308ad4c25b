// Device helpers of the fused tensor-parallel all-reduce (protocol in comm.h / kernels.h).
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace air {

AIR_DEVICE void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
AIR_DEVICE int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Store one partial-sum element into slot (parity, this rank) of every rank's buffer.
// The peer loop is unrolled over the compile-time maximum so the pointer table stays in
// the parameter space.
AIR_DEVICE void peer_store(const PeerPush& p, int par, int64_t idx, float v) {
  const int64_t off = ((int64_t)par * p.world + p.rank) * p.slot_elems + idx;
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r)
    if (r < p.world) p.data[r][off] = v;
}

// After every thread of the CTA has stored its elements of `tile`: make them visible
// system-wide, then raise this rank's flag for the tile on every rank.
AIR_DEVICE void peer_signal(const PeerPush& p, int tile, int epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < p.world) st_release_sys(p.flags[r] + p.rank * p.max_tiles + tile, epoch + 1);
  }
}

}  // namespace air
