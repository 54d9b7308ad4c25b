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

AIR_DEVICE void st_tagged(uint2* p, float v, uint32_t tag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag) : "memory");
}
AIR_DEVICE uint2 ld_tagged(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

// Store element (b, c) of a partial, tagged epoch + 1, into region (parity, this rank) of
// the receive buffers: every rank's (one-shot) or the owner's of column c (two-shot). The
// peer loop is unrolled over the compile-time maximum so the pointer table stays in the
// parameter space.
AIR_DEVICE void peer_store(const PeerPush& p, int epoch, int64_t b, int64_t c, float v) {
  const int64_t region = ((int64_t)(epoch & 1) * p.world + p.rank) * p.slot_elems;
  const uint32_t tag = (uint32_t)epoch + 1u;
  if (p.shard > 0) {
    const int o = (int)(c / p.shard);
    const int64_t cl = c - (int64_t)o * p.shard;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r == o) st_tagged(p.data[r] + region + b * p.shard + cl, v, tag);
    return;
  }
  const int64_t off = region + b * p.row_len + c;
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r)
    if (r < p.world) st_tagged(p.data[r] + off, v, tag);
}

}  // namespace air
