// Fused tensor-parallel all-reduce over NVLink peer memory (one process per GPU).
//
// The reference sums row-parallel partials over a host TCP ring after O and down
// (src/model.rs:596-607,728-739, src/distributed.rs). Here the sum is split across the two
// kernels that already surround it:
//   * producer: the row-parallel projection (decode GEMV epilogue kEpiPeerPush, or
//     peer_push after the tcgen05 GEMM) stores each finished 128-row output tile straight
//     into every rank's receive buffer over NVLink and raises one flag per tile there, so
//     the transfer overlaps the remaining tiles' math;
//   * consumer: the RMSNorm that follows (reduce_rmsnorm_quant) waits for all ranks' tile
//     flags in its own buffer (local memory, bounded wait), sums the partials into the
//     fp32 residual stream and normalises/quantises in the same pass.
// No extra launch, no NCCL call, and only this rank's share of bytes crosses each link.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "kernels.h"

namespace air {

// Consumer side: the local receive buffer plus the local counters.
struct PeerReduce {
  const float* data;          // local receive data base [2][world][slot_elems]
  const int* flags;           // local flags [world][max_tiles]
  int* epoch;                 // local collective counter (advanced here)
  int* done;                  // local CTA arrival counter (self-resetting)
  int* err;
  int64_t slot_elems;
  int world, max_tiles, ntiles;
  int64_t timeout_ns;
};

// x[b, :] += sum over ranks of their partials (ld = K); then, as rmsnorm_quant, y = x *
// rsqrt(mean(x^2) + eps) * (w + w_offset) written as int8 Q8A (q, ds) and/or bf16 y.
// K <= 16384. One CTA per row.
void launch_reduce_rmsnorm_quant(const PeerReduce& r, float* x, const float* w, float w_offset, int B, int K,
                                 float eps, int8_t* q, float2* ds, void* y_bf16, cudaStream_t st);

// Push a finished fp32 partial [B, ld] (columns [0, N)) into every rank's receive slot and
// raise the tile flags (the tcgen05 GEMM path, where the epilogue writes locally first).
void launch_peer_push(const PeerPush& p, const float* src, int B, int N, int64_t ld, cudaStream_t st);

// Bytes of one rank's receive buffer (flags region padded to 256 B, then the data).
inline int64_t peer_buffer_bytes(int world, int max_tiles, int64_t slot_elems) {
  const int64_t fb = ((int64_t)world * max_tiles * 4 + 255) / 256 * 256;
  return fb + 2LL * world * slot_elems * 4;
}
inline int64_t peer_flags_bytes(int world, int max_tiles) {
  return ((int64_t)world * max_tiles * 4 + 255) / 256 * 256;
}

}  // namespace air
