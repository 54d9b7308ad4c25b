// Fused tensor-parallel all-reduce over NVLink peer memory (one process per GPU).
//
// The reference sums row-parallel partials over a host TCP ring after O and down
// (src/model.rs:596-607,728-739, src/distributed.rs). Here the sum is split across the two
// kernels that already surround it:
//   * producer: the row-parallel projection (decode GEMV epilogue kEpiPeerPush, or
//     peer_push after the tcgen05 GEMM) stores every finished output element straight into
//     every rank's receive buffer over NVLink as one 8-byte (value, tag) store, so the
//     transfer overlaps the remaining tiles' math and needs no fence or flag;
//   * consumer: the RMSNorm that follows (reduce_rmsnorm_quant) reads its own buffer (local
//     memory), waits per element until the tag matches this collective (bounded), sums the
//     partials into the fp32 residual stream and normalises/quantises in the same pass.
// No extra launch on the GEMV path, no NCCL call, and each partial crosses NVLink once.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "kernels.h"

namespace air {

// Consumer side: the local receive buffer plus the local counters.
struct PeerReduce {
  const uint2* data;          // local receive buffer [2][world][slot_elems] (value, tag)
  int* epoch;                 // local collective counter (advanced here)
  int* done;                  // local CTA arrival counter (self-resetting)
  int* err;
  int64_t slot_elems;
  int world;
  int64_t timeout_ns;
};

// x[b, :] += sum over ranks of their partials (ld = K); then, as rmsnorm_quant, y = x *
// rsqrt(mean(x^2) + eps) * (w + w_offset) written as int8 Q8A (q, ds) and/or bf16 y.
// K <= 16384. One CTA per row.
void launch_reduce_rmsnorm_quant(const PeerReduce& r, float* x, const float* w, float w_offset, int B, int K,
                                 float eps, int8_t* q, float2* ds, void* y_bf16, cudaStream_t st);

// Push a finished fp32 partial [B, ld] (columns [0, N)) into every rank's receive slot
// (the tcgen05 GEMM path, whose epilogue writes locally first).
void launch_peer_push(const PeerPush& p, const float* src, int B, int N, int64_t ld, cudaStream_t st);

// Bytes of one rank's receive buffer.
inline int64_t peer_buffer_bytes(int world, int64_t slot_elems) { return 2LL * world * slot_elems * 8; }

}  // namespace air
