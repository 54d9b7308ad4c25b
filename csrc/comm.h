// Fused tensor-parallel all-reduce over NVLink peer memory (one process per GPU).
//
// The reference sums row-parallel partials over a host TCP ring after O and down
// (src/model.rs:596-607,728-739, src/distributed.rs). Here the sum is split across the two
// kernels that already surround it:
//   * producer: the row-parallel projection (decode GEMV epilogue kEpiPeerPush, the tcgen05
//     GEMM epilogue kGemmPeerPush, or peer_push after another kernel) stores every finished
//     output element over NVLink as one 8-byte (value, tag) store, so the transfer overlaps
//     the remaining tiles' math and needs no fence or flag;
//   * consumer: the RMSNorm that follows (tp_reduce_norm) waits per element until the tag
//     matches this collective (bounded), sums the partials into the fp32 residual stream and
//     normalises / quantises in the same pass.
// Two data paths (PeerPush::shard):
//   * one-shot: every producer writes its whole partial into every rank's buffer; each
//     consumer sums the world partials locally. One NVLink hop of latency, (world - 1) x the
//     partial's bytes out of each rank: best for small batches.
//   * two-shot (reduce-scatter + all-gather): a producer writes column c only to its owner
//     (c / shard). The owner's consumer sums its columns, adds the residual and writes the
//     new residual values, tagged, into every rank's all-gather region; every consumer then
//     waits for its whole row there and normalises. Two hops, 2 (world - 1) / world x the
//     partial's bytes out of each rank: best for large batches at 4 and 8 GPUs.
// No NCCL call, and every wait is on local memory.
// A third path (TPReduceArgs::nvls) uses NVLink SHARP: each producer stores its fp32 partial
// into its own slot of a multicast-bound symmetric buffer (plain local stores); the consumer
// CTA of row b raises row b's arrival flag on every rank, waits for every rank's flag, and
// reads the row with multimem.ld_reduce, so the NVSwitch returns the sum of all ranks' partials:
// one load per element, no per-rank partial crosses NVLink more than once.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "kernels.h"

namespace air {

// One rank's consumer state. The receive buffer is [2][world][slot_elems] (partials) then
// [2][slot_elems] (all-gather region, two-shot); ag_peer[r] is rank r's all-gather region.
struct TPReduceRank {
  const uint2* rs;            // local partial region
  const uint2* ag;            // local all-gather region
  uint2* ag_peer[kMaxPeers];  // every rank's all-gather region (mapped here)
  int* epoch;                 // local collective counter (advanced here)
  int* done;                  // local CTA arrival counter (self-resetting)
  int* err;
  float* x;                   // [B, K] fp32 residual stream (replicated on every rank)
  int8_t* q;                  // optional Q8A output [B, K]
  float2* ds;                 //   and its (d, d * sum) per 32 [B, K / 32]
  void* y_bf16;               // optional bf16 output [B, K]
  int rank;
  // NVLS mode: multicast address of this collective's partial region [rows][K] f32 (every
  // rank's copy, reduced by the switch on load), and the row arrival flags [rows][world]
  // of this rank (local) and of every rank (mapped here)
  const float* mc;
  int* flags;
  int* flags_peer[kMaxPeers];
};

struct TPReduceArgs {
  TPReduceRank r[kMaxPeers];  // ranks handled by this launch (several only when emulated)
  int n_local;                // ranks in this launch (gridDim.z); 1 on a real TP group
  int world;
  int64_t slot_elems;
  int64_t shard;              // two-shot columns per rank (0 = one-shot)
  int64_t timeout_ns;
  const float* w;             // norm weight [K] (null: no normalisation)
  float w_offset;
  const float* bias;          // optional norm bias [K]
  int layer;                  // 1: LayerNorm (mean subtracted), 0: RMSNorm
  float eps;
  int B, K;
  int nvls;                   // 1: partials in symmetric memory, summed by multimem.ld_reduce
};

// x[b, :] += sum over ranks of their partials; then y = x * rsqrt(mean(x^2) + eps) *
// (w + w_offset) written as Q8A (q, ds) and/or bf16. K <= 16384, one CTA per row and rank.
void launch_tp_reduce_norm(const TPReduceArgs& a, cudaStream_t st);

// Push a finished fp32 partial [B, ld] (columns [0, N)) into the receive buffers.
void launch_peer_push(const PeerPush& p, const float* src, int B, int N, int64_t ld, cudaStream_t st);

// Elements of one rank's receive buffer (partials + all-gather region) and its bytes.
inline int64_t peer_buffer_elems(int world, int64_t slot_elems) { return 2LL * world * slot_elems + 2LL * slot_elems; }
inline int64_t peer_buffer_bytes(int world, int64_t slot_elems) { return peer_buffer_elems(world, slot_elems) * 8; }

}  // namespace air
