// Host-side launch API of the air_rs CUDA kernels (no torch headers here, so the .cu
// files compile quickly; csrc/bindings.cpp adapts these to torch tensors).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace air {

// ---- weight formats understood by the decode GEMVs ----
enum WeightFormat : int {
  kFmtQ4K = 0,    // raw GGUF Q4_K blocks, [N, K/256*144] bytes
  kFmtQ8_0 = 1,   // repacked Q8_0: int8 qs [N, K] + f16 scales [N, K/32]
  kFmtBF16 = 2,   // dense bf16 [N, K]
  kFmtFP8 = 3,    // E4M3 codes [N, K] + f32 multiplier per row and 128-wide K block (GEMM only)
};

enum GemvEpilogue : int {
  kEpiStore = 0,      // out[b, n] = acc (fp32 or bf16)
  kEpiResidual = 1,   // resid[b, n] += acc (fp32 residual stream)
  kEpiSwiGLU = 2,     // out[b, n] = silu(W·x)[n] * (W2·x)[n]
  kEpiQKVRope = 3,    // rows = [q | k | v]; NeoX RoPE on q,k; k,v written to the paged cache
  kEpiPeerPush = 4,   // tensor-parallel partial: stored into every rank's receive slot over
                      // NVLink as tagged 8-byte elements (see comm.h)
};

constexpr int kMaxPeers = 8;

// Producer side of the fused tensor-parallel all-reduce (protocol in comm.h). Every rank
// owns one receive buffer, mapped into every peer process, of 8-byte (value, tag) elements
// carrying tag = epoch + 1, so a reader that sees the tag also sees the value (no fence, no
// separate flag). Its first region is [2 parities][world][slot_elems]; a producer writes
// element (b, c) of its [B, row_len] partial into region (parity, its rank) of
//   * one-shot (shard == 0): EVERY rank's buffer, at b * row_len + c;
//   * two-shot (shard > 0): only the buffer of the rank that owns column c
//     (owner = c / shard), at b * shard + c % shard: a reduce-scatter, each element
//     crossing NVLink once to one rank.
// `epoch` is the local collective counter, advanced by the consumer once all of its CTAs
// have read it.
struct PeerPush {
  uint2* data[kMaxPeers];     // per destination rank: its receive buffer (mapped here)
  const int* epoch;           // this rank's collective counter
  int64_t slot_elems;
  int64_t row_len;            // columns of one partial row (the hidden size)
  int64_t shard;              // two-shot: columns owned per rank (0 = one-shot)
  int world, rank;
};

struct GemvWeight {
  int fmt;
  const void* data;      // q4k blocks / q8 qs / bf16 values
  const void* scales;    // q8_0 f16 scales (else null)
  int64_t row_bytes;     // bytes per row of `data`
};

struct GemvEpiParams {
  int mode;
  float* out_f32;             // [B, ld_out]
  void* out_bf16;             // [B, ld_out]
  int64_t ld_out;
  float* resid;               // [B, ld_out]
  // SwiGLU second operand
  GemvWeight w2;
  // QKV + RoPE
  const float2* rope_cs;      // [max_pos, rot_dim/2] (cos, sin)
  const int* positions;       // [B]
  const int64_t* slots;       // [B] paged-cache slot (block*block_size + off); <0 = skip
  void* kv_cache;             // this layer: [num_blocks, 2, n_kv, block_size, head_dim] bf16
  float* q_out;               // [B, n_heads, head_dim] fp32
  int n_heads, n_kv, head_dim, block_size, rot_dim;
  int64_t num_blocks;
  int* err;
  PeerPush push;              // kEpiPeerPush
  // kEpiSwiGLU on the tiled Q4_K path: also (or only) write the product quantised to Q8A
  // (int8 [B, q_k] + float2 [B, q_k/32]) for the next GEMV; rows N..q_k are zero.
  int8_t* out_q;
  float2* out_ds;
  int q_k;
  // RMSNorm folded into the decode GEMV chain (tiled Q4_K path). Producer (kEpiResidual with
  // norm_w): after x += W.h, write Q8A of x * (norm_w + norm_offset) to out_q / out_ds and each
  // 32-row group's sum of x^2 to ss_out[b][row / 32]. Consumer (ss_in, norm_k = row length):
  // outputs are scaled by rsqrt(sum(ss_in[b]) / norm_k + eps) before the epilogue (the scale
  // is linear in the quantised input). Sums are taken in a fixed order (deterministic).
  const float* norm_w;
  float norm_offset;
  float* ss_out;
  const float* ss_in;
  int norm_k;
  float eps;
  int act;                    // kEpiSwiGLU gate activation (GateAct): SiLU or GELU (GeGLU)
};

// x: activations quantised by rmsnorm_quant (int8 [B,K] + float2 [B,K/32]).
void launch_gemv(const GemvWeight& w, int N, int K, int B, const int8_t* xq, const float2* xds,
                 const GemvEpiParams& ep, cudaStream_t st);

// layer = 0: RMSNorm, y = x * rsqrt(mean(x^2) + eps) * (w + w_offset) (+ bias);
// layer = 1: LayerNorm, y = (x - mean) * rsqrt(var + eps) * (w + w_offset) (+ bias).
void launch_rmsnorm_quant(const float* x, const void* x_bf16, const float* w, float w_offset,
                          const float* bias, int layer, int B, int K, float eps, int8_t* q, float2* ds,
                          void* y_bf16, cudaStream_t st);

}  // namespace air
