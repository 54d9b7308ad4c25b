#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace air {

struct SamplerArgs {
  const uint8_t* counts;          // [S, V] past-occurrence counts (null: no penalty)
  const int* count_row;           // [B] row of `counts` for each batch row (null: b)
  const uint32_t* allow_mask;     // [B, ceil(V/32)] grammar allow bits (null: all allowed)
  const float* temperature;       // [B] (null: greedy)
  const float* rep_penalty;       // [B]
  const int* top_k;               // [B]
  const float* top_p;             // [B]
  unsigned long long seed;
  long long* step;                // device step counter (Philox offset), bumped per call
  int* out_tokens;                // [B]
  float* out_prob;                // [B] probability of the chosen token's top-1 (optional)
  float4* part = nullptr;         // [B, sampler_chunks(V)] scratch for the multi-CTA pass (optional)
  // vocabulary-parallel partial pass: the logits are columns [v_off, v_off + V) of a V_total
  // vocabulary (counts and mask rows are V_total wide; v_off a multiple of 32)
  int v_off = 0;
  int v_total = 0;                // 0: V
};

int sampler_chunks(int V);

void launch_sampler(const float* logits, int B, int V, int64_t ld, const SamplerArgs& a,
                    cudaStream_t st);
// Greedy vocabulary-parallel sampling: each rank runs the partial pass over its logit shard
// (global indices, penalty and mask applied) into part[B, sampler_chunks(V_local)]; after an
// all-gather of the partials ([W, B, nch]) the merge takes each row's argmax (lowest index
// on ties, as the whole-vocabulary sampler) and bumps the step counter like launch_sampler.
void launch_sampler_partial(const float* logits, int B, int V, int nch, int64_t ld, const SamplerArgs& a,
                            cudaStream_t st);
void launch_sampler_greedy_merge(const float4* part_all, int W, int B, int nch, int* out_tokens,
                                 float* out_prob, long long* step, cudaStream_t st);
void launch_count_tokens(uint8_t* counts, int V, const int* tokens, int n, int per_row,
                         const int* count_row, cudaStream_t st);

}  // namespace air
