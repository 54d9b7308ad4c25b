// Fused on-device sampler: repetition penalty, grammar mask, greedy argmax, temperature,
// exact top-k (radix select), top-p nucleus and a seeded Philox draw — one CTA per row, after
// a pass that spreads each row's argmax and softmax denominator over many CTAs (one per 1024
// vocabulary entries), so a greedy step does not stream the vocabulary through one SM.
//
// Semantics follow the reference sampler (src/sampler.rs:83-164, 272-292): the penalty
// divides positive / multiplies negative logits once per past occurrence of a token
// (prompt and BOS included, so we keep an occurrence count per token), the mask is
// applied before temperature, greedy when T <= 0, softmax over the whole vocabulary,
// top-k then top-p on those probabilities (cumsum >= p keeps the crossing token), and a
// draw over the renormalised survivors. The reference's RNG is unseeded; ours is Philox
// keyed by (seed, row, step), so sampled output is reproducible.
#include <curand_kernel.h>
#include "common.cuh"
#include "sampler.h"

namespace air {

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxK = 1024;

AIR_DEVICE uint32_t ordered(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

AIR_DEVICE float penalised(float v, int c, float pen) {
  if (c == 0 || pen == 1.f) return v;
  const float f = __powf(pen, (float)c);
  return v > 0.f ? v / f : v * f;
}

constexpr int kChunk = 1024;          // vocabulary entries per CTA of the partial pass
constexpr int kPartThreads = 256;

struct RowView {
  const float* lg;
  const uint8_t* cnt;
  const uint32_t* mask;
  float pen;
  AIR_DEVICE float value(int i) const {
    float v = lg[i];
    if (cnt) v = penalised(v, cnt[i], pen);
    if (mask && !((mask[i >> 5] >> (i & 31)) & 1u)) v = -INFINITY;
    return v;
  }
};

AIR_DEVICE RowView row_view(const float* logits, int V, int64_t ld, const SamplerArgs& a, int row) {
  RowView r;
  const int vt = a.v_total > 0 ? a.v_total : V;   // counts / mask row width
  r.lg = logits + (size_t)row * ld;
  r.cnt = a.counts ? a.counts + (size_t)(a.count_row ? a.count_row[row] : row) * vt + a.v_off : nullptr;
  r.mask = a.allow_mask ? a.allow_mask + (size_t)row * ((vt + 31) / 32) + a.v_off / 32 : nullptr;
  r.pen = a.rep_penalty ? a.rep_penalty[row] : 1.f;
  return r;
}

AIR_DEVICE void argmax_merge(float& best, int& besti, float ov, int oi) {
  if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
}

// Pass over one vocabulary chunk of one row, spread over many CTAs: (max, argmax, and with a
// temperature the softmax denominator relative to the chunk max) -> part[row][chunk].
__global__ void __launch_bounds__(kPartThreads)
sampler_partial_kernel(const float* __restrict__ logits, int V, int64_t ld, SamplerArgs a, int nch) {
  const int chunk = blockIdx.x, row = blockIdx.y;
  const RowView rv = row_view(logits, V, ld, a, row);
  const float temp = a.temperature ? a.temperature[row] : 0.f;
  const int i0 = chunk * kChunk, i1 = min(V, i0 + kChunk);
  constexpr int kPer = kChunk / kPartThreads;
  float v[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = i0 + threadIdx.x + j * kPartThreads;
    v[j] = i < i1 ? rv.value(i) : -INFINITY;
  }
  float best = -INFINITY;
  int besti = 0x7fffffff;
#pragma unroll
  for (int j = 0; j < kPer; ++j) argmax_merge(best, besti, v[j], i0 + threadIdx.x + j * kPartThreads);
  __shared__ float red[32];
  __shared__ int redi[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_merge(best, besti, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, besti, o));
  if (lane == 0) { red[wid] = best; redi[wid] = besti; }
  __syncthreads();
  best = red[0];
  besti = redi[0];
  for (int w = 1; w < kPartThreads / 32; ++w) argmax_merge(best, besti, red[w], redi[w]);
  float z = 0.f;
  if (temp > 1e-6f && best != -INFINITY) {
    const float inv_t = 1.f / temp;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (v[j] != -INFINITY) z += __expf((v[j] - best) * inv_t);
    __syncthreads();
    z = block_sum(z, red);
  }
  if (threadIdx.x == 0)
    a.part[(size_t)row * nch + chunk] =
        make_float4(best, __int_as_float(besti == 0x7fffffff ? besti : besti + a.v_off), z, 0.f);
}

// one warp per row: argmax over the W x nch gathered partials (global indices)
__global__ void sampler_greedy_merge_kernel(const float4* __restrict__ part, int W, int B, int nch,
                                            int* __restrict__ out_tokens, float* __restrict__ out_prob) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= B) return;
  float best = -INFINITY;
  int besti = 0x7fffffff;
  for (int j = lane; j < W * nch; j += 32) {
    const int w = j / nch, c = j % nch;
    const float4 p = part[((size_t)w * B + row) * nch + c];
    argmax_merge(best, besti, p.x, __float_as_int(p.y));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    argmax_merge(best, besti, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, besti, o));
  if (lane == 0) {
    out_tokens[row] = besti == 0x7fffffff ? 0 : besti;
    if (out_prob) out_prob[row] = 1.f;
  }
}

__global__ void __launch_bounds__(kThreads)
sampler_kernel(const float* __restrict__ logits, int V, int64_t ld, SamplerArgs a) {
  const int row = blockIdx.x;
  const float* lg = logits + (size_t)row * ld;
  const uint8_t* cnt = a.counts ? a.counts + (size_t)(a.count_row ? a.count_row[row] : row) * V : nullptr;
  const uint32_t* mask = a.allow_mask ? a.allow_mask + (size_t)row * ((V + 31) / 32) : nullptr;
  const float temp = a.temperature ? a.temperature[row] : 0.f;
  const float pen = a.rep_penalty ? a.rep_penalty[row] : 1.f;
  const int topk_req = a.top_k ? a.top_k[row] : 0;
  const float topp = a.top_p ? a.top_p[row] : 1.f;

  __shared__ float red[32];
  __shared__ int redi[32];
  __shared__ uint32_t hist[256];
  __shared__ float cand_v[kMaxK];
  __shared__ int cand_i[kMaxK];
  __shared__ int n_cand, n_eq_taken;
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;

  auto value = [&](int i) -> float {
    float v = lg[i];
    if (cnt) v = penalised(v, cnt[i], pen);
    if (mask && !((mask[i >> 5] >> (i & 31)) & 1u)) v = -INFINITY;
    return v;
  };

  // ---- pass 1: argmax (lowest index on ties) and max (from the chunk partials if any) ----
  float best = -INFINITY;
  int besti = 0x7fffffff;
  const int nch = (V + kChunk - 1) / kChunk;
  if (a.part) {
    for (int c = threadIdx.x; c < nch; c += kThreads) {
      const float4 p = a.part[(size_t)row * nch + c];
      argmax_merge(best, besti, p.x, __float_as_int(p.y));
    }
  } else {
    for (int i = threadIdx.x; i < V; i += kThreads) {
      const float v = value(i);
      if (v > best || (v == best && i < besti)) { best = v; besti = i; }
    }
  }
  {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
    }
    if (lane == 0) { red[wid] = best; redi[wid] = besti; }
    __syncthreads();
    if (wid == 0) {
      best = red[lane];
      besti = redi[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ov > best || (ov == best && oi < besti)) { best = ov; besti = oi; }
      }
      if (lane == 0) { red[0] = best; redi[0] = besti; }
    }
    __syncthreads();
    best = red[0];
    besti = redi[0];
    __syncthreads();
  }
  if (temp <= 1e-6f || best == -INFINITY) {
    if (threadIdx.x == 0) {
      a.out_tokens[row] = besti == 0x7fffffff ? 0 : besti;
      if (a.out_prob) a.out_prob[row] = 1.f;
    }
    return;
  }
  const float inv_t = 1.f / temp;
  // ---- softmax denominator over the whole vocabulary ----
  float z = 0.f;
  if (a.part) {
    for (int c = threadIdx.x; c < nch; c += kThreads) {
      const float4 p = a.part[(size_t)row * nch + c];
      if (p.x != -INFINITY) z += p.z * __expf((p.x - best) * inv_t);
    }
  } else {
    for (int i = threadIdx.x; i < V; i += kThreads) {
      const float v = value(i);
      if (v != -INFINITY) z += __expf((v - best) * inv_t);
    }
  }
  z = block_sum(z, red);
  // ---- exact k-th largest by 4 x 8-bit radix select ----
  int k = topk_req > 0 ? min(topk_req, V) : V;
  k = min(k, kMaxK);
  if (threadIdx.x == 0) { s_prefix = 0; s_remaining = k; n_cand = 0; n_eq_taken = 0; }
  __syncthreads();
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    const uint32_t hmask = pass == 0 ? 0u : (0xFFFFFFFFu << (32 - 8 * pass));
    for (int i = threadIdx.x; i < V; i += kThreads) {
      const uint32_t u = ordered(value(i));
      if ((u & hmask) == (prefix & hmask)) atomicAdd(&hist[(u >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int rem = s_remaining;
      int dgt = 255;
      for (; dgt > 0; --dgt) {
        if ((int)hist[dgt] >= rem) break;
        rem -= hist[dgt];
      }
      s_prefix = prefix | ((uint32_t)dgt << shift);
      s_remaining = rem;
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;     // ordered value of the k-th largest
  const int eq_needed = s_remaining; // how many elements equal to thr belong to the top-k
  for (int i = threadIdx.x; i < V; i += kThreads) {
    const float v = value(i);
    const uint32_t u = ordered(v);
    bool take = u > thr;
    if (!take && u == thr) take = atomicAdd(&n_eq_taken, 1) < eq_needed;
    if (take) {
      const int slot = atomicAdd(&n_cand, 1);
      if (slot < kMaxK) { cand_v[slot] = v; cand_i[slot] = i; }
    }
  }
  __syncthreads();
  const int nc = min(n_cand, kMaxK);
  for (int i = threadIdx.x; i < kMaxK; i += kThreads) {
    if (i >= nc) { cand_v[i] = -INFINITY; cand_i[i] = 0x7fffffff; }
  }
  __syncthreads();
  // ---- bitonic sort, descending by value, ascending index on ties ----
  for (int size = 2; size <= kMaxK; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const int i = threadIdx.x;
      const int j = i ^ stride;
      if (j > i && i < kMaxK) {
        const bool desc = (i & size) == 0;
        const float vi = cand_v[i], vj = cand_v[j];
        const int ii = cand_i[i], ij = cand_i[j];
        const bool i_first = vi > vj || (vi == vj && ii < ij);
        if (desc != i_first) {
          cand_v[i] = vj; cand_v[j] = vi;
          cand_i[i] = ij; cand_i[j] = ii;
        }
      }
      __syncthreads();
    }
  }
  // ---- top-p, renormalise, draw (single thread; nc <= 1024) ----
  if (threadIdx.x == 0) {
    float cum = 0.f;
    int keep = nc;
    for (int i = 0; i < nc; ++i) {
      cum += __expf((cand_v[i] - best) * inv_t) / z;
      if (topp < 1.f && cum >= topp) { keep = i + 1; break; }
    }
    float total = 0.f;
    for (int i = 0; i < keep; ++i) total += __expf((cand_v[i] - best) * inv_t) / z;
    int tok = cand_i[0];
    if (total > 0.f) {
      curandStatePhilox4_32_10_t st;
      curand_init(a.seed, (unsigned long long)row, a.step ? (unsigned long long)(*a.step) * 4ull : 0ull, &st);
      const float r = curand_uniform(&st) * total;
      float c = 0.f;
      for (int i = 0; i < keep; ++i) {
        c += __expf((cand_v[i] - best) * inv_t) / z;
        if (c >= r) { tok = cand_i[i]; break; }
      }
    }
    a.out_tokens[row] = tok;
    if (a.out_prob) a.out_prob[row] = (total > 0.f) ? (__expf((cand_v[0] - best) * inv_t) / z) / total : 1.f;
  }
}

// counts[row, tok] += 1 (saturating at 255) for each new token; used after sampling.
__global__ void count_tokens_kernel(uint8_t* counts, int V, const int* tokens, int n, int per_row,
                                    const int* count_row) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int row = per_row > 0 ? i / per_row : i;
  if (count_row) row = count_row[row];
  const int t = tokens[i];
  if (t < 0 || t >= V || row < 0) return;
  uint8_t* c = counts + (size_t)row * V + t;
  // byte atomics are not available: use a 32-bit CAS on the containing word
  unsigned int* w = reinterpret_cast<unsigned int*>(reinterpret_cast<uintptr_t>(c) & ~(uintptr_t)3);
  const int sh = (int)(reinterpret_cast<uintptr_t>(c) & 3) * 8;
  unsigned int old = *w, assumed;
  do {
    assumed = old;
    const unsigned int b = (assumed >> sh) & 0xFF;
    if (b == 255) break;
    old = atomicCAS(w, assumed, assumed + (1u << sh));
  } while (old != assumed);
}

__global__ void bump_step_kernel(long long* step) { *step += 1; }

}  // namespace

void launch_sampler(const float* logits, int B, int V, int64_t ld, const SamplerArgs& a,
                    cudaStream_t st) {
  if (a.part) {
    const int nch = (V + kChunk - 1) / kChunk;
    sampler_partial_kernel<<<dim3(nch, B), kPartThreads, 0, st>>>(logits, V, ld, a, nch);
  }
  sampler_kernel<<<B, kThreads, 0, st>>>(logits, V, ld, a);
  if (a.step) bump_step_kernel<<<1, 1, 0, st>>>(a.step);
}

int sampler_chunks(int V) { return (V + kChunk - 1) / kChunk; }

void launch_sampler_partial(const float* logits, int B, int V, int nch, int64_t ld, const SamplerArgs& a,
                            cudaStream_t st) {
  // nch >= chunks of V: the layout's chunk count (chunks past V write (-inf, INT_MAX))
  sampler_partial_kernel<<<dim3(nch, B), kPartThreads, 0, st>>>(logits, V, ld, a, nch);
}

void launch_sampler_greedy_merge(const float4* part_all, int W, int B, int nch, int* out_tokens,
                                 float* out_prob, long long* step, cudaStream_t st) {
  sampler_greedy_merge_kernel<<<(B + 7) / 8, 256, 0, st>>>(part_all, W, B, nch, out_tokens, out_prob);
  if (step) bump_step_kernel<<<1, 1, 0, st>>>(step);
}

void launch_count_tokens(uint8_t* counts, int V, const int* tokens, int n, int per_row,
                         const int* count_row, cudaStream_t st) {
  if (n <= 0) return;
  count_tokens_kernel<<<(n + 255) / 256, 256, 0, st>>>(counts, V, tokens, n, per_row, count_row);
}

}  // namespace air
