// Paged attention over the HBM block-table KV pool (decode, chunked prefill and
// speculative tree verify share this kernel).
//
// Each CTA owns (query row r, KV head h, split s): the G = n_heads / n_kv query heads of
// the GQA group are scored together so every K/V byte is read once per group. Keys of
// one split are processed 32 at a time per warp with an online softmax; partial
// (max, sum, o) triples of the warps and then of the splits are merged with the
// log-sum-exp rule. This is the reference's FlashDecoding split-K math
// (src/flash_decode.rs:70-176) on the paged layout of src/paged_attention.rs (block 16),
// with causal / sliding-window / tree-ancestor visibility (src/ops.rs:762-845).
//
// KV layer layout: [num_blocks, 2 (K,V), n_kv, block_size, row]: a row is head_dim bf16, or
// (F8) head_dim E4M3 codes + f32 scale + padding (kv_f8.cuh).
#include "common.cuh"
#include "attention.h"
#include "kv_f8.cuh"
#include <stdlib.h>

namespace air {

namespace {

constexpr int kD = 128;          // head_dim supported by the fast path (64 also instantiated)
constexpr int kWarps = 4;
constexpr int kTPW = 16;            // keys per warp per iteration (4 per pass, 8 lanes per key)
constexpr int kNI = kTPW / 4;

template <int D>
struct Frag;  // per-lane slice sizes for a head dim

AIR_DEVICE bool key_visible(int t, const AttnRows& rows, int r, int ctx) {
  if (t >= ctx) return false;
  if (rows.window > 0 && t < ctx - rows.window) return false;
  if (rows.tree_base) {
    const int tb = rows.tree_base[r];
    if (t >= tb) {
      const int k = t - tb;
      if (k >= 64) return false;
      return (rows.tree_mask[r] >> k) & 1ull;
    }
  }
  return true;
}

// D = head dim; G = query heads per KV head (GQA group); F8: fp8 pool rows.
template <int D, int G, bool F8>
__global__ void __launch_bounds__(kWarps * 32)
paged_attn_kernel(const float* __restrict__ q, const uint8_t* __restrict__ kv,
                  const int* __restrict__ block_tables, int max_blocks, AttnRows rows,
                  int n_heads, int n_kv, int block_size, int64_t num_blocks, int n_splits,
                  int split_tokens, float scale, float* __restrict__ part_o,
                  float2* __restrict__ part_ml, float* __restrict__ out, int* err) {
  constexpr int DL = D / 32;        // dims per lane in the PV phase
  constexpr int TG = D / 16;        // 16 dims per lane-in-group in the QK phase (8 lanes/token)
  static_assert(D == 64 || D == 128, "head dim");
  __shared__ float q_s[G][D];
  __shared__ float red_m[kWarps][G], red_l[kWarps][G];
  __shared__ float red_o[kWarps][G][D];

  const int h = blockIdx.x, r = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = rows.row_seq ? rows.row_seq[r] : r;
  const int ctx = rows.ctx_len[r];
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    q_s[g][d] = q[((size_t)r * n_heads + h * G + g) * D + d] * scale;
  }
  __syncthreads();

  // split_tokens <= 0: divide this row's context evenly over the splits (multiple of kTPW),
  // so one captured launch serves every context length.
  const int st = split_tokens > 0 ? split_tokens
                                  : max(64, ((ctx + n_splits - 1) / n_splits + kTPW - 1) / kTPW * kTPW);
  int t_begin = split * st;
  int t_end = min(ctx, t_begin + st);
  if (rows.window > 0) t_begin = max(t_begin, ctx - rows.window);

  float m[G], l[G], acc[G][DL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < DL; ++j) acc[g][j] = 0.f;
  }
  const int* bt = block_tables + (size_t)seq * max_blocks;
  constexpr size_t kRowB = F8 ? kv_f8_row_bytes(D) : D * 2;        // bytes per (token, head) row
  const size_t head_stride = (size_t)block_size * kRowB;           // one head of one block
  const size_t kv_stride = (size_t)n_kv * head_stride;             // K -> V
  const size_t blk_stride = 2 * kv_stride;

  const int grp = lane >> 3, gl = lane & 7;   // QK phase: 4 tokens per pass, 8 lanes per token
  constexpr int KU = D / 64;                   // uint4 of K per lane per token
  for (int c0 = t_begin + warp * kTPW; c0 < t_end; c0 += kWarps * kTPW) {
    // ---- issue every K and V load of this 32-token chunk before any math ----
    uint4 kreg[kNI][KU];
    uint2 vreg[kNI][4];   // [i][gg]: V slice of token c0 + 4i + gg
    float ksc[kNI], vsc[kNI][4];   // F8 row scales
    bool kval[kNI];
#pragma unroll
    for (int i = 0; i < kNI; ++i) {
      const int t = c0 + 4 * i + grp;
      kval[i] = false;
      ksc[i] = 0.f;
#pragma unroll
      for (int u = 0; u < KU; ++u) kreg[i][u] = make_uint4(0, 0, 0, 0);
      if (t < t_end) {
        const int b = bt[t / block_size];
        if (b < 0 || b >= num_blocks) {
          set_error(err, kErrBounds);
        } else {
          kval[i] = true;
          const uint8_t* rp = kv + (size_t)b * blk_stride + h * head_stride + (size_t)(t % block_size) * kRowB;
          if constexpr (F8) {
            if constexpr (D == 128) {
              kreg[i][0] = __ldg(reinterpret_cast<const uint4*>(rp + gl * 16));
            } else {
              const uint2 c = __ldg(reinterpret_cast<const uint2*>(rp + gl * 8));
              kreg[i][0] = make_uint4(c.x, c.y, 0u, 0u);
            }
            ksc[i] = __ldg(reinterpret_cast<const float*>(rp + D));
          } else {
            const uint4* kp = reinterpret_cast<const uint4*>(rp + gl * (D / 8) * 2);
#pragma unroll
            for (int u = 0; u < KU; ++u) kreg[i][u] = __ldg(kp + u);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kNI; ++i) {
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) {
        const int t = c0 + 4 * i + gg;
        vreg[i][gg] = make_uint2(0, 0);
        vsc[i][gg] = 0.f;
        if (t < t_end) {
          const int b = bt[t / block_size];
          if (b >= 0 && b < num_blocks) {
            const uint8_t* rp = kv + (size_t)b * blk_stride + kv_stride + h * head_stride +
                                (size_t)(t % block_size) * kRowB;
            if constexpr (F8) {
              if (DL == 4) vreg[i][gg].x = __ldg(reinterpret_cast<const uint32_t*>(rp + lane * DL));
              else vreg[i][gg].x = __ldg(reinterpret_cast<const uint16_t*>(rp + lane * DL));
              vsc[i][gg] = __ldg(reinterpret_cast<const float*>(rp + D));
            } else {
              const __nv_bfloat16* vp = reinterpret_cast<const __nv_bfloat16*>(rp) + lane * DL;
              if (DL == 4) vreg[i][gg] = __ldg(reinterpret_cast<const uint2*>(vp));
              else vreg[i][gg].x = *reinterpret_cast<const uint32_t*>(vp);
            }
          }
        }
      }
    }
    // ---- scores for tokens c0 .. c0+kTPW-1: s[i][g] for token c0 + 4*i + grp ----
    float s[kNI][G];
#pragma unroll
    for (int i = 0; i < kNI; ++i) {
      const int t = c0 + 4 * i + grp;
      const bool vis = kval[i] && key_visible(t, rows, r, ctx);
      float part[G];
#pragma unroll
      for (int g = 0; g < G; ++g) part[g] = 0.f;
      if constexpr (F8) {
        constexpr int NE = D / 8;           // codes of this lane: 16 (D 128) or 8 (D 64)
        const uint32_t* w = reinterpret_cast<const uint32_t*>(&kreg[i][0]);
        float kf[NE];
#pragma unroll
        for (int e = 0; e < NE; e += 2) {
          const float2 f = e4m3x2_to_f2(w[e >> 2] >> (8 * (e & 3)));
          kf[e] = f.x;
          kf[e + 1] = f.y;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int e = 0; e < NE; ++e) part[g] += kf[e] * q_s[g][gl * NE + e];
          part[g] *= ksc[i];
        }
      } else {
#pragma unroll
        for (int u = 0; u < KU; ++u) {
          float kf[8];
          bf16x8_to_f32(kreg[i][u], kf);
#pragma unroll
          for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int e = 0; e < 8; ++e) part[g] += kf[e] * q_s[g][gl * (D / 8) + u * 8 + e];
          }
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float v = part[g];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        s[i][g] = vis ? soft_cap(v, rows.softcap) : -INFINITY;
      }
    }
    // ---- online softmax ----
    float p[kNI][G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kNI; ++i) mx = fmaxf(mx, s[i][g]);
      mx = warp_max(mx);
      const float mnew = fmaxf(m[g], mx);
      const float alpha = (mnew == -INFINITY) ? 1.f : __expf(m[g] - mnew);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < kNI; ++i) {
        p[i][g] = (s[i][g] == -INFINITY) ? 0.f : __expf(s[i][g] - mnew);
        sum += p[i][g];
      }
      // every token's p is replicated over its 8 lanes: divide the warp sum by 8
      sum = warp_sum(sum) * 0.125f;
      l[g] = l[g] * alpha + sum;
      m[g] = mnew;
#pragma unroll
      for (int j = 0; j < DL; ++j) acc[g][j] *= alpha;
    }
    // ---- o += p . V (V already in registers; invisible / absent tokens have p = 0) ----
#pragma unroll
    for (int i = 0; i < kNI; ++i) {
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) {
        float pv[G];
#pragma unroll
        for (int g = 0; g < G; ++g) pv[g] = __shfl_sync(0xffffffffu, p[i][g], gg * 8);
        float vf[4];
        if constexpr (F8) {
          const float2 a0 = e4m3x2_to_f2(vreg[i][gg].x), a1 = e4m3x2_to_f2(vreg[i][gg].x >> 16);
          const float sv = vsc[i][gg];
          vf[0] = a0.x * sv; vf[1] = a0.y * sv; vf[2] = a1.x * sv; vf[3] = a1.y * sv;
        } else {
          const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&vreg[i][gg]);
          const float2 a0 = __bfloat1622float2(hh[0]), a1 = __bfloat1622float2(hh[1]);
          vf[0] = a0.x; vf[1] = a0.y; vf[2] = a1.x; vf[3] = a1.y;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int j = 0; j < DL; ++j) acc[g][j] += pv[g] * vf[j];
        }
      }
    }
  }
  // ---- merge the warps of this CTA ----
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) { red_m[warp][g] = m[g]; red_l[warp][g] = l[g]; }
#pragma unroll
    for (int j = 0; j < DL; ++j) red_o[warp][g][lane * DL + j] = acc[g][j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red_m[w][g]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = (red_m[w][g] == -INFINITY) ? 0.f : __expf(red_m[w][g] - M);
      L += red_l[w][g] * f;
      O += red_o[w][g][d] * f;
    }
    const int head = h * G + g;
    if (n_splits == 1) {
      out[((size_t)r * n_heads + head) * D + d] = L > 0.f ? O / L : 0.f;
    } else {
      const size_t pi = ((size_t)r * n_heads + head) * n_splits + split;
      part_o[pi * D + d] = O;
      if (d == 0) part_ml[pi] = make_float2(M, L);
    }
  }
}

constexpr int kMaxMergeSplits = 256;

// Merge split partials; optionally quantise the output rows to int8 per 32 (Q8A).
template <int D>
__global__ void __launch_bounds__(D)
attn_merge_kernel(const float* __restrict__ part_o, const float2* __restrict__ part_ml,
                  int n_heads, int n_splits, float* __restrict__ out, int8_t* __restrict__ oq,
                  float2* __restrict__ ods, __nv_bfloat16* __restrict__ ob) {
  pdl_trigger();   // a dependent GEMV may start streaming its weights now
  const int head = blockIdx.x, r = blockIdx.y, d = threadIdx.x;
  const size_t base = ((size_t)r * n_heads + head) * n_splits;
  // split statistics staged once (one load per thread) instead of a serial chain per thread
  __shared__ float2 sml[kMaxMergeSplits];
  for (int s = d; s < n_splits; s += D) sml[s] = part_ml[base + s];
  __syncthreads();
  float M = -INFINITY;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, sml[s].x);
  float L = 0.f, O = 0.f;
#pragma unroll 8
  for (int s = 0; s < n_splits; ++s) {
    const float2 ml = sml[s];
    if (ml.x == -INFINITY) continue;       // a split that received no keys
    const float f = __expf(ml.x - M);
    L += ml.y * f;
    O += part_o[(base + s) * D + d] * f;
  }
  const float v = L > 0.f ? O / L : 0.f;
  const size_t o = ((size_t)r * n_heads + head) * D + d;
  if (out) out[o] = v;
  if (ob) ob[o] = f2bf(v);
  if (oq) {
    const float amax = warp_max(fabsf(v));
    const float dq = amax / 127.f;
    int qi = dq > 0.f ? __float2int_rn(v / dq) : 0;
    qi = max(-127, min(127, qi));
    oq[o] = (int8_t)qi;
    const int s = warp_sum_i(qi);
    if ((d & 31) == 0) ods[o / 32] = make_float2(dq, dq * (float)s);
  }
}

// Single-split path: quantise the final fp32 output in place of the merge.
template <int D>
__global__ void __launch_bounds__(D)
attn_quant_kernel(const float* __restrict__ out, int n_heads, int8_t* __restrict__ oq,
                  float2* __restrict__ ods) {
  pdl_trigger();   // a dependent GEMV may start streaming its weights now
  const int head = blockIdx.x, r = blockIdx.y, d = threadIdx.x;
  const size_t o = ((size_t)r * n_heads + head) * D + d;
  const float v = out[o];
  const float amax = warp_max(fabsf(v));
  const float dq = amax / 127.f;
  int qi = dq > 0.f ? __float2int_rn(v / dq) : 0;
  qi = max(-127, min(127, qi));
  oq[o] = (int8_t)qi;
  const int s = warp_sum_i(qi);
  if ((d & 31) == 0) ods[o / 32] = make_float2(dq, dq * (float)s);
}

template <int D, int G>
void launch_dg(const AttnArgs& a, cudaStream_t st) {
  dim3 grid(a.n_kv, a.n_rows, a.n_splits);
  static const bool simt = getenv("AIR_ATTN_SIMT") != nullptr;
  static const bool per_row = getenv("AIR_PREFILL_ATTN_PER_ROW") != nullptr;
  // prefill rows (a block-table row per query row) of 16 or more: the query-tiled kernel
  if (D == 128 && !simt && !per_row && a.rows.row_seq != nullptr && a.n_rows >= 16 &&
      launch_prefill_attention(a, st))
    return;
  if (!(D == 128 && !simt && launch_paged_attention_mma(a, st)))
  {
    auto kern = a.kv_fp8 ? paged_attn_kernel<D, G, true> : paged_attn_kernel<D, G, false>;
    kern<<<grid, kWarps * 32, 0, st>>>(
        a.q, (const uint8_t*)a.kv, a.block_tables, a.max_blocks, a.rows, a.n_heads, a.n_kv,
        a.block_size, a.num_blocks, a.n_splits, a.split_tokens, a.scale, a.part_o, a.part_ml,
        a.out, a.err);
  }
  if (a.n_splits > 1) {
    attn_merge_kernel<D><<<dim3(a.n_heads, a.n_rows), D, 0, st>>>(
        a.part_o, a.part_ml, a.n_heads, a.n_splits, a.out, a.out_q, a.out_ds, (__nv_bfloat16*)a.out_bf16);
  } else if (a.out_q) {
    attn_quant_kernel<D><<<dim3(a.n_heads, a.n_rows), D, 0, st>>>(a.out, a.n_heads, a.out_q, a.out_ds);
  }
}

template <int D>
bool launch_d(const AttnArgs& a, cudaStream_t st) {
  switch (a.n_heads / a.n_kv) {
    case 1: launch_dg<D, 1>(a, st); return true;
    case 2: launch_dg<D, 2>(a, st); return true;
    case 4: launch_dg<D, 4>(a, st); return true;
    case 8: launch_dg<D, 8>(a, st); return true;
    default: return false;
  }
}

}  // namespace

bool launch_paged_attention(const AttnArgs& a, cudaStream_t st) {
  if (a.head_dim == 128) return launch_d<128>(a, st);
  if (a.head_dim == 64) return launch_d<64>(a, st);
  return false;
}

}  // namespace air
