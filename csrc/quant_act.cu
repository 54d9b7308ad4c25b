// Activation preparation kernels: fused RMSNorm + int8 block quantisation.
//
// The decode GEMVs consume activations as int8 with one (scale, scale*sum) pair per
// 32 elements ("Q8A"), the same role Q8_1/Q8_K activations play in GGUF vec-dot
// kernels; candle's CPU QMatMul (the reference's oracle path, src/model.rs:534-536)
// also quantises activations before its integer dot products.
#include "common.cuh"
#include "kernels.h"

namespace air {

// Grid (ceil(K/1024), B), 1024 threads: each warp owns one 32-element group, so a row is
// spread over many CTAs (a single CTA per row is latency-bound at batch 1). Every CTA of a
// row recomputes that row's statistics (the row is at most a few tens of KB, L2-hot).
// x: fp32 [B, K] residual stream (or bf16 when x_bf16 != null).
// If w != nullptr: y = norm(x) * (w + w_offset) (+ bias), where norm is RMSNorm
// (x * rsqrt(mean(x^2) + eps)) or, with layer = 1, LayerNorm ((x - mean) * rsqrt(var + eps),
// the reference's src/ops.rs:49-70); else y = x.
// Writes q [B, K] int8, ds [B, K/32] float2(d, d*sum(q)); optionally y as bf16.
__device__ __forceinline__ float load_x(const float* xr, const __nv_bfloat16* xb, int i) {
  return xr ? xr[i] : bf2f(xb[i]);
}

__global__ void __launch_bounds__(1024)
rmsnorm_quant_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ x_bf16,
                     const float* __restrict__ w, float w_offset, const float* __restrict__ bias, int layer,
                     int K, float eps, int8_t* __restrict__ q, float2* __restrict__ ds,
                     __nv_bfloat16* __restrict__ y_out) {
  pdl_trigger();   // a dependent GEMV may start streaming its weights now
  __shared__ float red[32];
  const int b = blockIdx.y;
  const float* xr = x ? x + (size_t)b * K : nullptr;
  const __nv_bfloat16* xb = x_bf16 ? x_bf16 + (size_t)b * K : nullptr;
  float scale = 1.f, mean = 0.f;
  if (w) {
    if (layer) {
      float s = 0.f;
      for (int i = threadIdx.x; i < K; i += blockDim.x) s += load_x(xr, xb, i);
      mean = block_sum(s, red) / (float)K;
    }
    float ss = 0.f;
    if (xr && !layer) {
      const float4* x4 = reinterpret_cast<const float4*>(xr);
      for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = x4[i];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
    } else if (!layer) {
      const uint4* x8 = reinterpret_cast<const uint4*>(xb);
      for (int i = threadIdx.x; i < K / 8; i += blockDim.x) {
        float f[8];
        bf16x8_to_f32(x8[i], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
      }
    } else {
      for (int i = threadIdx.x; i < K; i += blockDim.x) {
        const float c = load_x(xr, xb, i) - mean;
        ss += c * c;
      }
    }
    ss = block_sum(ss, red);
    scale = rsqrtf(ss / (float)K + eps);
  }
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (g >= K / 32) return;
  const int i = g * 32 + lane;
  float v = (load_x(xr, xb, i) - mean) * scale;
  if (w) v *= (w[i] + w_offset);
  if (bias) v += bias[i];
  if (y_out) y_out[(size_t)b * K + i] = f2bf(v);
  if (q) {
    const float amax = warp_max(fabsf(v));
    const float d = amax / 127.f;
    int qi = d > 0.f ? __float2int_rn(v / d) : 0;
    qi = max(-127, min(127, qi));
    q[(size_t)b * K + i] = (int8_t)qi;
    const int s = warp_sum_i(qi);
    if (lane == 0) ds[(size_t)b * (K / 32) + g] = make_float2(d, d * (float)s);
  }
}

// Many-row variant (prefill chunks, batched decode): one 256-thread CTA per row, the row held in
// registers (KPT float4 per thread, element 4t + 1024k), so the statistics are computed once per
// row instead of once per 1024-element slice, and the CTAs are small enough for one wave.
// Q8A groups are 8 consecutive threads' float4.
template <int KPT>
__global__ void __launch_bounds__(256)
rmsnorm_quant_rows_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ x_bf16,
                          const float* __restrict__ w, float w_offset, const float* __restrict__ bias, int layer,
                          int K, float eps, int8_t* __restrict__ q, float2* __restrict__ ds,
                          __nv_bfloat16* __restrict__ y_out) {
  pdl_trigger();
  __shared__ float red[32];
  const int b = blockIdx.x, t = threadIdx.x;
  float v[KPT][4];
#pragma unroll
  for (int k = 0; k < KPT; ++k) {
    const int i = 4 * t + 1024 * k;
    if (i < K) {
      if (x) {
        const float4 f = *reinterpret_cast<const float4*>(x + (size_t)b * K + i);
        v[k][0] = f.x; v[k][1] = f.y; v[k][2] = f.z; v[k][3] = f.w;
      } else {
        const uint2 u = *reinterpret_cast<const uint2*>(x_bf16 + (size_t)b * K + i);
        const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        v[k][0] = lo.x; v[k][1] = lo.y; v[k][2] = hi.x; v[k][3] = hi.y;
      }
    } else {
      v[k][0] = v[k][1] = v[k][2] = v[k][3] = 0.f;
    }
  }
  float scale = 1.f, mean = 0.f;
  if (w) {
    if (layer) {
      float sm = 0.f;
#pragma unroll
      for (int k = 0; k < KPT; ++k) sm += v[k][0] + v[k][1] + v[k][2] + v[k][3];
      mean = block_sum(sm, red) / (float)K;
    }
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < KPT; ++k) {
      if (4 * t + 1024 * k >= K) continue;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float c = v[k][e] - mean;
        ss += c * c;
      }
    }
    ss = block_sum(ss, red);
    scale = rsqrtf(ss / (float)K + eps);
  }
#pragma unroll
  for (int k = 0; k < KPT; ++k) {
    const int i = 4 * t + 1024 * k;
    const bool in = i < K;            // uniform over each 8-thread Q8A group (K % 32 == 0)
    float y[4];
    if (in) {
      const float4 wv = w ? *reinterpret_cast<const float4*>(w + i) : make_float4(1.f, 1.f, 1.f, 1.f);
      const float4 bv = bias ? *reinterpret_cast<const float4*>(bias + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float wo = w ? w_offset : 0.f;
      y[0] = (v[k][0] - mean) * scale * (wv.x + wo) + bv.x;
      y[1] = (v[k][1] - mean) * scale * (wv.y + wo) + bv.y;
      y[2] = (v[k][2] - mean) * scale * (wv.z + wo) + bv.z;
      y[3] = (v[k][3] - mean) * scale * (wv.w + wo) + bv.w;
      if (y_out) {
        __nv_bfloat162 p0 = __floats2bfloat162_rn(y[0], y[1]), p1 = __floats2bfloat162_rn(y[2], y[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&p0);
        u.y = *reinterpret_cast<uint32_t*>(&p1);
        *reinterpret_cast<uint2*>(y_out + (size_t)b * K + i) = u;
      }
    } else {
      y[0] = y[1] = y[2] = y[3] = 0.f;
    }
    if (q) {
      float amax = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      const float d = amax / 127.f;
      int qs = 0;
      uint32_t packed = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int qi = d > 0.f ? __float2int_rn(y[e] / d) : 0;
        qi = max(-127, min(127, qi));
        qs += qi;
        packed |= (uint32_t)(qi & 0xFF) << (8 * e);
      }
      qs += __shfl_xor_sync(0xffffffffu, qs, 1);
      qs += __shfl_xor_sync(0xffffffffu, qs, 2);
      qs += __shfl_xor_sync(0xffffffffu, qs, 4);
      if (in) {
        *reinterpret_cast<uint32_t*>(q + (size_t)b * K + i) = packed;
        if ((t & 7) == 0) ds[(size_t)b * (K / 32) + i / 32] = make_float2(d, d * (float)qs);
      }
    }
  }
}

void launch_rmsnorm_quant(const float* x, const void* x_bf16, const float* w, float w_offset,
                          const float* bias, int layer, int B, int K, float eps, int8_t* q, float2* ds,
                          void* y_bf16, cudaStream_t st) {
  // 16 rows or more: one CTA per row (aligned rows of K a multiple of 32, K <= 8192)
  const bool aligned = reinterpret_cast<uintptr_t>(x ? (const void*)x : x_bf16) % 16 == 0 &&
                       (!w || reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
                       (!bias || reinterpret_cast<uintptr_t>(bias) % 16 == 0) &&
                       (!y_bf16 || reinterpret_cast<uintptr_t>(y_bf16) % 8 == 0);
  if (B >= 16 && K % 32 == 0 && K <= 8192 && aligned) {
    const int kpt = (K + 1023) / 1024;
    const __nv_bfloat16* xb = (const __nv_bfloat16*)x_bf16;
    __nv_bfloat16* yb = (__nv_bfloat16*)y_bf16;
#define AIR_RQ_ROWS(N) rmsnorm_quant_rows_kernel<N><<<B, 256, 0, st>>>(x, xb, w, w_offset, bias, layer, K, eps, q, ds, yb)
    if (kpt <= 2) AIR_RQ_ROWS(2);
    else if (kpt <= 4) AIR_RQ_ROWS(4);
    else AIR_RQ_ROWS(8);
#undef AIR_RQ_ROWS
    return;
  }
  const dim3 grid((K / 32 + 31) / 32, B);
  rmsnorm_quant_kernel<<<grid, 1024, 0, st>>>(x, (const __nv_bfloat16*)x_bf16, w, w_offset, bias, layer, K, eps,
                                              q, ds, (__nv_bfloat16*)y_bf16);
}

}  // namespace air
