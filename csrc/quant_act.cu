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

void launch_rmsnorm_quant(const float* x, const void* x_bf16, const float* w, float w_offset,
                          const float* bias, int layer, int B, int K, float eps, int8_t* q, float2* ds,
                          void* y_bf16, cudaStream_t st) {
  const dim3 grid((K / 32 + 31) / 32, B);
  rmsnorm_quant_kernel<<<grid, 1024, 0, st>>>(x, (const __nv_bfloat16*)x_bf16, w, w_offset, bias, layer, K, eps,
                                              q, ds, (__nv_bfloat16*)y_bf16);
}

}  // namespace air
