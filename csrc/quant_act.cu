// Activation preparation kernels: fused RMSNorm + int8 block quantisation.
//
// The decode GEMVs consume activations as int8 with one (scale, scale*sum) pair per
// 32 elements ("Q8A"), the same role Q8_1/Q8_K activations play in GGUF vec-dot
// kernels; candle's CPU QMatMul (the reference's oracle path, src/model.rs:534-536)
// also quantises activations before its integer dot products.
#include "common.cuh"
#include "kernels.h"

namespace air {

// One CTA per row. x: fp32 [B, K] residual stream (or bf16 when x_bf16 != null).
// If w != nullptr: y = x * rsqrt(mean(x^2) + eps) * (w + w_offset), else y = x.
// Writes q [B, K] int8, ds [B, K/32] float2(d, d*sum(q)); optionally y as bf16.
__global__ void __launch_bounds__(256)
rmsnorm_quant_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ x_bf16,
                     const float* __restrict__ w, float w_offset, int K, float eps,
                     int8_t* __restrict__ q, float2* __restrict__ ds,
                     __nv_bfloat16* __restrict__ y_out) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  const float* xr = x ? x + (size_t)b * K : nullptr;
  const __nv_bfloat16* xb = x_bf16 ? x_bf16 + (size_t)b * K : nullptr;
  auto ld = [&](int i) -> float { return xr ? xr[i] : bf2f(xb[i]); };
  float scale = 1.f;
  if (w) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
      float v = ld(i);
      ss += v * v;
    }
    ss = block_sum(ss, red);
    scale = rsqrtf(ss / (float)K + eps);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int g = wid; g < K / 32; g += nw) {
    const int i = g * 32 + lane;
    float v = ld(i) * scale;
    if (w) v *= (w[i] + w_offset);
    if (y_out) y_out[(size_t)b * K + i] = f2bf(v);
    if (q) {
      float amax = warp_max(fabsf(v));
      float d = amax / 127.f;
      int qi = d > 0.f ? __float2int_rn(v / d) : 0;
      qi = max(-127, min(127, qi));
      q[(size_t)b * K + i] = (int8_t)qi;
      int s = warp_sum_i(qi);
      if (lane == 0) ds[(size_t)b * (K / 32) + g] = make_float2(d, d * (float)s);
    }
  }
}

void launch_rmsnorm_quant(const float* x, const void* x_bf16, const float* w, float w_offset,
                          int B, int K, float eps, int8_t* q, float2* ds, void* y_bf16,
                          cudaStream_t st) {
  rmsnorm_quant_kernel<<<B, 256, 0, st>>>(x, (const __nv_bfloat16*)x_bf16, w, w_offset, K, eps,
                                           q, ds, (__nv_bfloat16*)y_bf16);
}

}  // namespace air
