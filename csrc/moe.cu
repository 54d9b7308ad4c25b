// Mixture-of-experts routing (softmax + top-k + renormalise, the reference's
// compute_routing, src/moe.rs:163-199) and the weighted combine of expert outputs.
#include "common.cuh"
#include "moe.h"

namespace air {

namespace {

constexpr int kRouteThreads = 256;

__global__ void __launch_bounds__(kRouteThreads)
moe_route_kernel(const float* __restrict__ xf, const __nv_bfloat16* __restrict__ xb, int64_t ldx, int H,
                 const float* __restrict__ router, int E, int k, bool normalize, float* __restrict__ cw,
                 int* __restrict__ ids, float* __restrict__ wts) {
  __shared__ float logit[256];
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = warp; e < E; e += kRouteThreads / 32) {
    const float* w = router + (int64_t)e * H;
    float s = 0.f;
    for (int h = lane; h < H; h += 32) {
      const float xv = xf ? xf[t * ldx + h] : bf2f(xb[t * ldx + h]);
      s += xv * w[h];
    }
    s = warp_sum(s);
    if (lane == 0) logit[e] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mx = -INFINITY;
    for (int e = 0; e < E; ++e) mx = fmaxf(mx, logit[e]);
    float sum = 0.f;
    for (int e = 0; e < E; ++e) {
      logit[e] = __expf(logit[e] - mx);
      sum += logit[e];
    }
    for (int e = 0; e < E; ++e) logit[e] /= sum;
    int sel[8];
    float sw[8];
    float ssum = 0.f;
    for (int j = 0; j < k; ++j) {   // descending, ties to the lower index (stable)
      int best = -1;
      for (int e = 0; e < E; ++e) {
        bool taken = false;
        for (int q = 0; q < j; ++q) taken |= (sel[q] == e);
        if (!taken && (best < 0 || logit[e] > logit[best])) best = e;
      }
      sel[j] = best;
      sw[j] = logit[best];
      ssum += sw[j];
    }
    if (normalize && ssum > 1e-9f)
      for (int j = 0; j < k; ++j) sw[j] /= ssum;
    for (int e = 0; e < E; ++e) cw[(int64_t)t * E + e] = 0.f;
    for (int j = 0; j < k; ++j) {
      cw[(int64_t)t * E + sel[j]] = sw[j];
      if (ids) ids[t * k + j] = sel[j];
      if (wts) wts[t * k + j] = sw[j];
    }
  }
}

__global__ void moe_combine_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t ldy,
                                   const float* __restrict__ cw, int e, int E, int H) {
  const int t = blockIdx.y;
  const float c = cw[(int64_t)t * E + e];
  if (c == 0.f) return;
  for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < H; h += gridDim.x * blockDim.x)
    x[(int64_t)t * H + h] += c * y[t * ldy + h];
}

}  // namespace

void launch_moe_route(const void* x, bool x_bf16, int64_t ldx, int T, int H, const float* router, int E, int k,
                      bool normalize, float* cw, int* ids, float* wts, cudaStream_t st) {
  if (T <= 0) return;
  moe_route_kernel<<<T, kRouteThreads, 0, st>>>(x_bf16 ? nullptr : (const float*)x,
                                                x_bf16 ? (const __nv_bfloat16*)x : nullptr, ldx, H, router, E, k,
                                                normalize, cw, ids, wts);
}

void launch_moe_combine(float* x, const float* y, int64_t ldy, const float* cw, int e, int E, int T, int H,
                        cudaStream_t st) {
  if (T <= 0) return;
  moe_combine_kernel<<<dim3((H + 1023) / 1024, T), 256, 0, st>>>(x, y, ldy, cw, e, E, H);
}

}  // namespace air
