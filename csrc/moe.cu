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

// One CTA: tokens routed to expert e (cw[t, e] > 0) in token order -> idx, wts, *count.
__global__ void __launch_bounds__(1024)
moe_select_kernel(const float* __restrict__ cw, int e, int E, int T, int* __restrict__ idx,
                  float* __restrict__ wts, int* __restrict__ count) {
  __shared__ int warp_tot[32];
  __shared__ int base;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    const float w = t < T ? cw[(int64_t)t * E + e] : 0.f;
    const bool sel = w > 0.f;
    const unsigned m = __ballot_sync(0xffffffffu, sel);
    if (lane == 0) warp_tot[warp] = __popc(m);
    __syncthreads();
    int off = base;
    for (int k = 0; k < warp; ++k) off += warp_tot[k];
    if (sel) {
      const int p = off + __popc(m & ((1u << lane) - 1));
      idx[p] = t;
      wts[p] = w;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int s = 0;
      for (int k = 0; k < (int)(blockDim.x >> 5); ++k) s += warp_tot[k];
      base += s;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = base;
}

// Grid (cap): row i < count copies x[idx[i]] (bf16) into xg[i].
__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int H, const int* __restrict__ idx,
                                  const int* __restrict__ count, __nv_bfloat16* __restrict__ xg) {
  const int i = blockIdx.x;
  if (i >= __ldg(count)) return;
  const uint4* s = reinterpret_cast<const uint4*>(x + (int64_t)idx[i] * ldx);
  uint4* d = reinterpret_cast<uint4*>(xg + (int64_t)i * H);
  for (int k = threadIdx.x; k < H / 8; k += blockDim.x) d[k] = s[k];
}

// Grid (cap): row i < count adds wts[i] * y[i] into out[idx[i]] (one expert per launch, so a
// token appears at most once).
__global__ void moe_scatter_kernel(float* __restrict__ out, const float* __restrict__ y, int64_t ldy, int H,
                                   const int* __restrict__ idx, const float* __restrict__ wts,
                                   const int* __restrict__ count) {
  const int i = blockIdx.x;
  if (i >= __ldg(count)) return;
  const float w = wts[i];
  float* o = out + (int64_t)idx[i] * H;
  const float* yr = y + (int64_t)i * ldy;
  for (int k = threadIdx.x; k < H; k += blockDim.x) o[k] += w * yr[k];
}

// Grouped variants over G local experts: group g covers rows [g * T, g * T + T) of the
// packed buffers. One CTA per group lists its expert's tokens in token order (idx, wts,
// count[g]) and records each token's packed row (pos[g * T + t], -1 when not routed).
__global__ void __launch_bounds__(1024)
moe_select_grouped_kernel(const float* __restrict__ cw, const int* __restrict__ experts, int E, int T,
                          int* __restrict__ idx, float* __restrict__ wts, int* __restrict__ count,
                          int* __restrict__ pos) {
  __shared__ int warp_tot[32];
  __shared__ int base;
  const int g = blockIdx.x, e = experts[g];
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int* gidx = idx + (int64_t)g * T;
  float* gwts = wts + (int64_t)g * T;
  int* gpos = pos + (int64_t)g * T;
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    const float w = t < T ? cw[(int64_t)t * E + e] : 0.f;
    const bool sel = w > 0.f;
    const unsigned m = __ballot_sync(0xffffffffu, sel);
    if (lane == 0) warp_tot[warp] = __popc(m);
    __syncthreads();
    int off = base;
    for (int k = 0; k < warp; ++k) off += warp_tot[k];
    if (t < T) gpos[t] = -1;
    if (sel) {
      const int p = off + __popc(m & ((1u << lane) - 1));
      gidx[p] = t;
      gwts[p] = w;
      gpos[t] = p;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int s = 0;
      for (int k = 0; k < (int)(blockDim.x >> 5); ++k) s += warp_tot[k];
      base += s;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) count[g] = base;
}

// Grid (T, G): packed row i < count[g] of group g = x[idx[g * T + i]].
__global__ void moe_gather_grouped_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int H,
                                          const int* __restrict__ idx, const int* __restrict__ count, int T,
                                          __nv_bfloat16* __restrict__ xg) {
  const int i = blockIdx.x, g = blockIdx.y;
  if (i >= __ldg(count + g)) return;
  const uint4* s = reinterpret_cast<const uint4*>(x + (int64_t)idx[(int64_t)g * T + i] * ldx);
  uint4* d = reinterpret_cast<uint4*>(xg + ((int64_t)g * T + i) * H);
  for (int k = threadIdx.x; k < H / 8; k += blockDim.x) d[k] = s[k];
}

// Grid (ceil(H / 256), T): out[t] += sum over groups g in order of wts * y[packed row of t in
// g] (a fixed order, so the sum does not depend on scheduling).
__global__ void moe_scatter_grouped_kernel(float* __restrict__ out, const float* __restrict__ y, int64_t ldy, int H,
                                           const int* __restrict__ pos, const float* __restrict__ wts, int G,
                                           int T) {
  const int t = blockIdx.y, h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= H) return;
  float acc = 0.f;
  bool any = false;
  for (int g = 0; g < G; ++g) {
    const int p = pos[(int64_t)g * T + t];
    if (p < 0) continue;
    const int64_t row = (int64_t)g * T + p;
    acc += wts[row] * y[row * ldy + h];
    any = true;
  }
  if (any) out[(int64_t)t * H + h] += acc;
}

}  // namespace

void launch_moe_select_grouped(const float* cw, const int* experts, int G, int E, int T, int* idx, float* wts,
                               int* count, int* pos, cudaStream_t st) {
  moe_select_grouped_kernel<<<G, 1024, 0, st>>>(cw, experts, E, T, idx, wts, count, pos);
}

void launch_moe_gather_grouped(const void* x, int64_t ldx, int H, const int* idx, const int* count, int G, int T,
                               void* xg, cudaStream_t st) {
  if (T <= 0) return;
  moe_gather_grouped_kernel<<<dim3(T, G), 128, 0, st>>>((const __nv_bfloat16*)x, ldx, H, idx, count, T,
                                                        (__nv_bfloat16*)xg);
}

void launch_moe_scatter_grouped(float* out, const float* y, int64_t ldy, int H, const int* pos, const float* wts,
                                int G, int T, cudaStream_t st) {
  if (T <= 0) return;
  moe_scatter_grouped_kernel<<<dim3((H + 255) / 256, T), 256, 0, st>>>(out, y, ldy, H, pos, wts, G, T);
}

void launch_moe_select(const float* cw, int e, int E, int T, int* idx, float* wts, int* count, cudaStream_t st) {
  moe_select_kernel<<<1, 1024, 0, st>>>(cw, e, E, T, idx, wts, count);
}

void launch_moe_gather(const void* x, int64_t ldx, int H, const int* idx, const int* count, int cap, void* xg,
                       cudaStream_t st) {
  if (cap <= 0) return;
  moe_gather_kernel<<<cap, 128, 0, st>>>((const __nv_bfloat16*)x, ldx, H, idx, count, (__nv_bfloat16*)xg);
}

void launch_moe_scatter(float* out, const float* y, int64_t ldy, int H, const int* idx, const float* wts,
                        const int* count, int cap, cudaStream_t st) {
  if (cap <= 0) return;
  moe_scatter_kernel<<<cap, 256, 0, st>>>(out, y, ldy, H, idx, wts, count);
}

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
