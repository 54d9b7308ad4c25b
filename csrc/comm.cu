// Consumer (reduce + RMSNorm + Q8A quantisation) and standalone producer kernels of the
// fused tensor-parallel all-reduce. Protocol: comm.h.
#include "comm.cuh"
#include "comm.h"
#include "sm100.cuh"

namespace air {

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxPer = 16;   // K <= 16 * 1024

// Wait (bounded) until the element carries this collective's tag; returns its value.
__device__ __forceinline__ float wait_tagged(const uint2* p, uint32_t tag, int64_t timeout_ns, bool& timed_out) {
  uint2 v = ld_tagged(p);
  if (v.y == tag) return __uint_as_float(v.x);
  const uint64_t t0 = sm100::global_ns();
  for (uint32_t it = 1;; ++it) {
    v = ld_tagged(p);
    if (v.y == tag) return __uint_as_float(v.x);
    if ((it & 31) == 0 && sm100::global_ns() - t0 > (uint64_t)timeout_ns) {
      timed_out = true;
      return 0.f;
    }
  }
}

// Grid (1, B): one CTA per row, so the reduced row can be held in registers between the
// sum-of-squares pass and the quantisation pass (no other CTA reads x meanwhile).
__global__ void __launch_bounds__(kThreads)
reduce_rmsnorm_quant_kernel(PeerReduce r, float* __restrict__ x, const float* __restrict__ w, float w_offset,
                            int K, float eps, int8_t* __restrict__ q, float2* __restrict__ ds,
                            __nv_bfloat16* __restrict__ y_out) {
  pdl_trigger();   // a dependent GEMV may start streaming its weights now
  __shared__ float red[32];
  const int b = blockIdx.y, t = threadIdx.x;
  const int e = *(volatile const int*)r.epoch;
  const uint32_t tag = (uint32_t)e + 1u;
  const uint2* base = r.data + (int64_t)(e & 1) * r.world * r.slot_elems + (int64_t)b * K;
  bool timed_out = false;
  // ---- x += sum of partials (each element waits for its tag); sum of squares ----
  float v[kMaxPer];
  float ss = 0.f;
  float* xr = x + (size_t)b * K;
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int i = j * kThreads + t;
    v[j] = 0.f;
    if (i < K) {
      float s = xr[i];
      for (int src = 0; src < r.world; ++src)
        s += wait_tagged(base + (int64_t)src * r.slot_elems + i, tag, r.timeout_ns, timed_out);
      xr[i] = s;
      v[j] = s;
      ss += s * s;
    }
  }
  if (timed_out) set_error(r.err, kErrTimeout);
  float scale = 1.f;
  if (w) {
    ss = block_sum(ss, red);
    scale = rsqrtf(ss / (float)K + eps);
  }
  const int lane = t & 31;
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int i = j * kThreads + t;
    if (j * kThreads >= K) break;          // uniform across the CTA
    float y = v[j] * scale;
    if (w && i < K) y *= (w[i] + w_offset);
    if (i < K && y_out) y_out[(size_t)b * K + i] = f2bf(y);
    if (q) {
      // a warp covers 32 consecutive elements = one Q8A group (K % 32 == 0)
      const float amax = warp_max(i < K ? fabsf(y) : 0.f);
      const float d = amax / 127.f;
      int qi = (d > 0.f && i < K) ? __float2int_rn(y / d) : 0;
      qi = max(-127, min(127, qi));
      if (i < K) q[(size_t)b * K + i] = (int8_t)qi;
      const int s = warp_sum_i(qi);
      if (lane == 0 && i < K) ds[(size_t)b * (K / 32) + i / 32] = make_float2(d, d * (float)s);
    }
  }
  // ---- the last CTA advances the epoch (every CTA read it before arriving) ----
  __syncthreads();
  if (t == 0) {
    __threadfence();
    if (atomicAdd(r.done, 1) == (int)gridDim.y - 1) {
      *r.done = 0;
      *r.epoch = e + 1;
      __threadfence();
    }
  }
}

__global__ void __launch_bounds__(256)
peer_push_kernel(PeerPush p, const float* __restrict__ src, int B, int N, int64_t ld) {
  const int e = *(volatile const int*)p.epoch;
  const int64_t n = (int64_t)B * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / N, c = i % N;
    peer_store(p, e, b * ld + c, __ldcg(src + b * ld + c));
  }
}

}  // namespace

void launch_reduce_rmsnorm_quant(const PeerReduce& r, float* x, const float* w, float w_offset, int B, int K,
                                 float eps, int8_t* q, float2* ds, void* y_bf16, cudaStream_t st) {
  reduce_rmsnorm_quant_kernel<<<dim3(1, B), kThreads, 0, st>>>(r, x, w, w_offset, K, eps, q, ds,
                                                              (__nv_bfloat16*)y_bf16);
}

void launch_peer_push(const PeerPush& p, const float* src, int B, int N, int64_t ld, cudaStream_t st) {
  const int64_t n = (int64_t)B * N;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4 * 148);
  peer_push_kernel<<<blocks, 256, 0, st>>>(p, src, B, N, ld);
}

}  // namespace air
