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
  if (timed_out) return 0.f;          // an earlier wait of this thread already gave up
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

// NVLink SHARP loads: the sum over every rank of the fp32 value(s) at multicast address p.
__device__ __forceinline__ float mm_ld_reduce(const float* p) {
  float v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float4 mm_ld_reduce4(const float* p) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p) : "memory");
  return v;
}
constexpr int kNvlsRowMax = 8192;   // rows up to this width are loaded 16 bytes at a time

// Grid (1, B, n_local): one CTA per (row, rank), so the reduced row can be held in registers
// between the sum-of-squares pass and the quantisation pass. In two-shot mode a CTA first
// reduces its rank's columns of the row and all-gathers them, then waits for the rest of
// the row from the other owners; every CTA of every rank is resident at once (B * n_local
// <= 2 * 148 is checked by the host), so these cross-CTA waits always make progress.
// MODE 0: one-shot, 1: two-shot, 2: NVLS (multimem.ld_reduce over the symmetric buffer).
template <int MODE>
__global__ void __launch_bounds__(kThreads) tp_reduce_norm_kernel(const __grid_constant__ TPReduceArgs a) {
  constexpr bool TWO = MODE == 1;
  pdl_trigger();   // a dependent GEMV may start streaming its weights now
  __shared__ float red[32];
  const TPReduceRank& R = a.r[blockIdx.z];
  const int b = blockIdx.y, t = threadIdx.x, K = a.K;
  const int e = *(volatile const int*)R.epoch;
  const uint32_t tag = (uint32_t)e + 1u;
  const int par = e & 1;
  bool timed_out = false;
  float* xr = R.x + (size_t)b * K;
  float v[kMaxPer];
  float ss = 0.f;
  if (TWO) {
    // ---- reduce-scatter half: this rank's columns [c0, c1) of row b ----
    const int64_t S = a.shard;
    const int c0 = (int)(R.rank * S);
    const int c1 = min(K, (int)(c0 + S));
    const uint2* rs = R.rs + (int64_t)par * a.world * a.slot_elems + (int64_t)b * S;
    const int64_t ag_off = (int64_t)par * a.slot_elems + (int64_t)b * K;
    for (int i = c0 + t; i < c1; i += kThreads) {
      float s = xr[i];
      for (int src = 0; src < a.world; ++src)
        s += wait_tagged(rs + (int64_t)src * a.slot_elems + (i - c0), tag, a.timeout_ns, timed_out);
#pragma unroll
      for (int d = 0; d < kMaxPeers; ++d)
        if (d < a.world) st_tagged(R.ag_peer[d] + ag_off + i, s, tag);
    }
    // ---- all-gather half: the whole row from its owners (local memory) ----
    const uint2* ag = R.ag + ag_off;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int i = j * kThreads + t;
      v[j] = 0.f;
      if (i < K) {
        const float s = wait_tagged(ag + i, tag, a.timeout_ns, timed_out);
        xr[i] = s;
        v[j] = s;
        ss += s * s;
      }
    }
  } else if (MODE == 2) {
    // ---- NVLS: row b's arrival flag to every rank, wait for all, then one switch-reduced
    // load per element (the producers' stores completed with their kernels) ----
    __shared__ int late;
    if (t == 0) late = 0;
    __syncthreads();
    if (t < a.world) {
      __threadfence_system();
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        if (r == t) st_release_sys(R.flags_peer[r] + (int64_t)b * a.world + R.rank, (int)tag);
      const int* f = R.flags + (int64_t)b * a.world + t;
      if ((int)(ld_acquire_sys(f) - (int)tag) < 0) {
        const uint64_t t0 = sm100::global_ns();
        for (uint32_t it = 1;; ++it) {
          if ((int)(ld_acquire_sys(f) - (int)tag) >= 0) break;
          if ((it & 31) == 0 && sm100::global_ns() - t0 > (uint64_t)a.timeout_ns) {
            timed_out = true;
            atomicExch(&late, 1);
            break;
          }
        }
      }
    }
    __syncthreads();
    const float* mrow = R.mc + (int64_t)b * K;
    // 16-byte switch loads into shared memory (4x fewer NVLS requests than scalar ones), then
    // the strided register layout the norm and the Q8A epilogue use
    __shared__ float4 srow[MODE == 2 ? kNvlsRowMax / 4 : 1];
    const bool vec = K <= kNvlsRowMax && !late;
    if (vec) {
      for (int i4 = t; i4 < K / 4; i4 += kThreads) srow[i4] = mm_ld_reduce4(mrow + 4 * i4);
      __syncthreads();
    }
    const float* srf = reinterpret_cast<const float*>(srow);
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int i = j * kThreads + t;
      v[j] = 0.f;
      if (i < K) {
        const float s = xr[i] + (late ? 0.f : (vec ? srf[i] : mm_ld_reduce(mrow + i)));
        xr[i] = s;
        v[j] = s;
        ss += s * s;
      }
    }
  } else {
    // ---- one-shot: x += sum of every rank's whole partial ----
    const uint2* base = R.rs + (int64_t)par * a.world * a.slot_elems + (int64_t)b * K;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int i = j * kThreads + t;
      v[j] = 0.f;
      if (i < K) {
        float s = xr[i];
        for (int src = 0; src < a.world; ++src)
          s += wait_tagged(base + (int64_t)src * a.slot_elems + i, tag, a.timeout_ns, timed_out);
        xr[i] = s;
        v[j] = s;
        ss += s * s;
      }
    }
  }
  if (timed_out) set_error(R.err, kErrTimeout);
  float scale = 1.f, mean = 0.f;
  if (a.w) {
    if (a.layer) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxPer; ++j) s += v[j];      // zero beyond K
      mean = block_sum(s, red) / (float)K;
      ss = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxPer; ++j)
        if (j * kThreads + t < K) ss += (v[j] - mean) * (v[j] - mean);
    }
    ss = block_sum(ss, red);
    scale = rsqrtf(ss / (float)K + a.eps);
  }
  const int lane = t & 31;
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int i = j * kThreads + t;
    if (j * kThreads >= K) break;          // uniform across the CTA
    float y = (v[j] - mean) * scale;
    if (a.w && i < K) y *= (a.w[i] + a.w_offset);
    if (a.bias && i < K) y += a.bias[i];
    if (i < K && R.y_bf16) static_cast<__nv_bfloat16*>(R.y_bf16)[(size_t)b * K + i] = f2bf(y);
    if (R.q) {
      // a warp covers 32 consecutive elements = one Q8A group (K % 32 == 0)
      const float amax = warp_max(i < K ? fabsf(y) : 0.f);
      const float d = amax / 127.f;
      int qi = (d > 0.f && i < K) ? __float2int_rn(y / d) : 0;
      qi = max(-127, min(127, qi));
      if (i < K) R.q[(size_t)b * K + i] = (int8_t)qi;
      const int s = warp_sum_i(qi);
      if (lane == 0 && i < K) R.ds[(size_t)b * (K / 32) + i / 32] = make_float2(d, d * (float)s);
    }
  }
  // ---- the rank's last CTA advances its epoch (every CTA read it before arriving) ----
  __syncthreads();
  if (t == 0) {
    __threadfence();
    if (atomicAdd(R.done, 1) == (int)gridDim.y - 1) {
      *R.done = 0;
      *R.epoch = e + 1;
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
    peer_store(p, e, b, c, __ldcg(src + b * ld + c));
  }
}

}  // namespace

void launch_tp_reduce_norm(const TPReduceArgs& a, cudaStream_t st) {
  const dim3 grid(1, a.B, a.n_local);
  if (a.nvls)
    tp_reduce_norm_kernel<2><<<grid, kThreads, 0, st>>>(a);
  else if (a.shard > 0)
    tp_reduce_norm_kernel<1><<<grid, kThreads, 0, st>>>(a);
  else
    tp_reduce_norm_kernel<0><<<grid, kThreads, 0, st>>>(a);
}

void launch_peer_push(const PeerPush& p, const float* src, int B, int N, int64_t ld, cudaStream_t st) {
  const int64_t n = (int64_t)B * N;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 4 * 148);
  peer_push_kernel<<<blocks, 256, 0, st>>>(p, src, B, N, ld);
}

}  // namespace air
