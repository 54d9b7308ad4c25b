// Shared device helpers for the air_rs sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define AIR_DEVICE __device__ __forceinline__

namespace air {

constexpr int kWarp = 32;

// Device-side error words (read by the host after a step; kernels never trap).
enum ErrorCode : int {
  kOk = 0,
  kErrBounds = 1,        // an index (block table, page id, expert id) was out of range
  kErrTimeout = 2,       // a bounded spin-wait on a peer flag ran out
  kErrBadArg = 3,
};

// Raise a kernel's dynamic shared-memory limit on the current device, once per device.
// cudaFuncSetAttribute applies to the device that is current when it is called, so a
// process that launches the same kernel on several GPUs must set it on each of them.
// `done` is a per-kernel bitmask of the devices already set (devices 0..63).
template <class Kernel>
inline bool set_max_smem_per_device(Kernel kernel, int bytes, unsigned long long& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  const unsigned long long bit = 1ull << dev;
  if (__atomic_load_n(&done, __ATOMIC_ACQUIRE) & bit) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  __atomic_fetch_or(&done, bit, __ATOMIC_ACQ_REL);
  return true;
}

// Gate activation of the gated FFNs: 0 = SiLU (SwiGLU), 1 = GELU, tanh form (GeGLU / dense
// GELU MLP; reference src/ops.rs:103-119: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))).
enum GateAct : int { kActSilu = 0, kActGelu = 1 };
AIR_DEVICE float gate_act(float x, int act) {
  if (act == kActGelu) return 0.5f * x * (1.f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
  return x / (1.f + __expf(-x));
}

// Attention logit soft-capping: cap * tanh(s / cap) when cap > 0.
AIR_DEVICE float soft_cap(float s, float cap) { return cap > 0.f ? cap * tanhf(s / cap) : s; }

AIR_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
AIR_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
AIR_DEVICE int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum for blockDim.x <= 1024; `red` must hold 32 floats.
AIR_DEVICE float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : 0.f;
  if (wid == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}
AIR_DEVICE float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (threadIdx.x < nw) ? red[threadIdx.x] : -INFINITY;
  if (wid == 0) t = warp_max(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

AIR_DEVICE float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
AIR_DEVICE __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }

// Unpack 8 bf16 from a uint4.
AIR_DEVICE void bf16x8_to_f32(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
AIR_DEVICE uint4 f32_to_bf16x8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// Streaming 16-byte global load that does not allocate in L1 (weights are read once).
AIR_DEVICE uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

AIR_DEVICE int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Programmatic dependent launch. A kernel launched with the programmatic-serialisation
// attribute may start while its predecessor in the stream still runs; it must call
// pdl_wait() before touching anything the predecessor writes or reads (a no-op when it was
// launched normally). pdl_trigger() lets such a successor start early.
AIR_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
AIR_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

AIR_DEVICE void set_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Q4_K header: d, dmin (f16) and 12 bytes of packed 6-bit scales/mins.
// Returns sub-block j's (scale, min) as integers.
AIR_DEVICE void q4k_scale_min(const uint8_t* sc12, int j, int& sc, int& m) {
  if (j < 4) {
    sc = sc12[j] & 63;
    m = sc12[j + 4] & 63;
  } else {
    sc = (sc12[j + 4] & 0xF) | ((sc12[j - 4] >> 6) << 4);
    m = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
  }
}

}  // namespace air

namespace air {
// Q4_K device layout ("tiled"): [ceil(N/128)][K/256][128 rows][144 B]. The 144-byte GGUF
// block is unchanged; rows are grouped 128 at a time per super-block column so one
// 128-row x 256-weight tile is 18 KB of contiguous memory (one bulk copy).
AIR_DEVICE const uint8_t* q4k_block(const uint8_t* base, int64_t r, int sb, int nsb) {
  return base + (((((r >> 7) * nsb + sb) << 7) + (r & 127)) * 144);
}
}  // namespace air
