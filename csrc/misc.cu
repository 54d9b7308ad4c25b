// Token-parallel kernels of the prefill / batched path: embedding gather with on-the-fly
// dequant (K1), RoPE + paged KV write for GEMM outputs (K4/K5), SwiGLU activation,
// residual add, and GGUF block -> bf16 dequant (K17).
#include <cuda_fp8.h>
#include "common.cuh"
#include "misc.h"
#include "kv_f8.cuh"

namespace air {

namespace {

AIR_DEVICE float h2f(const uint8_t* p) {
  return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(p)));
}

// Dequantise element range [k0, k0+32) of a GGUF row of format fmt into f.
// Row r of a weight: Q4_K uses the tiled device layout (base + r), other formats row-major.
AIR_DEVICE void dequant32(int fmt, const uint8_t* base, int64_t r, int64_t row_bytes, const void* scales,
                          int K, int k0, float* f) {
  const uint8_t* row = base + r * row_bytes;
  const void* scales_row = scales ? static_cast<const __half*>(scales) + r * (K / 32) : nullptr;
  if (fmt == kFmtQ4K) {
    const int blk = k0 >> 8, sub = (k0 >> 5) & 7;
    const uint8_t* bp = q4k_block(base, r, blk, K / 256);
    const float d = h2f(bp), dmin = h2f(bp + 2);
    int sc, m;
    q4k_scale_min(bp + 4, sub, sc, m);
    const uint8_t* qs = bp + 16 + 32 * (sub >> 1);
    const bool hi = sub & 1;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int q = hi ? (qs[l] >> 4) : (qs[l] & 0xF);
      f[l] = d * sc * q - dmin * m;
    }
  } else if (fmt == kFmtQ8_0) {
    const int8_t* q = reinterpret_cast<const int8_t*>(row) + k0;
    const float d = __half2float(static_cast<const __half*>(scales_row)[k0 >> 5]);
#pragma unroll
    for (int l = 0; l < 32; ++l) f[l] = d * q[l];
  } else if (fmt == kFmtFP8) {
    // E4M3 codes; one f32 multiplier per row and 128-wide K block
    const float d = static_cast<const float*>(scales)[r * (K / 128) + (k0 >> 7)];
#pragma unroll
    for (int l = 0; l < 32; l += 2) {
      const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(
          *reinterpret_cast<const __nv_fp8x2_storage_t*>(row + k0 + l), __NV_E4M3);
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&h));
      f[l] = v.x * d;
      f[l + 1] = v.y * d;
    }
  } else {
    const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(row) + k0;
#pragma unroll
    for (int l = 0; l < 32; ++l) f[l] = bf2f(w[l]);
  }
}

__global__ void embed_kernel(int fmt, const uint8_t* __restrict__ table, const void* scales,
                             int64_t row_bytes, int K, const int* __restrict__ ids, int n,
                             int64_t vocab, float* __restrict__ out_f32,
                             __nv_bfloat16* __restrict__ out_bf16, float mult, int* err) {
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) { set_error(err, kErrBounds); id = 0; }
  for (int g = threadIdx.x; g < K / 32; g += blockDim.x) {
    float f[32];
    dequant32(fmt, table, id, row_bytes, scales, K, g * 32, f);
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const size_t o = (size_t)t * K + g * 32 + l;
      if (out_f32) out_f32[o] = f[l] * mult;
      if (out_bf16) out_bf16[o] = f2bf(f[l] * mult);
    }
  }
}

__global__ void dequant_kernel(int fmt, const uint8_t* __restrict__ w, const void* scales,
                               int64_t row_bytes, int N, int K, __nv_bfloat16* __restrict__ out) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // 32-group index
  const int64_t groups = (int64_t)N * (K / 32);
  if (g >= groups) return;
  const int64_t r = g / (K / 32);
  const int k0 = (int)(g % (K / 32)) * 32;
  float f[32];
  dequant32(fmt, w, r, row_bytes, scales, K, k0, f);
  uint4* o = reinterpret_cast<uint4*>(out + r * K + k0);
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = f32_to_bf16x8(f + 8 * i);
}

// qkv: [T, (nh + 2 nkv) * d] (fp32 or bf16). One thread per (t, head, pair i < d/2).
template <typename TIn>
__global__ void rope_kv_kernel(const TIn* __restrict__ qkv, int T, RopeKvArgs a) {
  const int half = a.head_dim / 2;
  const int heads = a.n_heads + 2 * a.n_kv;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)T * heads * half) return;
  const int i = idx % half;
  const int head = (idx / half) % heads;
  const int t = idx / ((int64_t)half * heads);
  const TIn* row = qkv + (size_t)t * heads * a.head_dim + (size_t)head * a.head_dim;
  float x0, x1;
  if constexpr (sizeof(TIn) == 4) { x0 = row[i]; x1 = row[i + half]; }
  else { x0 = bf2f(row[i]); x1 = bf2f(row[i + half]); }
  if (a.bias) {   // q/k/v projection bias (Qwen2), added before RoPE
    x0 += a.bias[(size_t)head * a.head_dim + i];
    x1 += a.bias[(size_t)head * a.head_dim + i + half];
  }
  const bool is_v = head >= a.n_heads + a.n_kv;
  const int rh = a.rot_dim / 2;
  if (!is_v && i < rh) {
    const float2 cs = a.rope_cs[(size_t)a.positions[t] * rh + i];
    const float y0 = x0 * cs.x - x1 * cs.y, y1 = x0 * cs.y + x1 * cs.x;
    x0 = y0;
    x1 = y1;
  }
  if (head < a.n_heads) {
    float* q = a.q_out + ((size_t)t * a.n_heads + head) * a.head_dim;
    q[i] = x0;
    q[i + half] = x1;
    return;
  }
  const int64_t slot = a.slots[t];
  if (slot < 0) return;
  const int64_t blk = slot / a.block_size, off = slot % a.block_size;
  if (blk >= a.num_blocks) { set_error(a.err, kErrBounds); return; }
  const int kvh = is_v ? head - a.n_heads - a.n_kv : head - a.n_heads;
  __nv_bfloat16* base = static_cast<__nv_bfloat16*>(a.kv_cache) +
      ((((size_t)blk * 2 + (is_v ? 1 : 0)) * a.n_kv + kvh) * a.block_size + off) * a.head_dim;
  base[i] = f2bf(x0);
  base[i + half] = f2bf(x1);
}

// fp8 KV pool variant: one warp per (token, head) row, so the row's absmax (the E4M3 scale)
// is a warp reduction. Q rows are written as in rope_kv_kernel; K and V rows as E4M3 codes
// plus the f32 scale (kv_f8.cuh). head_dim is a multiple of 64 (one pair of rotated halves
// per lane per step).
template <typename TIn>
__global__ void __launch_bounds__(256) rope_kv_f8_kernel(const TIn* __restrict__ qkv, int T, RopeKvArgs a) {
  const int heads = a.n_heads + 2 * a.n_kv;
  const int64_t rowi = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (rowi >= (int64_t)T * heads) return;
  const int head = rowi % heads;
  const int t = rowi / heads;
  const int D = a.head_dim, half = D / 2, rh = a.rot_dim / 2;
  constexpr int kMaxPairs = 8;             // head_dim <= 512
  const int np = half / 32;
  const TIn* row = qkv + (size_t)t * heads * D + (size_t)head * D;
  const bool is_v = head >= a.n_heads + a.n_kv;
  float x0[kMaxPairs], x1[kMaxPairs];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxPairs; ++j) {
    if (j >= np) break;
    const int i = lane + 32 * j;
    float u0, u1;
    if constexpr (sizeof(TIn) == 4) { u0 = row[i]; u1 = row[i + half]; }
    else { u0 = bf2f(row[i]); u1 = bf2f(row[i + half]); }
    if (a.bias) {
      u0 += a.bias[(size_t)head * D + i];
      u1 += a.bias[(size_t)head * D + i + half];
    }
    if (!is_v && i < rh) {
      const float2 cs = a.rope_cs[(size_t)a.positions[t] * rh + i];
      const float y0 = u0 * cs.x - u1 * cs.y, y1 = u0 * cs.y + u1 * cs.x;
      u0 = y0;
      u1 = y1;
    }
    x0[j] = u0;
    x1[j] = u1;
    amax = fmaxf(amax, fmaxf(fabsf(u0), fabsf(u1)));
  }
  if (head < a.n_heads) {
    float* q = a.q_out + ((size_t)t * a.n_heads + head) * D;
#pragma unroll
    for (int j = 0; j < kMaxPairs; ++j) {
      if (j >= np) break;
      q[lane + 32 * j] = x0[j];
      q[lane + 32 * j + half] = x1[j];
    }
    return;
  }
  const int64_t slot = a.slots[t];
  if (slot < 0) return;
  const int64_t blk = slot / a.block_size, off = slot % a.block_size;
  if (blk >= a.num_blocks) {
    if (lane == 0) set_error(a.err, kErrBounds);
    return;
  }
  amax = warp_max(amax);
  const float s = amax / kE4M3Max;
  const float inv = s > 0.f ? 1.f / s : 0.f;
  const int kvh = is_v ? head - a.n_heads - a.n_kv : head - a.n_heads;
  const int rb = kv_f8_row_bytes(D);
  uint8_t* base = static_cast<uint8_t*>(a.kv_cache) +
      ((((size_t)blk * 2 + (is_v ? 1 : 0)) * a.n_kv + kvh) * a.block_size + off) * rb;
#pragma unroll
  for (int j = 0; j < kMaxPairs; ++j) {
    if (j >= np) break;
    const uint16_t c = f2_to_e4m3x2(x0[j] * inv, x1[j] * inv);
    base[lane + 32 * j] = (uint8_t)(c & 0xFF);
    base[lane + 32 * j + half] = (uint8_t)(c >> 8);
  }
  if (lane < 4) reinterpret_cast<float*>(base + D)[lane] = lane == 0 ? s : 0.f;
}

// out[t, j] = act(gu[t, j]) * gu[t, up_off + j]   (gate/up concatenated along columns);
// up_off < 0: out = act(gu[t, j]) (dense GELU MLP, no gate)
template <typename TIn>
__global__ void swiglu_kernel(const TIn* __restrict__ gu, int T, int F, int64_t ld_in, int64_t up_off,
                              int64_t ld_out,
                              __nv_bfloat16* __restrict__ out_bf16, float* __restrict__ out_f32, int act) {
  pdl_trigger();   // the down GEMM that follows may start streaming its weights
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)T * F) return;
  const int64_t t = idx / F, j = idx % F;
  float g, u = 1.f;
  if constexpr (sizeof(TIn) == 4) { g = gu[t * ld_in + j]; if (up_off >= 0) u = gu[t * ld_in + up_off + j]; }
  else { g = bf2f(gu[t * ld_in + j]); if (up_off >= 0) u = bf2f(gu[t * ld_in + up_off + j]); }
  const float v = gate_act(g, act) * u;
  if (out_bf16) out_bf16[t * ld_out + j] = f2bf(v);
  if (out_f32) out_f32[t * ld_out + j] = v;
}

// bf16 in / bf16 out, 8 columns per thread (16-byte loads and stores): F, ld_in, up_off and
// ld_out multiples of 8 with 16-byte aligned rows
__global__ void swiglu_bf16x8_kernel(const __nv_bfloat16* __restrict__ gu, int T, int F, int64_t ld_in,
                                     int64_t up_off, int64_t ld_out, __nv_bfloat16* __restrict__ out, int act) {
  pdl_trigger();
  const int F8 = F / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)T * F8) return;
  const int64_t t = idx / F8, j = (idx % F8) * 8;
  float g[8], u[8];
  bf16x8_to_f32(*reinterpret_cast<const uint4*>(gu + t * ld_in + j), g);
  if (up_off >= 0) {
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(gu + t * ld_in + up_off + j), u);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) u[e] = 1.f;
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) g[e] = gate_act(g[e], act) * u[e];
  *reinterpret_cast<uint4*>(out + t * ld_out + j) = f32_to_bf16x8(g);
}

template <typename TIn>
__global__ void residual_add_kernel(float* __restrict__ resid, const TIn* __restrict__ y, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if constexpr (sizeof(TIn) == 4) resid[i] += y[i];
  else resid[i] += bf2f(y[i]);
}

}  // namespace

void launch_embed(int fmt, const void* table, const void* scales, int64_t row_bytes, int K,
                  const int* ids, int n, int64_t vocab, float* out_f32, void* out_bf16, float mult,
                  int* err, cudaStream_t st) {
  if (n <= 0) return;
  embed_kernel<<<n, 128, 0, st>>>(fmt, (const uint8_t*)table, scales, row_bytes, K, ids, n, vocab,
                                  out_f32, (__nv_bfloat16*)out_bf16, mult, err);
}

void launch_dequant(int fmt, const void* w, const void* scales, int64_t row_bytes, int N, int K,
                    void* out, cudaStream_t st) {
  const int64_t groups = (int64_t)N * (K / 32);
  dequant_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, st>>>(fmt, (const uint8_t*)w, scales,
                                                                  row_bytes, N, K, (__nv_bfloat16*)out);
}

void launch_rope_kv(const void* qkv, bool bf16_in, int T, const RopeKvArgs& a, cudaStream_t st) {
  const int64_t n = (int64_t)T * (a.n_heads + 2 * a.n_kv) * (a.head_dim / 2);
  if (n <= 0) return;
  if (a.kv_fp8) {
    const int64_t rows = (int64_t)T * (a.n_heads + 2 * a.n_kv);
    const unsigned g8 = (unsigned)((rows + 7) / 8);
    if (bf16_in) rope_kv_f8_kernel<__nv_bfloat16><<<g8, 256, 0, st>>>((const __nv_bfloat16*)qkv, T, a);
    else rope_kv_f8_kernel<float><<<g8, 256, 0, st>>>((const float*)qkv, T, a);
    return;
  }
  const unsigned grid = (unsigned)((n + 255) / 256);
  if (bf16_in) rope_kv_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)qkv, T, a);
  else rope_kv_kernel<float><<<grid, 256, 0, st>>>((const float*)qkv, T, a);
}

void launch_swiglu(const void* gu, bool bf16_in, int T, int F, int64_t ld_in, int64_t up_off,
                   int64_t ld_out, void* out_bf16, float* out_f32, int act, cudaStream_t st) {
  const int64_t n = (int64_t)T * F;
  if (n <= 0) return;
  const bool vec = bf16_in && out_bf16 && !out_f32 && F % 8 == 0 && ld_in % 8 == 0 && ld_out % 8 == 0 &&
                   (up_off < 0 || up_off % 8 == 0) && reinterpret_cast<uintptr_t>(gu) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out_bf16) % 16 == 0;
  if (vec) {
    const int64_t n8 = (int64_t)T * (F / 8);
    swiglu_bf16x8_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, st>>>(
        (const __nv_bfloat16*)gu, T, F, ld_in, up_off, ld_out, (__nv_bfloat16*)out_bf16, act);
    return;
  }
  const unsigned grid = (unsigned)((n + 255) / 256);
  if (bf16_in) swiglu_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)gu, T, F, ld_in, up_off, ld_out, (__nv_bfloat16*)out_bf16, out_f32, act);
  else swiglu_kernel<float><<<grid, 256, 0, st>>>((const float*)gu, T, F, ld_in, up_off, ld_out, (__nv_bfloat16*)out_bf16, out_f32, act);
}

void launch_residual_add(float* resid, const void* y, bool bf16_in, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  const unsigned grid = (unsigned)((n + 255) / 256);
  if (bf16_in) residual_add_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(resid, (const __nv_bfloat16*)y, n);
  else residual_add_kernel<float><<<grid, 256, 0, st>>>(resid, (const float*)y, n);
}

}  // namespace air
