// FP8 (E4M3) paged KV rows.
//
// An fp8 KV pool keeps the bf16 pool's block structure [num_blocks, 2 (K,V), n_kv,
// block_size, row] but a row of one (token, KV head) is 16-byte aligned bytes:
//   [0, D)        D E4M3 codes, code = round(x / s) with s = max|x| / 448 (satfinite)
//   [D, D + 4)    s as f32
//   [D + 4, D+16) zero padding (keeps every row a whole number of 16-byte chunks)
// so the attention kernels fetch a row as D/16 + 1 cp.async chunks. The per-row scale is
// never multiplied into the codes on the read side: K's scale multiplies the score of its
// key (S = q . (s_k c_k) = s_k (q . c_k)) and V's scale multiplies that key's softmax
// weight before P V, so the MMAs run on the exactly converted codes (E4M3 -> f16 is exact).
// Reference: the optional Q8_0 quantisation of the host KV cache, src/kv_cache.rs:54-92
// (32-element blocks with an f16 scale); one scale per 128-wide head row here, E4M3 codes
// (hardware conversion on Blackwell) instead of int8.
#pragma once
#include "common.cuh"
#include <cuda_fp8.h>

namespace air {

__host__ __device__ constexpr int kv_f8_row_bytes(int head_dim) { return head_dim + 16; }
constexpr float kE4M3Max = 448.f;

// two E4M3 codes (low byte first) -> f16x2 bits
AIR_DEVICE uint32_t e4m3x2_to_h2(uint32_t two) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two & 0xFFFFu), __NV_E4M3);
  return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

// 16 codes -> 16 f16 (two 16-byte chunks, element order kept)
AIR_DEVICE void e4m3x16_to_h16(const uint4 c, uint4& lo, uint4& hi) {
  lo.x = e4m3x2_to_h2(c.x);       lo.y = e4m3x2_to_h2(c.x >> 16);
  lo.z = e4m3x2_to_h2(c.y);       lo.w = e4m3x2_to_h2(c.y >> 16);
  hi.x = e4m3x2_to_h2(c.z);       hi.y = e4m3x2_to_h2(c.z >> 16);
  hi.z = e4m3x2_to_h2(c.w);       hi.w = e4m3x2_to_h2(c.w >> 16);
}

// two codes -> float2
AIR_DEVICE float2 e4m3x2_to_f2(uint32_t two) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two & 0xFFFFu), __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// x / s -> two E4M3 codes (saturating)
AIR_DEVICE uint16_t f2_to_e4m3x2(float a, float b) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

}  // namespace air
