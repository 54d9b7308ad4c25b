// Decode GEMV (batch <= 8) over GGUF-quantised weights with fused epilogues.
//
// One warp owns one task (one or two weight rows) and streams those rows from HBM
// exactly once, reusing them for every batch row. Activations arrive pre-quantised to
// int8 per 32 elements, so the Q4_K / Q8_0 inner products are integer dp4a sums, scaled
// once per sub-block. Replaces the reference's candle QMatMul path
// (src/model.rs:534-536, 591-594, src/ops.rs:594-611) plus its separate RoPE
// (src/ops.rs:203-318), KV append (src/model.rs:568-570) and residual adds.
#include "common.cuh"
#include "kernels.h"

namespace air {

namespace {

constexpr int kWarpsPerCta = 4;

template <int K>
AIR_DEVICE int sc_byte(const uint4& hd) {
  // bytes 4..15 of the Q4_K header hold the 12 packed scale bytes
  static_assert(K >= 0 && K < 12, "scale byte");
  const uint32_t w = K < 4 ? hd.y : (K < 8 ? hd.z : hd.w);
  return (w >> (8 * (K & 3))) & 0xFF;
}

// (scale, min) of sub-blocks 4h .. 4h+3 for h in {0,1}.
AIR_DEVICE void q4k_scales_half(const uint4& hd, int h, int (&sc)[4], int (&mn)[4]) {
  if (h == 0) {
    sc[0] = sc_byte<0>(hd) & 63; mn[0] = sc_byte<4>(hd) & 63;
    sc[1] = sc_byte<1>(hd) & 63; mn[1] = sc_byte<5>(hd) & 63;
    sc[2] = sc_byte<2>(hd) & 63; mn[2] = sc_byte<6>(hd) & 63;
    sc[3] = sc_byte<3>(hd) & 63; mn[3] = sc_byte<7>(hd) & 63;
  } else {
    sc[0] = (sc_byte<8>(hd) & 0xF) | ((sc_byte<0>(hd) >> 6) << 4);
    mn[0] = (sc_byte<8>(hd) >> 4) | ((sc_byte<4>(hd) >> 6) << 4);
    sc[1] = (sc_byte<9>(hd) & 0xF) | ((sc_byte<1>(hd) >> 6) << 4);
    mn[1] = (sc_byte<9>(hd) >> 4) | ((sc_byte<5>(hd) >> 6) << 4);
    sc[2] = (sc_byte<10>(hd) & 0xF) | ((sc_byte<2>(hd) >> 6) << 4);
    mn[2] = (sc_byte<10>(hd) >> 4) | ((sc_byte<6>(hd) >> 6) << 4);
    sc[3] = (sc_byte<11>(hd) & 0xF) | ((sc_byte<3>(hd) >> 6) << 4);
    mn[3] = (sc_byte<11>(hd) >> 4) | ((sc_byte<7>(hd) >> 6) << 4);
  }
}

AIR_DEVICE float h2f_bits(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

// Per-lane partial dot products of one Q4_K row against MAXB activation rows.
template <int MAXB>
AIR_DEVICE void dot_q4k(const uint8_t* __restrict__ row, int K, int nB,
                        const int8_t* __restrict__ xq, const float2* __restrict__ xds,
                        float (&acc)[MAXB]) {
  const int lane = threadIdx.x & 31;
  const int nhb = K / 128;  // half-blocks of 128 elements
  for (int hb = lane; hb < nhb; hb += 32) {
    const int blk = hb >> 1, h = hb & 1;
    const uint8_t* bp = row + (size_t)blk * 144;
    const uint4 hd = ld_stream(bp);
    uint4 qv[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) qv[t] = ld_stream(bp + 16 + 64 * h + 16 * t);
    const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
    int sc[4], mn[4];
    q4k_scales_half(hd, h, sc, mn);
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const uint32_t w[8] = {qv[2 * jj].x, qv[2 * jj].y, qv[2 * jj].z, qv[2 * jj].w,
                             qv[2 * jj + 1].x, qv[2 * jj + 1].y, qv[2 * jj + 1].z,
                             qv[2 * jj + 1].w};
      const int xoff = blk * 256 + 128 * h + 64 * jj;   // element offset of sub-block lo
      const int g = xoff >> 5;                           // 32-group index of sub-block lo
      const float dl = d * (float)sc[2 * jj], ml = dmin * (float)mn[2 * jj];
      const float dh = d * (float)sc[2 * jj + 1], mh = dmin * (float)mn[2 * jj + 1];
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        if (b < nB) {
          const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)b * K + xoff);
          const int4 a0 = __ldg(xp), a1 = __ldg(xp + 1), c0 = __ldg(xp + 2), c1 = __ldg(xp + 3);
          const int xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          const int xc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          int sl = 0, sh = 0;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            sl = dp4a((int)(w[k] & 0x0F0F0F0Fu), xa[k], sl);
            sh = dp4a((int)((w[k] >> 4) & 0x0F0F0F0Fu), xc[k], sh);
          }
          const float2 gl = __ldg(xds + (size_t)b * (K / 32) + g);
          const float2 gh = __ldg(xds + (size_t)b * (K / 32) + g + 1);
          acc[b] += dl * gl.x * (float)sl - ml * gl.y + dh * gh.x * (float)sh - mh * gh.y;
        }
      }
    }
  }
}

// Repacked Q8_0: int8 qs [N, K] and f16 scales [N, K/32].
template <int MAXB>
AIR_DEVICE void dot_q8_0(const int8_t* __restrict__ qrow, const __half* __restrict__ srow, int K,
                         int nB, const int8_t* __restrict__ xq, const float2* __restrict__ xds,
                         float (&acc)[MAXB]) {
  const int lane = threadIdx.x & 31;
  for (int g = lane; g < K / 32; g += 32) {
    const uint4 w0 = ld_stream(qrow + (size_t)g * 32), w1 = ld_stream(qrow + (size_t)g * 32 + 16);
    const float dw = __half2float(srow[g]);
    const int w[8] = {(int)w0.x, (int)w0.y, (int)w0.z, (int)w0.w,
                      (int)w1.x, (int)w1.y, (int)w1.z, (int)w1.w};
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < nB) {
        const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)b * K + g * 32);
        const int4 a0 = __ldg(xp), a1 = __ldg(xp + 1);
        const int xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        int s = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) s = dp4a(w[k], xa[k], s);
        acc[b] += dw * __ldg(xds + (size_t)b * (K / 32) + g).x * (float)s;
      }
    }
  }
}

template <int MAXB>
AIR_DEVICE void dot_bf16(const __nv_bfloat16* __restrict__ wrow, int K, int nB,
                         const int8_t* __restrict__ xq, const float2* __restrict__ xds,
                         float (&acc)[MAXB]) {
  const int lane = threadIdx.x & 31;
  for (int g = lane; g < K / 32; g += 32) {
    float wf[32];
#pragma unroll
    for (int t = 0; t < 4; ++t) bf16x8_to_f32(ld_stream(wrow + (size_t)g * 32 + 8 * t), wf + 8 * t);
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < nB) {
        const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)b * K + g * 32);
        const int4 a0 = __ldg(xp), a1 = __ldg(xp + 1);
        const int xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
#pragma unroll
          for (int e = 0; e < 4; ++e) s += wf[4 * k + e] * (float)(int8_t)((xa[k] >> (8 * e)) & 0xFF);
        }
        acc[b] += __ldg(xds + (size_t)b * (K / 32) + g).x * s;
      }
    }
  }
}

template <int MAXB, int FMT>
AIR_DEVICE void dot_row(const GemvWeight& w, int64_t r, int K, int nB, const int8_t* xq,
                        const float2* xds, float (&acc)[MAXB]) {
#pragma unroll
  for (int b = 0; b < MAXB; ++b) acc[b] = 0.f;
  if (FMT == kFmtQ4K) {
    dot_q4k<MAXB>(static_cast<const uint8_t*>(w.data) + r * w.row_bytes, K, nB, xq, xds, acc);
  } else if (FMT == kFmtQ8_0) {
    dot_q8_0<MAXB>(static_cast<const int8_t*>(w.data) + r * (int64_t)K,
                   static_cast<const __half*>(w.scales) + r * (int64_t)(K / 32), K, nB, xq, xds, acc);
  } else {
    dot_bf16<MAXB>(static_cast<const __nv_bfloat16*>(w.data) + r * (int64_t)K, K, nB, xq, xds, acc);
  }
#pragma unroll
  for (int b = 0; b < MAXB; ++b) acc[b] = warp_sum(acc[b]);
}

template <int MAXB, int FMT, int MODE>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
gemv_kernel(GemvWeight w, int N, int K, int nB, const int8_t* __restrict__ xq,
            const float2* __restrict__ xds, GemvEpiParams ep, int n_tasks) {
  const int task = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (task >= n_tasks) return;
  const int lane = threadIdx.x & 31;
  if (MODE == kEpiStore || MODE == kEpiResidual) {
    float acc[MAXB];
    dot_row<MAXB, FMT>(w, task, K, nB, xq, xds, acc);
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < nB && lane == b) {
        const size_t o = (size_t)b * ep.ld_out + task;
        if (MODE == kEpiResidual) {
          ep.resid[o] += acc[b];
        } else {
          if (ep.out_f32) ep.out_f32[o] = acc[b];
          if (ep.out_bf16) static_cast<__nv_bfloat16*>(ep.out_bf16)[o] = f2bf(acc[b]);
        }
      }
    }
  } else if (MODE == kEpiSwiGLU) {
    float g[MAXB], u[MAXB];
    dot_row<MAXB, FMT>(w, task, K, nB, xq, xds, g);
    dot_row<MAXB, FMT>(ep.w2, task, K, nB, xq, xds, u);
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < nB && lane == b) {
        const float s = g[b] / (1.f + __expf(-g[b]));
        const size_t o = (size_t)b * ep.ld_out + task;
        if (ep.out_f32) ep.out_f32[o] = s * u[b];
        if (ep.out_bf16) static_cast<__nv_bfloat16*>(ep.out_bf16)[o] = f2bf(s * u[b]);
      }
    }
  } else {  // kEpiQKVRope: task -> (head, i) with rows head*d + i and head*d + i + d/2
    const int hd = ep.head_dim, half = hd / 2;
    const int head = task / half, i = task % half;
    const int64_t r0 = (int64_t)head * hd + i, r1 = r0 + half;
    float a0[MAXB], a1[MAXB];
    dot_row<MAXB, FMT>(w, r0, K, nB, xq, xds, a0);
    dot_row<MAXB, FMT>(w, r1, K, nB, xq, xds, a1);
    const int rh = ep.rot_dim / 2;
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < nB && lane == b) {
        float x0 = a0[b], x1 = a1[b];
        const bool is_v = head >= ep.n_heads + ep.n_kv;
        if (!is_v && i < rh) {
          // NeoX half-split pairs (i, i + rot/2); full rotary when rot_dim == head_dim
          const float2 cs = ep.rope_cs[(size_t)ep.positions[b] * rh + i];
          const float y0 = x0 * cs.x - x1 * cs.y, y1 = x0 * cs.y + x1 * cs.x;
          x0 = y0;
          x1 = y1;
        }
        if (head < ep.n_heads) {
          float* q = ep.q_out + ((size_t)b * ep.n_heads + head) * hd;
          q[i] = x0;
          q[i + half] = x1;
        } else {
          const int64_t slot = ep.slots[b];
          if (slot >= 0) {
            const int64_t blk = slot / ep.block_size, off = slot % ep.block_size;
            if (blk >= ep.num_blocks) {
              set_error(ep.err, kErrBounds);
            } else {
              const int kvh = is_v ? head - ep.n_heads - ep.n_kv : head - ep.n_heads;
              __nv_bfloat16* base = static_cast<__nv_bfloat16*>(ep.kv_cache) +
                  ((((size_t)blk * 2 + (is_v ? 1 : 0)) * ep.n_kv + kvh) * ep.block_size + off) * hd;
              base[i] = f2bf(x0);
              base[i + half] = f2bf(x1);
            }
          }
        }
      }
    }
  }
}

template <int MAXB, int FMT>
void launch_fmt(const GemvWeight& w, int N, int K, int B, const int8_t* xq, const float2* xds,
                const GemvEpiParams& ep, cudaStream_t st) {
  int tasks = N;
  if (ep.mode == kEpiQKVRope) tasks = N / 2;
  const int grid = (tasks + kWarpsPerCta - 1) / kWarpsPerCta;
  switch (ep.mode) {
    case kEpiStore:
      gemv_kernel<MAXB, FMT, kEpiStore><<<grid, kWarpsPerCta * 32, 0, st>>>(w, N, K, B, xq, xds, ep, tasks);
      break;
    case kEpiResidual:
      gemv_kernel<MAXB, FMT, kEpiResidual><<<grid, kWarpsPerCta * 32, 0, st>>>(w, N, K, B, xq, xds, ep, tasks);
      break;
    case kEpiSwiGLU:
      gemv_kernel<MAXB, FMT, kEpiSwiGLU><<<grid, kWarpsPerCta * 32, 0, st>>>(w, N, K, B, xq, xds, ep, tasks);
      break;
    default:
      gemv_kernel<MAXB, FMT, kEpiQKVRope><<<grid, kWarpsPerCta * 32, 0, st>>>(w, N, K, B, xq, xds, ep, tasks);
      break;
  }
}

template <int MAXB>
void launch_b(const GemvWeight& w, int N, int K, int B, const int8_t* xq, const float2* xds,
              const GemvEpiParams& ep, cudaStream_t st) {
  switch (w.fmt) {
    case kFmtQ4K: launch_fmt<MAXB, kFmtQ4K>(w, N, K, B, xq, xds, ep, st); break;
    case kFmtQ8_0: launch_fmt<MAXB, kFmtQ8_0>(w, N, K, B, xq, xds, ep, st); break;
    default: launch_fmt<MAXB, kFmtBF16>(w, N, K, B, xq, xds, ep, st); break;
  }
}

}  // namespace

void launch_gemv(const GemvWeight& w, int N, int K, int B, const int8_t* xq, const float2* xds,
                 const GemvEpiParams& ep, cudaStream_t st) {
  if (B <= 1) launch_b<1>(w, N, K, B, xq, xds, ep, st);
  else if (B <= 2) launch_b<2>(w, N, K, B, xq, xds, ep, st);
  else if (B <= 4) launch_b<4>(w, N, K, B, xq, xds, ep, st);
  else launch_b<8>(w, N, K, B, xq, xds, ep, st);
}

}  // namespace air
