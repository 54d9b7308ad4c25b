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

// Every warp task covers two weight rows (two output rows, gate+up of one output, or the
// NeoX pair (i, i+d/2) of one head). Both rows' bytes for a lane's slice are loaded before
// any arithmetic so each lane keeps 10 x 16 B in flight; this, not the integer math, is
// what sets the achieved HBM bandwidth of a decode GEMV.

// Q4_K: a lane owns half-blocks (128 weights = 16 B header + 64 B codes).
template <int MAXB>
AIR_DEVICE void dot2_q4k(const uint8_t* __restrict__ base0, int64_t r0, const uint8_t* __restrict__ base1,
                         int64_t r1, int K, int nB, const int8_t* __restrict__ xq,
                         const float2* __restrict__ xds, float (&acc)[2][MAXB]) {
  const int lane = threadIdx.x & 31;
  const int nhb = K / 128, nsb = K / 256;
  for (int hb = lane; hb < nhb; hb += 32) {
    const int blk = hb >> 1, h = hb & 1;
    const uint8_t* bp[2] = {q4k_block(base0, r0, blk, nsb), q4k_block(base1, r1, blk, nsb)};
    uint4 hd[2], qv[2][4];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      hd[r] = ld_stream(bp[r]);
#pragma unroll
      for (int t = 0; t < 4; ++t) qv[r][t] = ld_stream(bp[r] + 16 + 64 * h + 16 * t);
    }
    // activations of this half-block: 4 sub-blocks x 32 int8 + 4 (d, d*sum) pairs per batch row
    const int x0 = blk * 256 + 128 * h;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float d = h2f_bits(hd[r].x), dmin = h2f_bits(hd[r].x >> 16);
      int sc[4], mn[4];
      q4k_scales_half(hd[r], h, sc, mn);
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const uint32_t w[8] = {qv[r][2 * jj].x, qv[r][2 * jj].y, qv[r][2 * jj].z, qv[r][2 * jj].w,
                               qv[r][2 * jj + 1].x, qv[r][2 * jj + 1].y, qv[r][2 * jj + 1].z,
                               qv[r][2 * jj + 1].w};
        const int xoff = x0 + 64 * jj;
        const int g = xoff >> 5;
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
            const float4 gg = __ldg(reinterpret_cast<const float4*>(xds + (size_t)b * (K / 32) + g));
            acc[r][b] += dl * gg.x * (float)sl - ml * gg.y + dh * gg.z * (float)sh - mh * gg.w;
          }
        }
      }
    }
  }
}

// Repacked Q8_0: int8 qs [N, K] and f16 scales [N, K/32]; a lane owns 32-element groups.
template <int MAXB>
AIR_DEVICE void dot2_q8_0(const int8_t* __restrict__ q0, const int8_t* __restrict__ q1,
                          const __half* __restrict__ s0, const __half* __restrict__ s1, int K, int nB,
                          const int8_t* __restrict__ xq, const float2* __restrict__ xds,
                          float (&acc)[2][MAXB]) {
  const int lane = threadIdx.x & 31;
  for (int g = lane; g < K / 32; g += 32) {
    const uint4 w00 = ld_stream(q0 + (size_t)g * 32), w01 = ld_stream(q0 + (size_t)g * 32 + 16);
    const uint4 w10 = ld_stream(q1 + (size_t)g * 32), w11 = ld_stream(q1 + (size_t)g * 32 + 16);
    const float dw[2] = {__half2float(s0[g]), __half2float(s1[g])};
    const int w[2][8] = {{(int)w00.x, (int)w00.y, (int)w00.z, (int)w00.w, (int)w01.x, (int)w01.y, (int)w01.z, (int)w01.w},
                         {(int)w10.x, (int)w10.y, (int)w10.z, (int)w10.w, (int)w11.x, (int)w11.y, (int)w11.z, (int)w11.w}};
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < nB) {
        const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)b * K + g * 32);
        const int4 a0 = __ldg(xp), a1 = __ldg(xp + 1);
        const int xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float dx = __ldg(xds + (size_t)b * (K / 32) + g).x;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          int s = 0;
#pragma unroll
          for (int k = 0; k < 8; ++k) s = dp4a(w[r][k], xa[k], s);
          acc[r][b] += dw[r] * dx * (float)s;
        }
      }
    }
  }
}

template <int MAXB>
AIR_DEVICE void dot2_bf16(const __nv_bfloat16* __restrict__ w0, const __nv_bfloat16* __restrict__ w1,
                          int K, int nB, const int8_t* __restrict__ xq,
                          const float2* __restrict__ xds, float (&acc)[2][MAXB]) {
  const int lane = threadIdx.x & 31;
  for (int g = lane; g < K / 32; g += 32) {
    uint4 raw[2][4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      raw[0][t] = ld_stream(w0 + (size_t)g * 32 + 8 * t);
      raw[1][t] = ld_stream(w1 + (size_t)g * 32 + 8 * t);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float wf[32];
#pragma unroll
      for (int t = 0; t < 4; ++t) bf16x8_to_f32(raw[r][t], wf + 8 * t);
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
          acc[r][b] += __ldg(xds + (size_t)b * (K / 32) + g).x * s;
        }
      }
    }
  }
}

template <int MAXB, int FMT>
AIR_DEVICE void dot2(const GemvWeight& wa, int64_t ra, const GemvWeight& wb, int64_t rb, int K,
                     int nB, const int8_t* xq, const float2* xds, float (&acc)[2][MAXB]) {
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int b = 0; b < MAXB; ++b) acc[r][b] = 0.f;
  if (FMT == kFmtQ4K) {
    dot2_q4k<MAXB>(static_cast<const uint8_t*>(wa.data), ra, static_cast<const uint8_t*>(wb.data), rb, K,
                   nB, xq, xds, acc);
  } else if (FMT == kFmtQ8_0) {
    dot2_q8_0<MAXB>(static_cast<const int8_t*>(wa.data) + ra * (int64_t)K,
                    static_cast<const int8_t*>(wb.data) + rb * (int64_t)K,
                    static_cast<const __half*>(wa.scales) + ra * (int64_t)(K / 32),
                    static_cast<const __half*>(wb.scales) + rb * (int64_t)(K / 32), K, nB, xq, xds, acc);
  } else {
    dot2_bf16<MAXB>(static_cast<const __nv_bfloat16*>(wa.data) + ra * (int64_t)K,
                    static_cast<const __nv_bfloat16*>(wb.data) + rb * (int64_t)K, K, nB, xq, xds, acc);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int b = 0; b < MAXB; ++b) acc[r][b] = warp_sum(acc[r][b]);
}

template <int MAXB, int FMT, int MODE>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
gemv_kernel(GemvWeight w, int N, int K, int nB, const int8_t* __restrict__ xq,
            const float2* __restrict__ xds, GemvEpiParams ep, int n_tasks) {
  const int task = blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (task >= n_tasks) return;
  const int lane = threadIdx.x & 31;
  float acc[2][MAXB];
  if (MODE == kEpiStore || MODE == kEpiResidual) {
    const int64_t r0 = 2 * (int64_t)task;
    const int64_t r1 = r0 + 1 < N ? r0 + 1 : r0;
    dot2<MAXB, FMT>(w, r0, w, r1, K, nB, xq, xds, acc);
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        if (b < nB && lane == 2 * b + r && (r == 0 || r0 + 1 < N)) {
          const size_t o = (size_t)b * ep.ld_out + r0 + r;
          if (MODE == kEpiResidual) {
            ep.resid[o] += acc[r][b];
          } else {
            if (ep.out_f32) ep.out_f32[o] = acc[r][b];
            if (ep.out_bf16) static_cast<__nv_bfloat16*>(ep.out_bf16)[o] = f2bf(acc[r][b]);
          }
        }
      }
    }
  } else if (MODE == kEpiSwiGLU) {
    dot2<MAXB, FMT>(w, task, ep.w2, task, K, nB, xq, xds, acc);
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < nB && lane == b) {
        const float g = acc[0][b], u = acc[1][b];
        const float s = gate_act(g, ep.act);
        const size_t o = (size_t)b * ep.ld_out + task;
        if (ep.out_f32) ep.out_f32[o] = s * u;
        if (ep.out_bf16) static_cast<__nv_bfloat16*>(ep.out_bf16)[o] = f2bf(s * u);
      }
    }
  } else {  // kEpiQKVRope: task -> (head, i) with rows head*d + i and head*d + i + d/2
    const int hd = ep.head_dim, half = hd / 2;
    const int head = task / half, i = task % half;
    const int64_t r0 = (int64_t)head * hd + i, r1 = r0 + half;
    dot2<MAXB, FMT>(w, r0, w, r1, K, nB, xq, xds, acc);
    const int rh = ep.rot_dim / 2;
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < nB && lane == b) {
        float x0 = acc[0][b], x1 = acc[1][b];
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
  int tasks = N;                                            // SwiGLU: one output per task
  if (ep.mode == kEpiQKVRope) tasks = N / 2;                // NeoX row pairs
  if (ep.mode == kEpiStore || ep.mode == kEpiResidual) tasks = (N + 1) / 2;  // row pairs
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
