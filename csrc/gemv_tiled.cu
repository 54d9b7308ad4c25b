// Decode GEMV (batch <= 8) over tiled Q4_K weights, streamed by the bulk-copy engine.
//
// CTA = (128-row weight tile, K split), 128 threads, thread t owns weight row t of the
// tile. The tile's 18 KB super-block slabs ([128 rows][144 B], contiguous in the tiled
// device layout) are brought into a shared-memory ring with cp.async.bulk + mbarrier
// complete_tx, so HBM sees long sequential reads and the SM keeps several slabs in
// flight. Activations are int8 with per-32 (d, d*sum) pairs (Q8A, see quant_act.cu), staged
// once per CTA in shared memory and read as broadcasts. The inner product is the GGUF
// Q4_K math: per 32-weight sub-block an integer dp4a sum times d*sc, minus dmin*m times
// the activation block sum.
//
// Split-K partials go to a caller-provided fp32 workspace; the last CTA of a tile (per-tile
// arrival counter, reset by that CTA) reduces them and runs the fused epilogue:
//   store / residual add / SwiGLU (gate and up tiles streamed together) /
//   QKV + NeoX RoPE + paged KV write (a 128-row tile is one head: pairs (i, i+64)) /
//   tensor-parallel peer push (each element goes to every rank's receive buffer over
//   NVLink as one tagged 8-byte store; comm.h).
#include "common.cuh"
#include "sm100.cuh"
#include "kernels.h"
#include "gemv_tiled.h"
#include "comm.cuh"
#include <stdlib.h>

namespace air {

namespace {

using namespace sm100;

constexpr int kRows = 128;
constexpr int kSlab = kRows * 144;   // 18432 B
constexpr int kMaxStages = 4;

struct Smem {
  uint64_t full[kMaxStages];
  int last;
};

template <int MAXB, bool DUAL>
__global__ void __launch_bounds__(kRows)
gemv_tiled_kernel(const uint8_t* __restrict__ w1, const uint8_t* __restrict__ w2, int N, int K, int nB,
                  const int8_t* __restrict__ xq, const float2* __restrict__ xds, GemvEpiParams ep,
                  GemvTiledScratch sc) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int t = threadIdx.x;
  const int tile = blockIdx.x, split = blockIdx.y, splits = gridDim.y;
  const int nsb = K / 256;
  const int kper = (nsb + splits - 1) / splits;
  const int sb0 = split * kper;
  const int nk = max(0, min(nsb, sb0 + kper) - sb0);
  constexpr int W = DUAL ? 2 : 1;
  const int S = min(kMaxStages, kper);                    // ring depth (host sizes smem the same way)
  uint8_t* slabs = smem;                                   // [S][W][kSlab]
  int8_t* xs = reinterpret_cast<int8_t*>(smem + (size_t)S * W * kSlab);     // [nB][kper*256]
  float2* xd = reinterpret_cast<float2*>(xs + MAXB * kper * 256);          // [nB][kper*8]
  Smem* bar = reinterpret_cast<Smem*>(xd + MAXB * kper * 8);

  if (t == 0) {
    for (int s = 0; s < kMaxStages; ++s) mbar_init(&bar->full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;
  auto issue = [&](int i) {
    const int s = i % S;
    issued = i + 1;
    mbar_expect_tx(&bar->full[s], W * kSlab);
    const size_t off = ((size_t)tile * nsb + sb0 + i) * kSlab;
    const int np = sc.wsplit > 0 ? sc.wsplit : 1;     // split copies: more requests in flight
    const uint32_t piece = kSlab / np;
    for (int p = 0; p < np; ++p) {
      bulk_load(slabs + (size_t)(s * W) * kSlab + p * piece, w1 + off + p * piece, piece, &bar->full[s]);
      if (DUAL) bulk_load(slabs + (size_t)(s * W + 1) * kSlab + p * piece, w2 + off + p * piece, piece, &bar->full[s]);
    }
  };
  if (t == 0)
    for (int i = 0; i < min(S, nk); ++i) issue(i);
  // stage this split's activations (overlaps the first weight copies)
  for (int b = 0; b < nB; ++b) {
    const int4* src = reinterpret_cast<const int4*>(xq + (size_t)b * K + (size_t)sb0 * 256);
    int4* dst = reinterpret_cast<int4*>(xs + (size_t)b * kper * 256);
    for (int i = t; i < nk * 16; i += kRows) dst[i] = src[i];
    const float2* ds = xds + (size_t)b * (K / 32) + (size_t)sb0 * 8;
    for (int i = t; i < nk * 8; i += kRows) xd[b * kper * 8 + i] = ds[i];
  }
  __syncthreads();

  float acc[W][MAXB];
#pragma unroll
  for (int u = 0; u < W; ++u)
#pragma unroll
    for (int b = 0; b < MAXB; ++b) acc[u][b] = 0.f;

  bool ok = true;
  for (int i = 0; i < nk; ++i) {
    const int s = i % S;
    if (!mbar_wait(&bar->full[s], (i / S) & 1, ep.err)) {
      ok = false;
      set_error(ep.err, kErrTimeout);
    }
    if (ok) {
#pragma unroll
      for (int u = 0; u < W; ++u) {
        const uint8_t* rb = slabs + (size_t)(s * W + u) * kSlab + t * 144;
        const uint4 hd = *reinterpret_cast<const uint4*>(rb);
        const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
        const uint8_t* s12 = rb + 4;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          int scl, mnl, sch, mnh;
          q4k_scale_min(s12, 2 * c, scl, mnl);
          q4k_scale_min(s12, 2 * c + 1, sch, mnh);
          const uint4 qa = *reinterpret_cast<const uint4*>(rb + 16 + 32 * c);
          const uint4 qb = *reinterpret_cast<const uint4*>(rb + 32 + 32 * c);
          const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
          const float fl = d * (float)scl, ml = dmin * (float)mnl;
          const float fh = d * (float)sch, mh = dmin * (float)mnh;
#pragma unroll
          for (int b = 0; b < MAXB; ++b) {
            if (b < nB) {
              const int4* xp = reinterpret_cast<const int4*>(xs + (size_t)b * kper * 256 + i * 256 + 64 * c);
              const int4 a0 = xp[0], a1 = xp[1], c0 = xp[2], c1 = xp[3];
              const int xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
              const int xc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
              int sl = 0, sh = 0;
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                sl = dp4a((int)(w[k] & 0x0F0F0F0Fu), xa[k], sl);
                sh = dp4a((int)((w[k] >> 4) & 0x0F0F0F0Fu), xc[k], sh);
              }
              const float4 g = *reinterpret_cast<const float4*>(xd + b * kper * 8 + i * 8 + 2 * c);
              acc[u][b] += fl * g.x * (float)sl - ml * g.y + fh * g.z * (float)sh - mh * g.w;
            }
          }
        }
      }
    }
    __syncthreads();                       // slab s fully consumed by every row
    if (t == 0 && ok && i + S < nk) issue(i + S);
  }
  if (!ok && t == 0)  // never exit with bulk copies still landing in this CTA's shared memory
    for (int i = max(0, issued - S); i < issued; ++i) mbar_wait(&bar->full[i % S], (i / S) & 1, nullptr, 50000000ull);

  // ---- split-K reduction (last CTA of the tile) ----
  if (splits > 1) {
    float* part = sc.ws + (((size_t)tile * splits + split) * kRows + t) * (W * MAXB);
#pragma unroll
    for (int u = 0; u < W; ++u)
#pragma unroll
      for (int b = 0; b < MAXB; ++b) part[u * MAXB + b] = acc[u][b];
    __threadfence();
    __syncthreads();
    if (t == 0) bar->last = (atomicAdd(&sc.counters[tile], 1) == splits - 1);
    __syncthreads();
    if (!bar->last) return;
    __threadfence();
    if (t == 0) sc.counters[tile] = 0;
#pragma unroll
    for (int u = 0; u < W; ++u)
#pragma unroll
      for (int b = 0; b < MAXB; ++b) acc[u][b] = 0.f;
    for (int sp = 0; sp < splits; ++sp) {
      const float* pp = sc.ws + (((size_t)tile * splits + sp) * kRows + t) * (W * MAXB);
#pragma unroll
      for (int u = 0; u < W; ++u)
#pragma unroll
        for (int b = 0; b < MAXB; ++b) acc[u][b] += __ldcg(pp + u * MAXB + b);
    }
  }

  // ---- epilogue ----
  const int row = tile * kRows + t;
  if (ep.mode == kEpiQKVRope) {
    // rows of this tile = one head: x0 = row i (< 64), x1 = row i + 64
    float* xch = reinterpret_cast<float*>(slabs);  // reuse the (drained) ring
    __syncthreads();
#pragma unroll
    for (int b = 0; b < MAXB; ++b) xch[b * kRows + t] = acc[0][b];
    __syncthreads();
    const int hd = ep.head_dim, half = hd / 2;
    if (t < half) {
      const int head = row / hd, i = t;
      const bool is_v = head >= ep.n_heads + ep.n_kv;
      const int rh = ep.rot_dim / 2;
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        if (b >= nB) break;
        float x0 = xch[b * kRows + t], x1 = xch[b * kRows + t + half];
        if (!is_v && i < rh) {
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
    return;
  }
  if (ep.mode == kEpiPeerPush) {
    const int e = *(volatile const int*)ep.push.epoch;
    if (row < N) {
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        if (b >= nB) break;
        peer_store(ep.push, e, (int64_t)b * ep.ld_out + row, acc[0][b]);
      }
    }
    return;
  }
  if (row >= N) return;
#pragma unroll
  for (int b = 0; b < MAXB; ++b) {
    if (b >= nB) break;
    const size_t o = (size_t)b * ep.ld_out + row;
    float v = acc[0][b];
    if (DUAL) v = v / (1.f + __expf(-v)) * acc[W - 1][b];
    if (ep.mode == kEpiResidual) {
      ep.resid[o] += v;
    } else {
      if (ep.out_f32) ep.out_f32[o] = v;
      if (ep.out_bf16) static_cast<__nv_bfloat16*>(ep.out_bf16)[o] = f2bf(v);
    }
  }
}

template <int MAXB, bool DUAL>
const char* launch_t(const GemvWeight& w, int N, int K, int B, const int8_t* xq, const float2* xds,
                     const GemvEpiParams& ep, const GemvTiledScratch& sc, int splits, cudaStream_t st) {
  const int tiles = (N + kRows - 1) / kRows;
  const int nsb = K / 256;
  const int kper = (nsb + splits - 1) / splits;
  constexpr int Wn = DUAL ? 2 : 1;
  const int S = kper < kMaxStages ? kper : kMaxStages;
  const size_t smem = (size_t)S * Wn * kSlab + (size_t)MAXB * kper * 256 + (size_t)MAXB * kper * 64 +
                      sizeof(Smem) + 64;
  if (smem > 227 * 1024) return "gemv_tiled: activation slice too large for shared memory (raise splits)";
  static size_t attr = 0;
  if (smem > attr) {
    if (cudaFuncSetAttribute(gemv_tiled_kernel<MAXB, DUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return "gemv_tiled: cudaFuncSetAttribute failed";
    attr = smem;
  }
  gemv_tiled_kernel<MAXB, DUAL><<<dim3(tiles, splits), kRows, smem, st>>>(
      static_cast<const uint8_t*>(w.data), static_cast<const uint8_t*>(ep.w2.data), N, K, B, xq, xds, ep, sc);
  return nullptr;
}

template <int MAXB>
const char* launch_b(const GemvWeight& w, int N, int K, int B, const int8_t* xq, const float2* xds,
                     const GemvEpiParams& ep, const GemvTiledScratch& sc, int splits, cudaStream_t st) {
  if (ep.mode == kEpiSwiGLU) return launch_t<MAXB, true>(w, N, K, B, xq, xds, ep, sc, splits, st);
  return launch_t<MAXB, false>(w, N, K, B, xq, xds, ep, sc, splits, st);
}

}  // namespace

int gemv_tiled_splits(int N, int K, int mode) {
  const int tiles = (N + kRows - 1) / kRows;
  const int nsb = K / 256;
  const int target = mode == kEpiSwiGLU ? 2 * 148 : 4 * 148;
  int s = (target + tiles - 1) / tiles;
  s = s < 1 ? 1 : s;
  const int max_s = nsb / 2 > 0 ? nsb / 2 : 1;   // at least two super-blocks per split
  return s > max_s ? max_s : s;
}

size_t gemv_tiled_workspace_floats(int N, int splits, int mode) {
  const size_t tiles = (N + kRows - 1) / kRows;
  return splits > 1 ? tiles * splits * kRows * 8 * (mode == kEpiSwiGLU ? 2 : 1) : 0;
}

size_t gemv_tiled_counters(int N) { return (N + kRows - 1) / kRows; }

static int gemv_wsplit() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("AIR_GEMV_WSPLIT");
    v = e ? atoi(e) : 1;
    if (v != 2 && v != 4 && v != 8 && v != 9 && v != 18) v = 1;
  }
  return v;
}

const char* launch_gemv_tiled(const GemvWeight& w, int N, int K, int B, const int8_t* xq,
                              const float2* xds, const GemvEpiParams& ep, const GemvTiledScratch& sc_in,
                              int splits, cudaStream_t st) {
  GemvTiledScratch sc = sc_in;
  if (sc.wsplit <= 0) sc.wsplit = gemv_wsplit();
  if (w.fmt != kFmtQ4K) return "gemv_tiled: Q4_K only";
  if (K % 256) return "gemv_tiled: K must be a multiple of 256";
  if (ep.mode == kEpiQKVRope && ep.head_dim != kRows) return "gemv_tiled: QKV epilogue needs head_dim 128";
  if (splits > 1 && (!sc.ws || !sc.counters)) return "gemv_tiled: split-K needs workspace and counters";
  if (B <= 1) return launch_b<1>(w, N, K, B, xq, xds, ep, sc, splits, st);
  if (B <= 2) return launch_b<2>(w, N, K, B, xq, xds, ep, sc, splits, st);
  if (B <= 4) return launch_b<4>(w, N, K, B, xq, xds, ep, sc, splits, st);
  return launch_b<8>(w, N, K, B, xq, xds, ep, sc, splits, st);
}

}  // namespace air
