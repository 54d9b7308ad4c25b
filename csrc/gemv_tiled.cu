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
constexpr int kMaxStages = 12;

struct Smem {
  uint64_t full[kMaxStages];
  int last;
  float scale[8];      // fused RMSNorm: 1/rms of each batch row
};

// Work range of CTA c: units [c * kper, min((c + 1) * kper, units)), unit = (tile,
// super-block) in the tiled layout's own order, so a CTA streams one contiguous byte range of
// each weight. When kper divides the super-blocks per tile (or the reverse) no range
// straddles a tile boundary.

// TPR threads per weight row (1 or 4); a thread covers 4 / TPR of the super-block's four
// 64-weight chunks. S ring stages of W slabs each.
template <int MAXB, bool DUAL, int TPR>
__global__ void __launch_bounds__(kRows * TPR)
gemv_tiled_kernel(const uint8_t* __restrict__ w1, const uint8_t* __restrict__ w2, int N, int K, int nB,
                  const int8_t* __restrict__ xq, const float2* __restrict__ xds, GemvEpiParams ep,
                  GemvTiledScratch sc, int S, int XW, int kper) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int W = DUAL ? 2 : 1;
  constexpr int CPT = 4 / TPR;                            // chunks per thread
  const int t = threadIdx.x;
  const int row_l = t / TPR, c4 = t % TPR;               // weight row of the tile, chunk group
  const int nsb = K / 256;
  const int tiles = (N + kRows - 1) / kRows;
  const int units = tiles * nsb;
  const int cta = blockIdx.x;
  const int u_begin = min(cta * kper, units), u_end = min(u_begin + kper, units);
  const int nk = u_end - u_begin;
  uint8_t* slabs = smem;                                          // [S][W][kSlab]
  float* xch = reinterpret_cast<float*>(smem + (size_t)S * W * kSlab);   // [MAXB][kRows]
  // activation window: the XW super-blocks this CTA touches (all of K when XW == nsb)
  int8_t* xs = reinterpret_cast<int8_t*>(xch + MAXB * kRows);              // [nB][XW][256]
  float2* xd = reinterpret_cast<float2*>(xs + (size_t)nB * XW * 256);      // [nB][XW][8]
  Smem* bar = reinterpret_cast<Smem*>(xd + (size_t)nB * XW * 8);
  const int sb_first = u_begin % nsb;

  if (t == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar->full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;
  auto issue = [&](int i) {
    const int s = i % S;
    issued = i + 1;
    mbar_expect_tx(&bar->full[s], W * kSlab);
    const size_t off = (size_t)(u_begin + i) * kSlab;
    const int np = sc.wsplit > 0 ? sc.wsplit : 1;     // split copies: more requests in flight
    const uint32_t piece = kSlab / np;
    for (int p = 0; p < np; ++p) {
      bulk_load(slabs + (size_t)(s * W) * kSlab + p * piece, w1 + off + p * piece, piece, &bar->full[s]);
      if (DUAL) bulk_load(slabs + (size_t)(s * W + 1) * kSlab + p * piece, w2 + off + p * piece, piece, &bar->full[s]);
    }
  };
  // Weights are never written by a kernel, so they stream in before the dependency on the
  // previous kernel (activations, residual, scratch) resolves.
  if (t == 0)
    for (int i = 0; i < min(S, nk); ++i) issue(i);
  pdl_wait();
  if (ep.ss_in) {
    // 1/rms per batch row from the producer's per-32-row partial sums, in a fixed order
    const int ng = ep.norm_k / 32, warp = t >> 5, lane = t & 31;
    for (int b = warp; b < nB; b += (kRows * TPR) >> 5) {
      float sum = 0.f;
      for (int g = lane; g < ng; g += 32) sum += __ldcg(ep.ss_in + (size_t)b * ng + g);
      sum = warp_sum(sum);
      if (lane == 0) bar->scale[b] = rsqrtf(sum / (float)ep.norm_k + ep.eps);
    }
  }
  {
    const int nw = XW == nsb ? nsb : min(nk, XW);
    for (int idx = t; idx < nB * nw * 20; idx += kRows * TPR) {
      const int b = idx / (nw * 20), r = idx % (nw * 20), j = r / 20, q = r % 20;
      const int sb = XW == nsb ? j : (sb_first + j) % nsb;
      if (q < 16) {
        reinterpret_cast<int4*>(xs + ((size_t)b * XW + j) * 256)[q] =
            __ldg(reinterpret_cast<const int4*>(xq + (size_t)b * K + (size_t)sb * 256) + q);
      } else {
        reinterpret_cast<int4*>(xd + ((size_t)b * XW + j) * 8)[q - 16] =
            __ldg(reinterpret_cast<const int4*>(xds + (size_t)b * (K / 32) + (size_t)sb * 8) + (q - 16));
      }
    }
  }
  __syncthreads();

  float acc[W][MAXB];
  auto zero = [&]() {
#pragma unroll
    for (int u = 0; u < W; ++u)
#pragma unroll
      for (int b = 0; b < MAXB; ++b) acc[u][b] = 0.f;
  };
  zero();

  // Epilogue of one finished 128-row tile (every lane of a row holds the full sums; lane c4
  // owns batch rows b with b % TPR == c4).
  auto epilogue = [&](int tile) {
    const int row = tile * kRows + row_l;
    if (ep.ss_in) {
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        const float sc = b < nB ? bar->scale[b] : 0.f;
#pragma unroll
        for (int u = 0; u < W; ++u) acc[u][b] *= sc;
      }
    }
    if (ep.mode == kEpiQKVRope) {
#pragma unroll
      for (int b = 0; b < MAXB; ++b)
        if ((b % TPR) == c4) xch[b * kRows + row_l] = acc[0][b];
      __syncthreads();
      const int hd = ep.head_dim, half = hd / 2;
      for (int pb = t; pb < half * nB; pb += kRows * TPR) {
      const int i = pb % half, b = pb / half;
      const int rowp = tile * kRows + i;
      {
        const int head = rowp / hd;
        const bool is_v = head >= ep.n_heads + ep.n_kv;
        const int rh = ep.rot_dim / 2;
        float x0 = xch[b * kRows + i], x1 = xch[b * kRows + i + half];
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
      __syncthreads();                     // xch is reused by the next tile
      return;
    }
    if (DUAL && TPR == 1 && ep.out_q) {
      // one warp = 32 consecutive rows = one Q8A group of the next GEMV's input
      if (tile * kRows + (row_l & ~31) >= ep.q_k) return;       // warp-uniform
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        if (b >= nB) break;
        float v = 0.f;
        if (row < N) v = gate_act(acc[0][b], ep.act) * acc[1][b];
        if (ep.out_f32) { if (row < N) ep.out_f32[(size_t)b * ep.ld_out + row] = v; }
        const float amax = warp_max(fabsf(v));
        const float dq = amax / 127.f;
        int qi = dq > 0.f ? __float2int_rn(v / dq) : 0;
        qi = max(-127, min(127, qi));
        ep.out_q[(size_t)b * ep.q_k + row] = (int8_t)qi;
        const int sq = warp_sum_i(qi);
        if ((t & 31) == 0) ep.out_ds[(size_t)b * (ep.q_k / 32) + row / 32] = make_float2(dq, dq * (float)sq);
      }
      return;
    }
    if (TPR == 1 && ep.norm_w) {
      // residual add + next RMSNorm's Q8A input and sum of squares (one warp = 32 rows)
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        if (b >= nB) break;
        float v = 0.f, y = 0.f;
        if (row < N) {
          const size_t o = (size_t)b * ep.ld_out + row;
          v = ep.resid[o] + acc[0][b];
          ep.resid[o] = v;
          y = v * (ep.norm_w[row] + ep.norm_offset);
        }
        const float amax = warp_max(fabsf(y));
        const float dq = amax / 127.f;
        int qi = dq > 0.f ? __float2int_rn(y / dq) : 0;
        qi = max(-127, min(127, qi));
        const float ss = warp_sum(v * v);
        if (row < ep.q_k) ep.out_q[(size_t)b * ep.q_k + row] = (int8_t)qi;
        const int sq = warp_sum_i(qi);
        if ((t & 31) == 0 && row < ep.q_k) {
          ep.out_ds[(size_t)b * (ep.q_k / 32) + row / 32] = make_float2(dq, dq * (float)sq);
          ep.ss_out[(size_t)b * (ep.q_k / 32) + row / 32] = ss;
        }
      }
      return;
    }
    if (row >= N) return;
    if (ep.mode == kEpiPeerPush) {
      const int e = *(volatile const int*)ep.push.epoch;
#pragma unroll
      for (int b = 0; b < MAXB; ++b)
        if ((b % TPR) == c4 && b < nB) peer_store(ep.push, e, b, row, acc[0][b]);
      return;
    }
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if ((b % TPR) != c4 || b >= nB) continue;
      const size_t o = (size_t)b * ep.ld_out + row;
      float v = acc[0][b];
      if (DUAL) v = gate_act(v, ep.act) * acc[W - 1][b];
      if (ep.mode == kEpiResidual) {
        ep.resid[o] += v;
      } else {
        if (ep.out_f32) ep.out_f32[o] = v;
        if (ep.out_bf16) static_cast<__nv_bfloat16*>(ep.out_bf16)[o] = f2bf(v);
      }
    }
  };

  // A tile's super-blocks done by this CTA: [sb_lo, sb_hi). Whole tile -> epilogue; else
  // publish the partial (slot 0: this CTA's first tile, slot 1: its last) and let the last
  // contributor of the tile (per-tile arrival counter over super-blocks) reduce.
  auto finish_tile = [&](int tile, int sb_lo, int sb_hi) {
    if (TPR > 1) {
#pragma unroll
      for (int u = 0; u < W; ++u)
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
          acc[u][b] += __shfl_xor_sync(0xffffffffu, acc[u][b], 1);
          acc[u][b] += __shfl_xor_sync(0xffffffffu, acc[u][b], 2);
        }
    }
    if (sb_hi - sb_lo == nsb) {
      epilogue(tile);
      return;
    }
    const int first_tile = u_begin / nsb;
    const int slot = tile == first_tile ? 0 : 1;
    float* part = sc.ws + (((size_t)cta * 2 + slot) * kRows + row_l) * (W * MAXB);
#pragma unroll
    for (int u = 0; u < W; ++u)
#pragma unroll
      for (int b = 0; b < MAXB; ++b)
        if ((b % TPR) == c4) part[u * MAXB + b] = acc[u][b];
    __threadfence();
    __syncthreads();
    if (t == 0) bar->last = (atomicAdd(&sc.counters[tile], sb_hi - sb_lo) + (sb_hi - sb_lo) == nsb);
    __syncthreads();
    if (!bar->last) return;
    __threadfence();
    if (t == 0) sc.counters[tile] = 0;
    // contributors: the CTAs whose ranges meet [tile*nsb, (tile+1)*nsb); their partials are
    // loaded four at a time so the L2 round trips overlap
    const int ua = tile * nsb, ub = ua + nsb;
    const int c_lo = ua / kper, c_hi = (ub - 1) / kper;
    // every partial (this CTA's own included) is summed in contributor order, so the result
    // does not depend on which CTA arrived last
    zero();
    for (int c0 = c_lo; c0 <= c_hi; c0 += 4) {
      float v[4][W][MAXB];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = c0 + j;
        const bool use = c <= c_hi;
        const int sl = (c * kper) / nsb == tile ? 0 : 1;
        const float* pp = sc.ws + (((size_t)(use ? c : 0) * 2 + sl) * kRows + row_l) * (W * MAXB);
#pragma unroll
        for (int u = 0; u < W; ++u)
#pragma unroll
          for (int b = 0; b < MAXB; ++b)
            v[j][u][b] = (use && (b % TPR) == c4) ? __ldcg(pp + u * MAXB + b) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int u = 0; u < W; ++u)
#pragma unroll
          for (int b = 0; b < MAXB; ++b) acc[u][b] += v[j][u][b];
    }
    epilogue(tile);
  };

  bool ok = true;
  int cur_tile = nk > 0 ? u_begin / nsb : -1, sb_lo = nk > 0 ? u_begin % nsb : 0;
  for (int i = 0; i < nk; ++i) {
    const int u_glob = u_begin + i;
    const int tile = u_glob / nsb, sb = u_glob % nsb;
    if (tile != cur_tile) {
      finish_tile(cur_tile, sb_lo, nsb);
      zero();
      cur_tile = tile;
      sb_lo = 0;
    }
    const int s = i % S;
    const int widx = XW == nsb ? sb : (sb - sb_first + nsb) % nsb;
    if (!mbar_wait(&bar->full[s], (i / S) & 1, ep.err)) {
      ok = false;
      set_error(ep.err, kErrTimeout);
    }
    if (ok) {
#pragma unroll
      for (int u = 0; u < W; ++u) {
        const uint8_t* rb = slabs + (size_t)(s * W + u) * kSlab + row_l * 144;
        const uint4 hd = *reinterpret_cast<const uint4*>(rb);
        const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) {
          const int c = c4 * CPT + cc;
          int scl, mnl, sch, mnh;
          q4k_scale_min(rb + 4, 2 * c, scl, mnl);
          q4k_scale_min(rb + 4, 2 * c + 1, sch, mnh);
          const uint4 qa = *reinterpret_cast<const uint4*>(rb + 16 + 32 * c);
          const uint4 qb = *reinterpret_cast<const uint4*>(rb + 32 + 32 * c);
          const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
          const float fl = d * (float)scl, ml = dmin * (float)mnl;
          const float fh = d * (float)sch, mh = dmin * (float)mnh;
#pragma unroll
          for (int b = 0; b < MAXB; ++b) {
            if (b < nB) {
              const int4* xp = reinterpret_cast<const int4*>(xs + ((size_t)b * XW + widx) * 256 + 64 * c);
              const int4 a0 = xp[0], a1 = xp[1], e0 = xp[2], e1 = xp[3];
              const int xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
              const int xc[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
              int sl = 0, sh = 0;
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                sl = dp4a((int)(w[k] & 0x0F0F0F0Fu), xa[k], sl);
                sh = dp4a((int)((w[k] >> 4) & 0x0F0F0F0Fu), xc[k], sh);
              }
              const float4 g = *reinterpret_cast<const float4*>(xd + ((size_t)b * XW + widx) * 8 + 2 * c);
              acc[u][b] += fl * g.x * (float)sl - ml * g.y + fh * g.z * (float)sh - mh * g.w;
            }
          }
        }
      }
    }
    __syncthreads();                       // slab s fully consumed by every row
    if (t == 0 && ok && i + S < nk) issue(i + S);
  }
  if (sc.early_trigger) pdl_trigger();   // a dependent GEMV's weights stream during these tiles
  if (nk > 0) finish_tile(cur_tile, sb_lo, (u_end - 1) / nsb == cur_tile ? (u_end - 1) % nsb + 1 : nsb);
  if (!ok && t == 0)  // never exit with bulk copies still landing in this CTA's shared memory
    for (int i = max(0, issued - S); i < issued; ++i) mbar_wait(&bar->full[i % S], (i / S) & 1, nullptr, 50000000ull);
}

struct GemvCfg {
  int tpr, stages;
};

// Threads per row and ring depth: AIR_GEMV_TPR (1 | 4), AIR_GEMV_STAGES (slabs of W
// weights per CTA). Defaults: one thread per row, 3 stages (2 for SwiGLU's pair of weights);
// the grid is as many CTAs as fit at once (several per SM), so that whole units from
// different CTAs are in flight together.
static GemvCfg gemv_cfg(bool dual) {
  static int tpr = -1, st = -1;
  if (tpr < 0) {
    const char* e = getenv("AIR_GEMV_TPR");
    tpr = (e && atoi(e) == 4) ? 4 : 1;
    const char* f = getenv("AIR_GEMV_STAGES");
    st = f ? atoi(f) : 0;
    if (st < 0 || st > kMaxStages) st = 0;
  }
  GemvCfg c;
  c.tpr = tpr;
  c.stages = st > 0 ? st : (dual ? 2 : 3);
  return c;
}

static bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("AIR_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <int MAXB, bool DUAL, int TPR>
const char* launch_t(const GemvWeight& w, int N, int K, int B, const int8_t* xq, const float2* xds,
                     const GemvEpiParams& ep, const GemvTiledScratch& sc, int cap, int S, cudaStream_t st) {
  constexpr int Wn = DUAL ? 2 : 1;
  const int nsb = K / 256;
  const long long units = (long long)((N + kRows - 1) / kRows) * nsb;
  auto smem_for = [&](int kper) {
    const int xw = kper < nsb ? kper : nsb;
    return (size_t)S * Wn * kSlab + (size_t)MAXB * kRows * sizeof(float) + (size_t)B * xw * 320 +
           sizeof(Smem) + 64;
  };
  // units per CTA: at least two (fewer partial tiles to reduce), else enough that the grid
  // fits on the GPU at once
  auto kper_for = [&](long long max_grid) {
    long long k = (units + max_grid - 1) / max_grid;
    if (k < 2) k = 2;
    return (int)k;
  };
  static unsigned long long attr_done = 0;
  if (!set_max_smem_per_device(gemv_tiled_kernel<MAXB, DUAL, TPR>, 227 * 1024, attr_done))
    return "gemv_tiled: cudaFuncSetAttribute failed";
  int kper = kper_for(cap);
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_tiled_kernel<MAXB, DUAL, TPR>, kRows * TPR,
                                                    smem_for(kper)) != cudaSuccess || occ < 1)
    occ = 1;
  const long long resident = 148LL * occ;
  kper = kper_for(resident < cap ? resident : cap);
  const int grid = (int)((units + kper - 1) / kper);
  const int XW = kper < nsb ? kper : nsb;
  const size_t smem = smem_for(kper);
  if (smem > 227 * 1024) return "gemv_tiled: ring + activation window too large";
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kRows * TPR);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, gemv_tiled_kernel<MAXB, DUAL, TPR>, static_cast<const uint8_t*>(w.data),
                         static_cast<const uint8_t*>(ep.w2.data), N, K, B, xq, xds, ep, sc, S, XW, kper) != cudaSuccess)
    return "gemv_tiled: launch failed";
  return nullptr;
}

template <int MAXB>
const char* launch_b(const GemvWeight& w, int N, int K, int B, const int8_t* xq, const float2* xds,
                     const GemvEpiParams& ep, const GemvTiledScratch& sc, int grid, cudaStream_t st) {
  const bool dual = ep.mode == kEpiSwiGLU;
  GemvCfg c = gemv_cfg(dual);
  if (ep.out_q || ep.norm_w) c.tpr = 1;   // the quantising epilogues map one warp to 32 rows
  if (dual)
    return c.tpr == 4 ? launch_t<MAXB, true, 4>(w, N, K, B, xq, xds, ep, sc, grid, c.stages, st)
                      : launch_t<MAXB, true, 1>(w, N, K, B, xq, xds, ep, sc, grid, c.stages, st);
  return c.tpr == 4 ? launch_t<MAXB, false, 4>(w, N, K, B, xq, xds, ep, sc, grid, c.stages, st)
                    : launch_t<MAXB, false, 1>(w, N, K, B, xq, xds, ep, sc, grid, c.stages, st);
}

}  // namespace

// The launch is persistent: "splits" is the number of CTAs (a few per SM), each streaming a
// contiguous run of (tile, super-block) units.
int gemv_tiled_splits(int N, int K, int mode) {
  const long long units = (long long)((N + kRows - 1) / kRows) * (K / 256);
  (void)mode;
  const long long g = 148LL * 4;    // upper bound; the launch sizes the grid by occupancy
  return (int)(units < g ? units : g);
}

size_t gemv_tiled_workspace_floats(int N, int splits, int mode) {
  (void)N;
  return (size_t)splits * 2 * kRows * 8 * (mode == kEpiSwiGLU ? 2 : 1);
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
  if (sc.early_trigger < 0) {
    static int v = -1;
    if (v < 0) {
      const char* e = getenv("AIR_PDL_EARLY");
      v = (e && e[0] == '0') ? 0 : 1;
    }
    sc.early_trigger = v;
  }
  if (w.fmt != kFmtQ4K) return "gemv_tiled: Q4_K only";
  if (K % 256) return "gemv_tiled: K must be a multiple of 256";
  if (ep.mode == kEpiQKVRope && ep.head_dim != kRows) return "gemv_tiled: QKV epilogue needs head_dim 128";
  if (splits < 1) return "gemv_tiled: grid must be >= 1";
  if (!sc.ws || !sc.counters) return "gemv_tiled: needs workspace and counters";
  if (B <= 1) return launch_b<1>(w, N, K, B, xq, xds, ep, sc, splits, st);
  if (B <= 2) return launch_b<2>(w, N, K, B, xq, xds, ep, sc, splits, st);
  if (B <= 4) return launch_b<4>(w, N, K, B, xq, xds, ep, sc, splits, st);
  return launch_b<8>(w, N, K, B, xq, xds, ep, sc, splits, st);
}

}  // namespace air
