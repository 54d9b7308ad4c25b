// Dequant-fused tensor-core GEMM for the prefill / batched-decode path (sm_100a):
//     out[t, n] (op)= sum_k x[t, k] * W[n, k]
// with W in raw GGUF Q4_K blocks (or dense bf16) and x bf16 activations.
//
// Swap-AB tiling: the MMA's M = 128 weight rows, its N = a tile of NT tokens, so small
// decode batches (16..128 tokens) still fill the 128-row tcgen05 datapath. Per CTA:
//   warp 0      TMA producer: raw weight box (128 rows x one 256-weight super-block, the
//               144-byte GGUF blocks copied verbatim) + the matching x boxes (SW128 swizzle)
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer (f32 accumulators in TMEM)
//   warps 2..    (8 or 16 of them) dequantise the staged Q4_K blocks into bf16 K-major SW128 tiles with packed
//               bf16x2 arithmetic (the GGUF scale/min math), then run the epilogue
//               (tcgen05.ld -> store / residual add / split-K reduction).
// Stages are handed over with mbarriers (TMA complete_tx, tcgen05.commit). Split-K uses a
// caller-provided fp32 workspace and per-tile arrival counters; the last CTA of a tile
// reduces the partials and resets its counter, so the scratch needs no clearing per call.
//
// Replaces the reference's candle QMatMul GEMM path (src/model.rs:534-536, 591-594,
// src/ops.rs:594-611 via candle-core's CUDA quantized matmul).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp8.h>
#include "common.cuh"
#include "sm100.cuh"
#include "gemm_tc.h"
#include "comm.cuh"
#include <stdlib.h>
#include <string.h>

namespace air {

namespace {

using namespace sm100;

constexpr int kRawRowBytes = 144;           // one Q4_K super-block of one row
constexpr int kRawTile = 128 * kRawRowBytes; // 18432 B (multiple of 1024)
// Q8_0 stage of 128 rows x 256 weights: the int8 codes as two 128-byte-wide SW128 TMA boxes
// (16 KB each) plus the eight f16 block scales per row (one 16-byte box row): 34 KB
constexpr int kQ8Half = 128 * 128;
constexpr int kQ8Tile = 2 * kQ8Half + 128 * 16;
constexpr int kATile = 128 * 128;            // 128 rows x 64 bf16

template <int NT, int FMT, int NA, bool AT, int NACC = 1, int CPS = 1>
struct Cfg {
  static constexpr int kChunks = FMT == kFmtQ4K ? 4 : 1;         // 64-wide K chunks per stage
  static constexpr int kBChunk = NT * 128;                       // NT rows x 128 B
  static constexpr int kStageBytes = (FMT == kFmtQ4K ? kRawTile : kATile) + kChunks * kBChunk;
  // dequantised A in shared memory (NA 64-wide chunks), unless AT: then it lives in TMEM
  static constexpr int kABuf = (FMT == kFmtQ4K && !AT) ? NA * kATile : 0;
  static constexpr int kBudget = 227 * 1024 - 2048 - 1024;
  static constexpr int kStages = (kBudget - kABuf) / kStageBytes > 8 ? 8 : (kBudget - kABuf) / kStageBytes;
  static constexpr int kSmem = 1024 + kStages * kStageBytes + kABuf + 1024;
  // AT: NACC interleaved accumulators (K steps alternate between them, so consecutive MMAs
  // do not wait on each other's result) in the low columns, then 128-column stage buffers of
  // A up to column 512 (three when the accumulators fit in 128 columns, else two)
  // CPS = 2 (decode shapes): two CTAs per SM, each with half of the shared memory and of
  // TMEM; A is handed over in half-stage units (two 64-wide chunks, 64 columns)
  static constexpr int kAccW = NT < 32 ? 32 : NT;
  static constexpr int kTmemCols = AT ? (CPS == 2 ? 256 : 512) : (NT < 32 ? 32 : NT);
  static constexpr int kUA = CPS == 2 ? 2 : 4;            // 64-wide chunks per A unit
  static constexpr int kUPS = 4 / kUA;                    // A units per stage
  static constexpr int kATmemCol = AT ? (CPS == 2 ? NACC * kAccW : (NACC * kAccW > 128 ? NACC * kAccW : 128)) : 128;
  static constexpr int kAbufs = AT ? (kTmemCols - kATmemCol) / (32 * kUA) : NA;
  static_assert(!AT || kAbufs >= 2, "TMEM: not enough room for two A buffers");
  static_assert(kAbufs <= 4, "A buffer barriers");
  static_assert(AT || kStages >= 2, "not enough shared memory for two stages");
  // AT: decoupled rings — raw weight tiles (streamed from HBM, as many in flight as fit) and
  // activation tiles (L2-resident, a short ring), each with its own producer warp
  // activation ring: one item per K stage (four 64-wide chunks) for token tiles up to 128;
  // 256-token tiles stage single chunks (a whole stage would be 128 KB), and the MMA frees a
  // chunk as soon as its four K16 steps are issued
  // (Q8_0 weight tiles are twice the Q4_K size: the two-CTA decode variant stages chunks too)
  static constexpr int kXC = (NT >= 256 || (FMT != kFmtQ4K && CPS == 2)) ? 1 : 4;   // chunks per X item
  static constexpr int kXStage = kXC * kBChunk;
  static constexpr int kXStages = kXC == 1 ? (NT >= 256 ? 3 : 4) : ((NT >= 64 || CPS == 2) ? 2 : 3);
  // one raw weight stage: Q4_K tile / Q8_0 codes + scales / FP8 codes (scales read directly)
  static constexpr int kWTile = FMT == kFmtQ8_0 ? kQ8Tile : (FMT == kFmtFP8 ? 2 * kQ8Half : kRawTile);
  static constexpr int kBudgetAT = CPS == 2 ? 112 * 1024 - 2048 : kBudget;
  static constexpr int kWStagesRaw = (kBudgetAT - kXStages * kXStage) / kWTile;
  static constexpr int kWStages = kWStagesRaw > 12 ? 12 : kWStagesRaw;
  static constexpr int kSmemAT = 1024 + kWStages * kWTile + kXStages * kXStage + 1024;
  static_assert(!AT || kWStages >= 2, "not enough shared memory for two raw weight stages");
  static constexpr int kFirstDq = AT ? 3 : 2;       // first dequant/epilogue warp
  static constexpr int kSmemLaunch = AT ? kSmemAT : kSmem;
};

// Per-group weight tensor maps of a grouped launch (unused otherwise).
struct GroupMaps {
  CUtensorMap w[kGemmMaxGroups];
  CUtensorMap s[kGemmMaxGroups];
};

struct Bars {
  uint64_t full[12];
  uint64_t empty[12];
  uint64_t xfull[8];
  uint64_t xempty[8];
  uint64_t afull[4];
  uint64_t aempty[4];
  uint64_t done;
  uint32_t tmem;
  int abort;
  int last;
};

// Sum of the NACC interleaved accumulators (kAccW columns apart) for 16 columns.
template <int ACCW, int NACC>
__device__ __forceinline__ void load_acc(uint32_t taddr, float (&v)[16]) {
  tmem_ld16(taddr, v);
#pragma unroll
  for (int j = 1; j < NACC; ++j) {
    float w[16];
    tmem_ld16(taddr + ACCW * j, w);
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] += w[e];
  }
}

template <int DQ>
__device__ __forceinline__ void named_sync_epi() { asm volatile("bar.sync 1, %0;" ::"n"(32 * DQ) : "memory"); }

// One 16-byte output chunk (8 bf16) = s * q - mm for 8 nibbles taken from 2 words.
__device__ __forceinline__ uint32_t q4_pair(uint32_t t, __nv_bfloat162 s, __nv_bfloat162 negm) {
  const uint32_t v = (t & 0x000F000Fu) | 0x43004300u;         // bf16x2 (128 + q0, 128 + q1)
  __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&v);
  const __nv_bfloat162 c128 = __floats2bfloat162_rn(128.f, 128.f);
  b = __hsub2(b, c128);                                          // exact q
  b = __hfma2(b, s, negm);
  return *reinterpret_cast<uint32_t*>(&b);
}

template <int NT, int FMT, int NA, int DQ, bool AT, int NACC, int CPS>
__global__ void __launch_bounds__((AT ? 96 : 64) + 32 * DQ, CPS)
gemm_q_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_x,
              const __grid_constant__ CUtensorMap tm_s0, const __grid_constant__ GroupMaps gm,
              const __grid_constant__ GemmArgs a) {
  using C = Cfg<NT, FMT, NA, AT, NACC, CPS>;
  static_assert(!AT || FMT == kFmtQ4K || FMT == kFmtQ8_0 || FMT == kFmtFP8, "A-in-TMEM path: Q4_K, Q8_0, FP8");
  // Programmatic dependent launch: this grid may start while the previous kernel finishes.
  // Set-up, the weight stream (read-only), the dequantisation and the MMAs run ahead; the
  // activation producer and the epilogue (the only readers of activations / scratch and the
  // only global writers) wait for the previous grid first (griddepcontrol.wait), as does
  // everything when a device row count gates the tiles.
  if (a.row_count != nullptr) pdl_wait();
  pdl_trigger();
  // grouped launch: this CTA's group (routed expert) and token tile; the per-group weight
  // pointers, tensor maps and row range are looked up where they are used (GROUP_* below),
  // so they hold no registers across the kernel
  const int grp = a.groups > 0 ? (int)blockIdx.y / a.tiles_per_group : 0;
  const int ty = a.groups > 0 ? (int)blockIdx.y % a.tiles_per_group : (int)blockIdx.y;
#define GROUP_ROWBASE (a.groups > 0 ? grp * a.group_rows : 0)
#define GROUP_TLIM (a.groups > 0 ? a.group_rows : a.T)
#define GROUP_WQ (a.groups > 0 ? a.wq_g[grp] : a.wq)
#define GROUP_TMW (a.groups > 0 ? &gm.w[grp] : &tm_w0)
#define GROUP_TMS (a.groups > 0 ? &gm.s[grp] : &tm_s0)
#define GROUP_WSCALES static_cast<const float*>(a.groups > 0 ? a.wscales_g[grp] : a.wscales)
  // routed-expert GEMMs: token tiles beyond the device row count do nothing (uniform per CTA,
  // before any barrier, TMEM allocation or copy)
  if (a.row_count != nullptr && ty * NT >= *(volatile const int*)(a.row_count + grp)) return;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* abuf = stages + C::kStages * C::kStageBytes;
  // AT lays out [weight ring][activation ring] instead; the barriers follow whichever layout
  Bars* bars = reinterpret_cast<Bars*>(AT ? stages + C::kWStages * C::kWTile + C::kXStages * C::kXStage
                                          : abuf + C::kABuf);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * 128, n0 = ty * NT;   // n0: first token row within the group
  const int split = blockIdx.z, splits = gridDim.z;
  const int ksteps = FMT == kFmtBF16 ? a.K / 64 : a.K / 256;
  const int kper = (ksteps + splits - 1) / splits;
  const int kb0 = split * kper;
  const int nk = max(0, min(ksteps, kb0 + kper) - kb0);

  if (threadIdx.x == 0) {
    if constexpr (AT) {
      for (int s = 0; s < C::kWStages; ++s) {
        mbar_init(&bars->full[s], 1);
        mbar_init(&bars->empty[s], 8);        // the dequant group that read the raw tile
      }
      for (int s = 0; s < C::kXStages; ++s) {
        mbar_init(&bars->xfull[s], 1);
        mbar_init(&bars->xempty[s], 1);       // MMA commit
      }
    } else {
      for (int s = 0; s < C::kStages; ++s) {
        mbar_init(&bars->full[s], 1);
        mbar_init(&bars->empty[s], FMT == kFmtQ4K ? DQ + 1 : 1);
      }
    }
    for (int i = 0; i < (AT ? C::kAbufs : NA); ++i) {
      mbar_init(&bars->afull[i], AT ? 8 : DQ);
      mbar_init(&bars->aempty[i], 1);
    }
    mbar_init(&bars->done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    if (FMT != kFmtQ4K) prefetch_tmap(GROUP_TMW);
    if (FMT == kFmtQ8_0) prefetch_tmap(GROUP_TMS);
    prefetch_tmap(&tm_x);
  }
  if (warp == 1) tmem_alloc(&bars->tmem, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  long long* dbg = (a.dbg && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) ? a.dbg : nullptr;
  // profiling aid (dbg[255], only with a dbg buffer): 1 = skip the dequant math, 2 = skip the MMAs
  const int dmode = a.dbg ? (int)a.dbg[255] : 0;
  if (dbg && threadIdx.x == 0) dbg[225] = clock64();

  if (AT && (warp == 0 || warp == 2)) {
    // ------------------------------------------------------------ producers (AT)
    // warp 0: raw weight tiles into the deep ring; warp 2: activation tiles into the short ring
    if (lane == 0) {
      // items: one raw weight tile per K stage (warp 0), one 64-wide activation chunk per
      // quarter stage (warp 2)
      const bool wprod = warp == 0;
      const int S = wprod ? C::kWStages : C::kXStages;
      uint64_t* fullb = wprod ? bars->full : bars->xfull;
      uint64_t* emptyb = wprod ? bars->empty : bars->xempty;
      uint8_t* ring = wprod ? stages : stages + C::kWStages * C::kWTile;
      const uint32_t bytes = wprod ? C::kWTile : C::kXStage;
      const int items = wprod ? nk : nk * (4 / C::kXC);
      if (!wprod) pdl_wait();                          // activations come from the previous kernel
      int issued = 0;
      for (int i = 0; i < items; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait(&emptyb[s], ((i / S) - 1) & 1, a.err)) {
          set_error(a.err, kErrTimeout);
          bars->abort = 1;
          break;
        }
        if (*(volatile int*)&bars->abort) break;
        uint8_t* st = ring + s * bytes;
        if (dbg && wprod && i < 32) dbg[i] = clock64();
        mbar_expect_tx(&fullb[s], bytes);
        if (wprod && (FMT == kFmtQ8_0 || FMT == kFmtFP8)) {
          // codes [rows m0.., K kb*256..] as two SW128 boxes; Q8_0 then the rows' eight scales
          const int kb = kb0 + i;
          tma_load_2d(st, GROUP_TMW, &fullb[s], kb * 256, m0);
          tma_load_2d(st + kQ8Half, GROUP_TMW, &fullb[s], kb * 256 + 128, m0);
          if (FMT == kFmtQ8_0) tma_load_2d(st + 2 * kQ8Half, GROUP_TMS, &fullb[s], kb * 8, m0);
        } else if (wprod) {
          // the tile as a.wsplit back-to-back bulk copies (more requests in flight per CTA)
          const uint8_t* src = GROUP_WQ + ((size_t)blockIdx.x * ksteps + kb0 + i) * kRawTile;
          const int np = a.wsplit > 0 ? a.wsplit : 1;
          const uint32_t piece = kRawTile / np;
          for (int p = 0; p < np; ++p) bulk_load(st + p * piece, src + p * piece, piece, &fullb[s]);
        } else {
#pragma unroll
          for (int c = 0; c < C::kXC; ++c) {
            const int ch = i * C::kXC + c;              // chunk index along K
            tma_load_2d(st + c * C::kBChunk, &tm_x, &fullb[s], (kb0 + ch / 4) * 256 + 64 * (ch % 4), GROUP_ROWBASE + n0);
          }
        }
        issued = i + 1;
      }
      for (int i = max(0, issued - S); i < issued; ++i)
        mbar_wait(&fullb[i % S], (i / S) & 1, a.err, 50ull * 1000 * 1000);
    }
  } else if (!AT && warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      pdl_wait();                                      // the stages carry activations
      const uint32_t tx = C::kStageBytes;
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::kStages;
        if (i >= C::kStages && !mbar_wait(&bars->empty[s], ((i / C::kStages) - 1) & 1, a.err)) {
          set_error(a.err, kErrTimeout);
          bars->abort = 1;
          break;
        }
        if (*(volatile int*)&bars->abort) break;
        uint8_t* st = stages + s * C::kStageBytes;
        if (dbg && i < 32) dbg[i] = clock64();
        mbar_expect_tx(&bars->full[s], tx);
        const int kb = kb0 + i;
        if (FMT == kFmtQ4K) {
          // tiled Q4_K: the 128-row x 256-weight tile is 18 KB contiguous -> one bulk copy
          bulk_load(st, GROUP_WQ + ((size_t)blockIdx.x * ksteps + kb) * kRawTile, kRawTile, &bars->full[s]);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            tma_load_2d(st + kRawTile + c * C::kBChunk, &tm_x, &bars->full[s], kb * 256 + 64 * c, GROUP_ROWBASE + n0);
        } else {
          tma_load_2d(st, GROUP_TMW, &bars->full[s], kb * 64, m0);
          tma_load_2d(st + kATile, &tm_x, &bars->full[s], kb * 64, GROUP_ROWBASE + n0);
        }
        issued = i + 1;
      }
      // never leave the CTA with copies in flight into its shared memory
      for (int i = max(0, issued - C::kStages); i < issued; ++i)
        mbar_wait(&bars->full[i % C::kStages], (i / C::kStages) & 1, a.err, 50ull * 1000 * 1000);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, NT);
      int g = 0;
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        if constexpr (AT) {
          uint8_t* xring = stages + C::kWStages * C::kWTile;
          for (int u = 0; u < C::kUPS && ok; ++u) {
            const int g = i * C::kUPS + u;
            const int ab = g % C::kAbufs;
            if (!mbar_wait(&bars->afull[ab], (g / C::kAbufs) & 1, a.err)) { ok = false; break; }
            tc_fence_after();
            if (dbg && u == 0 && i < 64) dbg[32 + i] = clock64();
            const uint32_t ta = tmem + C::kATmemCol + 32 * C::kUA * ab;
#pragma unroll
            for (int cu = 0; cu < C::kUA; ++cu) {
              const int c = u * C::kUA + cu;
              const int gc = 4 * i + c;                 // activation chunk
              const int gx = gc / C::kXC;               // its X ring item
              const int xs = gx % C::kXStages;
              if (gc % C::kXC == 0) {
                if (!mbar_wait(&bars->xfull[xs], (gx / C::kXStages) & 1, a.err)) { ok = false; break; }
                tc_fence_after();
              }
              const uint64_t bd = sw128_desc(xring + xs * C::kXStage + (gc % C::kXC) * C::kBChunk);
#pragma unroll
              for (int k = 0; k < 4; ++k) {  // K16 steps: 8 TMEM columns of A, +32 B of B
                const int j = (4 * c + k) % NACC;       // interleaved accumulators
                const uint32_t acc = (i == 0 && 4 * c + k < NACC) ? 0u : 1u;
                if (dmode != 2)
                  mma_bf16_ts(tmem + C::kAccW * j, ta + 32 * cu + 8 * k, bd + 2 * k, idesc, acc);
              }
              if (gc % C::kXC == C::kXC - 1) mma_commit(&bars->xempty[xs]);   // item read once these retire
            }
            if (!ok) break;
            mma_commit(&bars->aempty[ab]);
          }
          if (!ok) break;
          continue;
        }
        const int s = i % C::kStages;
        if (!mbar_wait(&bars->full[s], (i / C::kStages) & 1, a.err)) { ok = false; break; }
        uint8_t* st = stages + s * C::kStageBytes;
        for (int c = 0; c < C::kChunks; ++c, ++g) {
          const uint8_t* A;
          if (FMT == kFmtQ4K) {
            const int ab = g % NA;
            if (!mbar_wait(&bars->afull[ab], (g / NA) & 1, a.err)) { ok = false; break; }
            A = abuf + ab * kATile;
          } else {
            A = st;
          }
          tc_fence_after();
          if (dbg && g < 64) dbg[32 + g] = clock64();
          const uint64_t ad = sw128_desc(A);
          const uint64_t bd = sw128_desc(st + (FMT == kFmtQ4K ? kRawTile : kATile) + c * C::kBChunk);
#pragma unroll
          for (int k = 0; k < 4; ++k)  // 4 x K16 per 64-wide chunk: +32 B along K
            mma_bf16(tmem, ad + 2 * k, bd + 2 * k, idesc, (i | c | k) != 0 ? 1u : 0u);
          if (FMT == kFmtQ4K) mma_commit(&bars->aempty[g % NA]);
        }
        mma_commit(&bars->empty[s]);
      }
      if (!ok) {
        set_error(a.err, kErrTimeout);
        bars->abort = 1;
      }
      mma_commit(&bars->done);
    }
  } else {
    // ------------------------------------------------------------ dequant (Q4_K)
    // Thread = (weight row t, nibble half hf, code-byte part sub): hf = 0 expands the low
    // nibbles (sub-blocks 0,2,4,6 of the super-block), hf = 1 the high nibbles (1,3,5,7);
    // with 16 warps each (row, half) is further split into two 16-byte parts. Scales are
    // decoded once per stage; per 64-wide chunk a thread turns its code bytes into bf16 with
    // 3 ops per pair: PRMT places two nibbles under a 0x43 exponent byte (= 128 + q, exact),
    // HSUB2 removes the 128, HFMA2 applies d*sc and -dmin*m.
    constexpr int kParts = DQ / 8;             // 1 or 2 code-byte parts per (row, half)
    constexpr int kWords = 8 / kParts;          // 32-bit code words per thread per chunk
    const int t = (threadIdx.x - 64) & 127;
    const int hf = ((threadIdx.x - 64) >> 7) / kParts;   // warp-uniform
    const int sub = ((threadIdx.x - 64) >> 7) % kParts;
    if constexpr (AT) {
      // A in TMEM: warp w owns TMEM lanes 32*(w%4).. (rows), h = which nibble half; per
      // stage a thread writes 4 chunks x 16 columns of its row (two bf16 per column), then
      // one wait::st + fence + arrive hands the whole stage to the MMA issuer. With 16
      // warps, two groups of 8 take alternate stages, so one group's fixed per-stage
      // latency (shared-memory loads, TMEM store completion) overlaps the other's work;
      // three TMEM stage buffers let both groups run ahead of the MMA.
      constexpr int G = DQ / 8;
      const int grp = (warp - C::kFirstDq) >> 3;
      const int r = 32 * (warp & 3) + lane;
      const int h = ((warp - C::kFirstDq) >> 2) & 1;
      const __nv_bfloat162 c128 = __floats2bfloat162_rn(128.f, 128.f);
      bool ok = true;
      for (int i = grp; i < nk && ok; i += G) {
        const int s = i % C::kWStages;
        if (!mbar_wait(&bars->full[s], (i / C::kWStages) & 1, a.err)) { ok = false; break; }
        if (dbg && threadIdx.x == 32 * C::kFirstDq && i < 64) dbg[96 + i] = clock64();
        const uint8_t* rb = stages + s * C::kWTile + r * kRawRowBytes;
        float d = 0.f, dmin = 0.f;
        if constexpr (FMT == kFmtQ4K) {
          const uint32_t hdr = *reinterpret_cast<const uint32_t*>(rb);
          d = __half2float(__ushort_as_half((unsigned short)(hdr & 0xFFFF)));
          dmin = __half2float(__ushort_as_half((unsigned short)(hdr >> 16)));
        }
        const uint8_t* q8 = stages + s * C::kWTile;     // Q8_0: [2 SW128 halves][scales]
        const uint32_t tlane = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + C::kATmemCol + 16 * h;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int g = i * C::kUPS + c / C::kUA;     // A unit of this chunk
          const int ab = g % C::kAbufs;
          if (c % C::kUA == 0 && g >= C::kAbufs &&
              !mbar_wait(&bars->aempty[ab], ((g / C::kAbufs) - 1) & 1, a.err)) { ok = false; break; }
          const uint32_t ta = tlane + 32 * C::kUA * ab - 32 * (c / C::kUA) * C::kUA;
          uint32_t o[16];
          if constexpr (FMT == kFmtFP8) {
            // 32 E4M3 codes of row r (two 16-byte chunks of its SW128 half) x the f32 multiplier
            // of K block (kb * 256 + 64 c) / 128
            const uint8_t* row = q8 + (c >> 1) * kQ8Half + r * 128;
            const int j0 = 4 * (c & 1) + 2 * h;
            const uint4 qa = *reinterpret_cast<const uint4*>(row + ((j0 ^ (r & 7)) << 4));
            const uint4 qb = *reinterpret_cast<const uint4*>(row + (((j0 + 1) ^ (r & 7)) << 4));
            const int grow = m0 + r;
            const float dq = grow < a.N ? __ldg(GROUP_WSCALES +
                                               (size_t)grow * (a.K / 128) + (kb0 + i) * 2 + (c >> 1))
                                        : 0.f;
            const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
                    (__nv_fp8x2_storage_t)((w[k] >> (16 * e)) & 0xFFFF), __NV_E4M3);
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&hr));
                __nv_bfloat162 b = __floats2bfloat162_rn(v.x * dq, v.y * dq);
                o[2 * k + e] = *reinterpret_cast<uint32_t*>(&b);
              }
            }
          } else if constexpr (FMT == kFmtQ8_0) {
            // block 2c + h of the stage: 32 codes = two 16-byte chunks of row r's SW128 half
            const uint8_t* row = q8 + (c >> 1) * kQ8Half + r * 128;
            const int j0 = 4 * (c & 1) + 2 * h;
            const uint4 qa = *reinterpret_cast<const uint4*>(row + ((j0 ^ (r & 7)) << 4));
            const uint4 qb = *reinterpret_cast<const uint4*>(row + (((j0 + 1) ^ (r & 7)) << 4));
            const float dq = __half2float(*reinterpret_cast<const __half*>(q8 + 2 * kQ8Half + r * 16 + (2 * c + h) * 2));
            const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int32_t v = (int32_t)w[k];
              const float f0 = (float)(int8_t)(v & 0xFF), f1 = (float)(int8_t)((v >> 8) & 0xFF);
              const float f2 = (float)(int8_t)((v >> 16) & 0xFF), f3 = (float)(int8_t)(v >> 24);
              __nv_bfloat162 b0 = __floats2bfloat162_rn(f0 * dq, f1 * dq);
              __nv_bfloat162 b1 = __floats2bfloat162_rn(f2 * dq, f3 * dq);
              o[2 * k] = *reinterpret_cast<uint32_t*>(&b0);
              o[2 * k + 1] = *reinterpret_cast<uint32_t*>(&b1);
            }
          } else {
            int sc, mn;
            q4k_scale_min(rb + 4, 2 * c + h, sc, mn);
            const __nv_bfloat162 sv = __float2bfloat162_rn(d * (float)sc);
            const __nv_bfloat162 mv = __float2bfloat162_rn(-dmin * (float)mn);
            const uint4 qa = *reinterpret_cast<const uint4*>(rb + 16 + 32 * c);
            const uint4 qb = *reinterpret_cast<const uint4*>(rb + 32 + 32 * c);
            uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t wk = h ? (w[k] >> 4) & 0x0F0F0F0Fu : w[k] & 0x0F0F0F0Fu;
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const uint32_t v = __byte_perm(wk, 0x43434343u, e ? 0x4342 : 0x4140);
                __nv_bfloat162 bv = *reinterpret_cast<const __nv_bfloat162*>(&v);
                bv = __hfma2(__hsub2(bv, c128), sv, mv);
                o[2 * k + e] = *reinterpret_cast<uint32_t*>(&bv);
              }
            }
          }
          if (dmode != 1) tmem_st16(ta + 32 * c, o);
          if (c % C::kUA == C::kUA - 1) {           // unit complete: hand it to the MMA issuer
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->afull[ab]);
          }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->empty[s]);   // raw tile fully read
        if (dbg && threadIdx.x == 32 * C::kFirstDq && i < 64) dbg[160 + i] = clock64();
      }
      if (!ok) {
        set_error(a.err, kErrTimeout);
        bars->abort = 1;
      }
    } else if (FMT == kFmtQ4K) {
      int g = 0;
      bool ok = true;
      const __nv_bfloat162 c128 = __floats2bfloat162_rn(128.f, 128.f);
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % C::kStages;
        if (!mbar_wait(&bars->full[s], (i / C::kStages) & 1, a.err)) { ok = false; break; }
        const uint8_t* rb = stages + s * C::kStageBytes + t * kRawRowBytes;
        const uint32_t hdr = *reinterpret_cast<const uint32_t*>(rb);
        const float d = __half2float(__ushort_as_half((unsigned short)(hdr & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr >> 16)));
        __nv_bfloat162 sv[4], mv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          int sc, mn;
          q4k_scale_min(rb + 4, 2 * c + hf, sc, mn);
          sv[c] = __float2bfloat162_rn(d * (float)sc);
          mv[c] = __float2bfloat162_rn(-dmin * (float)mn);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c, ++g) {
          const int ab = g % NA;
          if (g >= NA && !mbar_wait(&bars->aempty[ab], ((g / NA) - 1) & 1, a.err)) { ok = false; break; }
          if (dbg && threadIdx.x == 64 && g < 64) dbg[96 + g] = clock64();
          uint32_t w[kWords];
#pragma unroll
          for (int u = 0; u < kWords / 4; ++u) {
            const uint4 qv = *reinterpret_cast<const uint4*>(rb + 16 + 32 * c + 16 * (sub + u));
            w[4 * u] = qv.x;
            w[4 * u + 1] = qv.y;
            w[4 * u + 2] = qv.z;
            w[4 * u + 3] = qv.w;
          }
#pragma unroll
          for (int k = 0; k < kWords; ++k) w[k] = hf ? (w[k] >> 4) & 0x0F0F0F0Fu : w[k] & 0x0F0F0F0Fu;
          uint8_t* arow = abuf + ab * kATile + t * 128;
#pragma unroll
          for (int c2 = 0; c2 < kWords / 2; ++c2) {
            const int cc = c2 + sub * (kWords / 2);
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t v = __byte_perm(w[2 * c2 + (e >> 1)], 0x43434343u, (e & 1) ? 0x4342 : 0x4140);
              __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&v);
              b = __hfma2(__hsub2(b, c128), sv[c], mv[c]);
              o[e] = *reinterpret_cast<uint32_t*>(&b);
            }
            *reinterpret_cast<uint4*>(arow + (((cc + 4 * hf) ^ (t & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
          fence_proxy_async_smem();  // generic-proxy stores -> visible to tcgen05 (async proxy)
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->afull[ab]);
          if (dbg && threadIdx.x == 64 && g < 64) dbg[160 + g] = clock64();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->empty[s]);
      }
      if (!ok) {
        set_error(a.err, kErrTimeout);
        bars->abort = 1;
      }
    }
    // ------------------------------------------------------------ epilogue
    pdl_wait();                                        // epilogue: scratch and output writes
    const bool done_ok = mbar_wait(&bars->done, 0, a.err);
    if (dbg && threadIdx.x == 32 * C::kFirstDq) dbg[224] = clock64();
    tc_fence_after();
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int m = 32 * q + lane;     // weight row within the tile
    const int jh = (warp - C::kFirstDq) >> 2;  // the DQ/4 warps of a quarter split the column groups
    constexpr int kJW = DQ / 4;
    const int mg = m0 + m;
    // warp-uniform: every tcgen05.ld below must be executed by all 32 lanes or none
    const bool valid = __all_sync(0xffffffffu, done_ok && !(*(volatile int*)&bars->abort) && nk > 0);
    if (!done_ok) set_error(a.err, kErrTimeout);
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    if (splits > 1) {
      float* part = a.ws + ((size_t)tile * splits + split) * NT * 128;
#pragma unroll 1
      for (int j = 0; j < NT / 16; ++j) {
        if ((j % kJW) != jh) continue;
        float v[16];
        if (valid) load_acc<C::kAccW, AT ? NACC : 1>(tmem + ((uint32_t)(32 * q) << 16) + 16 * j, v);
#pragma unroll
        for (int e = 0; e < 16; ++e) part[(16 * j + e) * 128 + m] = valid ? v[e] : 0.f;
      }
      __threadfence();
      named_sync_epi<DQ>();
      if (threadIdx.x == 32 * C::kFirstDq) {
        const int old = atomicAdd(&a.counters[tile], 1);
        bars->last = (old == splits - 1);
      }
      named_sync_epi<DQ>();
      if (!bars->last) goto finish;
      __threadfence();
      if (threadIdx.x == 32 * C::kFirstDq) a.counters[tile] = 0;  // self-cleaning for the next call
    }
    {  // all lanes stay in: tcgen05.ld is warp-collective; rows >= N are masked at the store
#pragma unroll 1
      for (int j = 0; j < NT / 16; ++j) {
        if ((j % kJW) != jh) continue;
        float v[16];
        if (splits > 1) {
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = 0.f;
          for (int sp = 0; sp < splits; ++sp) {
            const float* part = a.ws + ((size_t)tile * splits + sp) * NT * 128;
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] += __ldcg(part + (16 * j + e) * 128 + m);
          }
        } else if (valid) {
          load_acc<C::kAccW, AT ? NACC : 1>(tmem + ((uint32_t)(32 * q) << 16) + 16 * j, v);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = 0.f;
        }
        if (a.mode == kGemmPeerPush) {
          const int ep = *(volatile const int*)a.push.epoch;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int n = n0 + 16 * j + e;
            if (n < a.T && mg < a.N) peer_store(a.push, ep, n, mg, v[e]);
          }
          continue;
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int n = n0 + 16 * j + e;
          if (n < GROUP_TLIM && mg < a.N) {
            const size_t o = (size_t)(GROUP_ROWBASE + n) * a.ldo + mg;
            if (a.mode == kGemmStoreF32) static_cast<float*>(a.out)[o] = v[e];
            else if (a.mode == kGemmStoreBF16) static_cast<__nv_bfloat16*>(a.out)[o] = f2bf(v[e]);
            else static_cast<float*>(a.out)[o] += v[e];
          }
        }
      }
    }
  finish:;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}
#undef GROUP_ROWBASE
#undef GROUP_TLIM
#undef GROUP_WQ
#undef GROUP_TMW
#undef GROUP_TMS
#undef GROUP_WSCALES

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, uint64_t inner, uint64_t outer,
               uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swz) {
  auto fn = get_encode();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// AIR_PDL=0 turns programmatic dependent launch off (for the GEMVs too).
bool gemm_pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("AIR_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <int NT, int FMT, int NA, int DQ, bool AT = false, int NACC = 1, int CPS = 1>
const char* launch_na(const GemmArgs& a, const void* w, int64_t w_row_bytes, const void* x, int64_t ldx,
                      dim3 grid, cudaStream_t st) {
  using C = Cfg<NT, FMT, NA, AT, NACC, CPS>;
  CUtensorMap tw, tx, ts;
  thread_local GroupMaps gmaps;  // host staging of the per-group maps (copied into the launch)
  bool ok;
  GemmArgs b = a;
  b.wq = static_cast<const uint8_t*>(w);
  // the weight operand's tensor maps: Q8_0 int8 codes [N, K] in 128-byte-wide SW128 boxes plus
  // f16 scales [N, K/32] (8 per row per stage); FP8 codes like Q8_0's (multipliers are read by
  // the dequant warps); bf16 [N, K]; the tiled Q4_K operand is fetched with bulk copies
  auto encode_w = [&](const void* wp, const void* sp, CUtensorMap* m, CUtensorMap* ms) -> bool {
    memset(m, 0, sizeof(*m));
    memset(ms, 0, sizeof(*ms));
    if (FMT == kFmtQ4K) return true;
    if (FMT == kFmtQ8_0)
      return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, wp, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)w_row_bytes,
                       128, 128, CU_TENSOR_MAP_SWIZZLE_128B) &&
             sp != nullptr &&
             encode_2d(ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sp, (uint64_t)(a.K / 32), (uint64_t)a.N,
                       (uint64_t)(a.K / 32) * 2, 8, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (FMT == kFmtFP8)
      return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, wp, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)w_row_bytes,
                       128, 128, CU_TENSOR_MAP_SWIZZLE_128B) &&
             sp != nullptr;
    return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, wp, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)w_row_bytes,
                     64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  ok = encode_w(w, a.wscales, &tw, &ts);
  memset(&gmaps, 0, sizeof(gmaps));
  for (int g = 0; g < a.groups && ok; ++g) ok = encode_w(a.wq_g[g], a.wscales_g[g], &gmaps.w[g], &gmaps.s[g]);
  if (!ok) return "cuTensorMapEncodeTiled failed for the weight operand";
  if (!encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)a.K, (uint64_t)a.T,
                 (uint64_t)ldx * 2, 64, NT, CU_TENSOR_MAP_SWIZZLE_128B))
    return "cuTensorMapEncodeTiled failed for the activation operand";
  static unsigned long long attr_done = 0;
  if (!set_max_smem_per_device(gemm_q_kernel<NT, FMT, NA, DQ, AT, NACC, CPS>, C::kSmemLaunch, attr_done))
    return "cudaFuncSetAttribute(max dynamic smem) failed";
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3((AT ? 96 : 64) + 32 * DQ);
  cfg.dynamicSmemBytes = C::kSmemLaunch;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = gemm_pdl_enabled() ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, gemm_q_kernel<NT, FMT, NA, DQ, AT, NACC, CPS>, tw, tx, ts, gmaps, b) != cudaSuccess)
    return "gemm_q: launch failed";
  return nullptr;
}

// Q4_K variant: "tmem" (default) keeps the dequantised A operand in tensor memory;
// AIR_GEMM_A=smem selects the shared-memory A path; AIR_GEMM_DQ=16 doubles the dequant warps.
int a_path() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("AIR_GEMM_A");
    const char* q = getenv("AIR_GEMM_DQ");
    v = (e && strcmp(e, "smem") == 0) ? ((q && atoi(q) == 16) ? 2 : 1) : 0;
  }
  return v;
}

template <int NT, int FMT>
const char* launch_t(const GemmArgs& a, const void* w, int64_t w_row_bytes, const void* x, int64_t ldx,
                     dim3 grid, cudaStream_t st) {
  constexpr int NA = (FMT == kFmtQ4K && NT == 128) ? 2 : 4;
  if constexpr (FMT == kFmtQ4K && NT >= 256) {
    // 256-token tiles: A in TMEM only (one 256-column accumulator + two A stage buffers)
    // 16 dequantising warps (AIR_GEMM_PREFILL_DQ=8 for 8): 4-18 % faster on the Llama-3-8B
    // shapes at T = 512
    const char* e = getenv("AIR_GEMM_PREFILL_DQ");
    if (e && atoi(e) == 8) return launch_na<NT, FMT, NA, 8, true, 1>(a, w, w_row_bytes, x, ldx, grid, st);
    return launch_na<NT, FMT, NA, 16, true, 1>(a, w, w_row_bytes, x, ldx, grid, st);
  } else if constexpr (FMT == kFmtQ4K) {
    const int p = a_path();
    if (p == 0) {
      constexpr int NACC = NT <= 64 ? 4 : 2;
      const char* e = getenv("AIR_GEMM_DQ");
      const char* n = getenv("AIR_GEMM_NACC");
      if (n && atoi(n) == 1) return launch_na<NT, FMT, NA, 8, true, 1>(a, w, w_row_bytes, x, ldx, grid, st);
      if constexpr (NT <= 64) {
        // Decode token tiles: grids that fit in one wave of SMs (the split-K shapes: QKV, O,
        // down) run one CTA per SM with 16 dequantising warps; larger grids (gate|up, LM
        // head) run two CTAs per SM with 8 each. Measured on Llama-3-8B at T = 64: QKV 17.8 ->
        // 14.0 us, O 15.5 -> 12.7, down 31.3 -> 23.0; gate|up 33.6 vs 42.6 the other way.
        const char* c2 = getenv("AIR_GEMM_CPS");
        const long long ctas = (long long)grid.x * grid.y * grid.z;
        const int cps = c2 ? atoi(c2) : (ctas <= 148 ? 1 : 2);
        if (cps == 1 && !(e && atoi(e) == 8))
          return launch_na<NT, FMT, NA, 16, true, NACC>(a, w, w_row_bytes, x, ldx, grid, st);
        if (cps != 1 && e && atoi(e) == 16)   // two CTAs per SM with 16 dequant warps each (trial)
          return launch_na<NT, FMT, NA, 16, true, 1, 2>(a, w, w_row_bytes, x, ldx, grid, st);
        if (cps != 1) return launch_na<NT, FMT, NA, 8, true, 1, 2>(a, w, w_row_bytes, x, ldx, grid, st);
      }
      if (e && atoi(e) == 16) return launch_na<NT, FMT, NA, 16, true, NACC>(a, w, w_row_bytes, x, ldx, grid, st);
      return launch_na<NT, FMT, NA, 8, true, NACC>(a, w, w_row_bytes, x, ldx, grid, st);
    }
    if (p == 2) return launch_na<NT, FMT, NA, 16>(a, w, w_row_bytes, x, ldx, grid, st);
    return launch_na<NT, FMT, NA, 8>(a, w, w_row_bytes, x, ldx, grid, st);
  } else if constexpr (FMT == kFmtQ8_0 || FMT == kFmtFP8) {
    // Q8_0 / FP8: A (dequantised codes x block scale) in TMEM, as the default Q4_K path
    if constexpr (NT >= 256) {
      return launch_na<NT, FMT, 4, 8, true, 1>(a, w, w_row_bytes, x, ldx, grid, st);
    } else if constexpr (NT <= 64) {
      return launch_na<NT, FMT, 4, 8, true, 1, 2>(a, w, w_row_bytes, x, ldx, grid, st);
    } else {
      return launch_na<NT, FMT, 4, 8, true, 2>(a, w, w_row_bytes, x, ldx, grid, st);
    }
  } else {
    return launch_na<NT, FMT, NA, 8>(a, w, w_row_bytes, x, ldx, grid, st);
  }
}

}  // namespace

int gemm_q_token_tile(int T) {
  if (T <= 16) return 16;
  if (T <= 32) return 32;
  if (T <= 64) return 64;
  if (T <= 128) return 128;
  const char* e = getenv("AIR_GEMM_NT256");
  return (e && e[0] == '0') ? 128 : 256;
}

int gemm_q_splits(int N, int K, int T, int fmt) {
  const int nt = gemm_q_token_tile(T);
  const int tiles = ((N + 127) / 128) * ((T + nt - 1) / nt);
  const int ksteps = fmt == kFmtBF16 ? K / 64 : K / 256;
  // as many K splits as fit in ONE wave (a partial second wave costs a whole wave of time);
  // the decode variant runs two CTAs per SM, so its wave is 2 x 148 CTAs. More than one wave
  // of tiles already fills the machine.
  const char* w = getenv("AIR_GEMM_WAVE");
  const char* c2 = getenv("AIR_GEMM_CPS");
  const bool cps2 = fmt == kFmtQ4K && nt <= 64 && a_path() == 0 && !(c2 && atoi(c2) == 1);
  const int wave = w ? atoi(w) : 148;   // 2 x 148 for the two-CTA variant measured slower on split shapes
  (void)cps2;
  const char* mk = getenv("AIR_GEMM_MINK");
  const int mink = mk ? atoi(mk) : 2;                     // K-steps per split at least
  const int max_s = ksteps / mink > 0 ? ksteps / mink : 1;
  if (nt >= 128) {
    // one CTA per SM: time ~ waves x (tile math / s + partial traffic), in units of one
    // tile's math. A partial last wave costs a whole wave. Writing and re-reading a tile's
    // fp32 partial (2 x 128 x nt x 4 B at an SM's share of HBM, ~43 GB/s) against its math
    // (2 x 128 x nt x K FLOP at an SM's share of the tensor peak, ~9.5 TFLOP/s) is ~884 / K.
    int best = 1;
    double best_cost = 1e30;
    for (int s = 1; s <= max_s && s <= 16; ++s) {
      const double waves = (double)((s * tiles + wave - 1) / wave);
      const double cost = waves * (1.0 / s + (s > 1 ? 884.0 / K : 0.0));
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best = s;
      }
    }
    return best;
  }
  int s = wave / tiles;
  s = s < 1 ? 1 : s;
  return s > max_s ? max_s : s;
}

size_t gemm_q_workspace_floats(int N, int K, int T, int fmt, int splits) {
  const int nt = gemm_q_token_tile(T);
  const size_t tiles = (size_t)((N + 127) / 128) * ((T + nt - 1) / nt);
  return splits > 1 ? tiles * splits * nt * 128 : 0;
}

size_t gemm_q_counters(int N, int T) {
  const int nt = gemm_q_token_tile(T);
  return (size_t)((N + 127) / 128) * ((T + nt - 1) / nt);
}

// Pieces per raw weight tile copy (AIR_GEMM_WSPLIT: 1, 2, 4, 8, 9 or 18; default 1).
static int wsplit() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("AIR_GEMM_WSPLIT");
    v = e ? atoi(e) : 1;
    if (v != 2 && v != 4 && v != 8 && v != 9 && v != 18) v = 1;
  }
  return v;
}

const char* launch_gemm_q_tiles(int fmt, const void* w, int64_t w_row_bytes, const void* x, int64_t ldx,
                                const GemmArgs& a, int nt, dim3 grid, cudaStream_t st);

const char* launch_gemm_q(int fmt, const void* w, int64_t w_row_bytes, const void* x, int64_t ldx,
                          const GemmArgs& a_in, cudaStream_t st) {
  GemmArgs a = a_in;
  a.wsplit = wsplit();
  if (a.K % (fmt == kFmtBF16 ? 64 : 256)) return "gemm_q: K must be a multiple of 256 (Q4_K, Q8_0) or 64 (bf16)";
  if (fmt != kFmtQ4K && fmt != kFmtBF16 && fmt != kFmtQ8_0 && fmt != kFmtFP8)
    return "gemm_q: weight format not supported by the tensor-core path";
  if ((fmt == kFmtQ8_0 || fmt == kFmtFP8) && (a.wscales == nullptr || reinterpret_cast<uintptr_t>(a.wscales) % 16))
    return "gemm_q: Q8_0 / FP8 need 16-byte aligned block scales";
  if (reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(x) % 16 || w_row_bytes % 16 ||
      (ldx * 2) % 16)
    return "gemm_q: operands must be 16-byte aligned with 16-byte-multiple row strides";
  const int nt = gemm_q_token_tile(a.T);
  dim3 grid((a.N + 127) / 128, (a.T + nt - 1) / nt, a.splits);
  if (a.splits > 1 && (!a.ws || !a.counters)) return "gemm_q: split-K needs workspace and counters";
  a.groups = 0;
  return launch_gemm_q_tiles(fmt, w, w_row_bytes, x, ldx, a, nt, grid, st);
}

// Dispatch on format and token tile (checks done by the callers).
const char* launch_gemm_q_tiles(int fmt, const void* w, int64_t w_row_bytes, const void* x, int64_t ldx,
                                const GemmArgs& a, int nt, dim3 grid, cudaStream_t st) {
  if (fmt == kFmtQ4K) {
    switch (nt) {
      case 16: return launch_t<16, kFmtQ4K>(a, w, w_row_bytes, x, ldx, grid, st);
      case 32: return launch_t<32, kFmtQ4K>(a, w, w_row_bytes, x, ldx, grid, st);
      case 64: return launch_t<64, kFmtQ4K>(a, w, w_row_bytes, x, ldx, grid, st);
      case 128: return launch_t<128, kFmtQ4K>(a, w, w_row_bytes, x, ldx, grid, st);
      default: return launch_t<256, kFmtQ4K>(a, w, w_row_bytes, x, ldx, grid, st);
    }
  }
  if (fmt == kFmtFP8) {
    switch (nt) {
      case 16: return launch_t<16, kFmtFP8>(a, w, w_row_bytes, x, ldx, grid, st);
      case 32: return launch_t<32, kFmtFP8>(a, w, w_row_bytes, x, ldx, grid, st);
      case 64: return launch_t<64, kFmtFP8>(a, w, w_row_bytes, x, ldx, grid, st);
      case 128: return launch_t<128, kFmtFP8>(a, w, w_row_bytes, x, ldx, grid, st);
      default: return launch_t<256, kFmtFP8>(a, w, w_row_bytes, x, ldx, grid, st);
    }
  }
  if (fmt == kFmtQ8_0) {
    switch (nt) {
      case 16: return launch_t<16, kFmtQ8_0>(a, w, w_row_bytes, x, ldx, grid, st);
      case 32: return launch_t<32, kFmtQ8_0>(a, w, w_row_bytes, x, ldx, grid, st);
      case 64: return launch_t<64, kFmtQ8_0>(a, w, w_row_bytes, x, ldx, grid, st);
      case 128: return launch_t<128, kFmtQ8_0>(a, w, w_row_bytes, x, ldx, grid, st);
      default: return launch_t<256, kFmtQ8_0>(a, w, w_row_bytes, x, ldx, grid, st);
    }
  }
  switch (nt) {
    case 16: return launch_t<16, kFmtBF16>(a, w, w_row_bytes, x, ldx, grid, st);
    case 32: return launch_t<32, kFmtBF16>(a, w, w_row_bytes, x, ldx, grid, st);
    case 64: return launch_t<64, kFmtBF16>(a, w, w_row_bytes, x, ldx, grid, st);
    case 128: return launch_t<128, kFmtBF16>(a, w, w_row_bytes, x, ldx, grid, st);
    default: return launch_t<256, kFmtBF16>(a, w, w_row_bytes, x, ldx, grid, st);
  }
}

const char* launch_gemm_q_grouped(int fmt, const void* const* w, const void* const* scales, int G,
                                  int64_t w_row_bytes, const void* x, int64_t ldx, int rows, const GemmArgs& a_in,
                                  cudaStream_t st) {
  if (G < 1 || G > kGemmMaxGroups) return "gemm_q grouped: 1..8 groups";
  if (a_in.mode != kGemmStoreF32 && a_in.mode != kGemmStoreBF16) return "gemm_q grouped: store modes only";
  if (a_in.splits > 1) return "gemm_q grouped: no split-K";
  GemmArgs a = a_in;
  a.wsplit = wsplit();
  if (a.K % (fmt == kFmtBF16 ? 64 : 256)) return "gemm_q grouped: K must be a multiple of 256 (64 for bf16)";
  if (fmt != kFmtQ4K && fmt != kFmtBF16 && fmt != kFmtQ8_0 && fmt != kFmtFP8)
    return "gemm_q grouped: weight format not supported";
  if (reinterpret_cast<uintptr_t>(x) % 16 || w_row_bytes % 16 || (ldx * 2) % 16 || rows < 1)
    return "gemm_q grouped: operands must be 16-byte aligned with 16-byte-multiple row strides";
  for (int g = 0; g < G; ++g)
    if ((fmt == kFmtQ8_0 || fmt == kFmtFP8) &&
        (!scales || !scales[g] || reinterpret_cast<uintptr_t>(scales[g]) % 16))
      return "gemm_q grouped: Q8_0 / FP8 need 16-byte aligned block scales";
  a.groups = G;
  a.group_rows = rows;
  a.T = G * rows;
  const int nt = gemm_q_token_tile(rows);
  a.tiles_per_group = (rows + nt - 1) / nt;
  for (int g = 0; g < G; ++g) {
    a.wq_g[g] = static_cast<const uint8_t*>(w[g]);
    a.wscales_g[g] = scales ? scales[g] : nullptr;
    if (reinterpret_cast<uintptr_t>(w[g]) % 16) return "gemm_q grouped: 16-byte aligned weights";
  }
  // the token-tile size follows the per-group rows; the grid covers every group's tiles
  a.wscales = a.wscales_g[0];
  return launch_gemm_q_tiles(fmt, w[0], w_row_bytes, x, ldx, a, nt, dim3((a.N + 127) / 128, G * a.tiles_per_group, 1), st);
}

}  // namespace air
