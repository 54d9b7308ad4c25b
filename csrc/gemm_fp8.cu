// W8A8 FP8 GEMM on the 5th-generation tensor cores (sm_100a), for block-scaled FP8 weights:
//     out[t, n] (op)= sx[t] * sum_kb  sw[n, kb] * sum_{k in block kb} qw[n, k] * qx[t, k]
// qw: E4M3 weight codes [N, K] with one f32 multiplier sw per row and 128-wide K block (the
// framework's internal FP8 block format); qx: E4M3 activation codes [T, K] with one f32 scale
// sx per token (dynamic per-token quantisation: quant_fp8_rows_kernel below).
//
// The codes go straight from HBM into shared memory by TMA and into `tcgen05.mma
// kind::f8f6f4` with no dequantisation pass. Because the weight multiplier changes every 128 K,
// each K block is accumulated on its own in one of two TMEM buffers, and the epilogue warps
// promote it into f32 registers (one FMA per element with the row's multiplier) while the
// tensor core already fills the other buffer (the per-block promotion of block-scaled FP8
// recipes). Per CTA (swap-AB: the MMA's M = 128 weight rows, N = NT tokens):
//   warp 0        TMA producer: W box 128 rows x 128 B + X box NT rows x 128 B per K block
//   warp 1        TMEM owner + single-thread MMA issuer (4 x K32 per block, commit per block)
//   warps 2..     PW promotion warps (row = TMEM lane, a group of the NT columns each), then
//                 the epilogue (per-token scale, store / residual add)
// Wide decode grids (more CTAs than SMs) run two CTAs per SM. Split-K: fp32 partials in a
// caller-provided workspace; the last CTA of a tile (per-tile arrival counter, self-resetting)
// reduces them. Every wait is bounded (error word, no trap).
//
// Replaces the reference's FP8 / W8A8 matmuls (src/fp8.rs:28-310, src/w8a8.rs:40-160), which
// dequantise on the CPU / in candle before a bf16 or f32 GEMM.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp8.h>
#include <string.h>
#include "common.cuh"
#include "sm100.cuh"
#include "gemm_tc.h"
#include "gemm_fp8.h"

namespace air {

namespace {

using namespace sm100;

constexpr int kF8WTile = 128 * 128;     // 128 weight rows x 128 codes

// NT tokens per tile, PW promotion / epilogue warps, CPS CTAs per SM.
template <int NT, int PW, int CPS>
struct F8Cfg {
  static constexpr int kXTile = NT * 128;
  static constexpr int kStage = kF8WTile + kXTile;
  static constexpr int kBudget = (CPS == 2 ? 113 * 1024 : 227 * 1024) - 2048;
  static constexpr int kStages = (kBudget / kStage) > 8 ? 8 : (kBudget / kStage);
  static constexpr int kSmem = 1024 + kStages * kStage + 1024;
  static constexpr int kTmemCols = 2 * NT < 32 ? 32 : 2 * NT;   // two block accumulators
  static constexpr int kParts = PW / 4;                         // column groups per TMEM lane quarter
  static constexpr int kCols = NT / kParts;                     // columns per promotion thread
  static constexpr int kThreads = 64 + 32 * PW;
  static_assert(kStages >= 2, "two stages at least");
  static_assert(kCols % 16 == 0, "16-column TMEM loads");
};

struct F8Bars {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t accfull[2];
  uint64_t accempty[2];
  uint32_t tmem;
  int abort;
  int last;
};

// 32 lanes x 32 columns of 32-bit in one load (one wait)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <int NT, int PW, int CPS>
__global__ void __launch_bounds__(64 + 32 * PW, CPS)
gemm_fp8_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                const __grid_constant__ GemmF8Args a) {
  using C = F8Cfg<NT, PW, CPS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  F8Bars* bars = reinterpret_cast<F8Bars*>(smem + C::kStages * C::kStage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * 128, n0 = blockIdx.y * NT;
  const int split = blockIdx.z, splits = gridDim.z;
  const int kblocks = a.K / 128;
  const int kper = (kblocks + splits - 1) / splits;
  const int kb0 = split * kper;
  const int nk = max(0, min(kblocks, kb0 + kper) - kb0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->accfull[b], 1);
      mbar_init(&bars->accempty[b], PW);
    }
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
  }
  if (warp == 1) tmem_alloc(&bars->tmem, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  // the activations (codes and scales) come from the previous kernel
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::kStages;
        if (i >= C::kStages && !mbar_wait(&bars->empty[s], ((i / C::kStages) - 1) & 1, a.err)) {
          set_error(a.err, kErrTimeout);
          bars->abort = 1;
          break;
        }
        if (*(volatile int*)&bars->abort) break;
        uint8_t* st = smem + s * C::kStage;
        mbar_expect_tx(&bars->full[s], C::kStage);
        tma_load_2d(st, &tm_w, &bars->full[s], (kb0 + i) * 128, m0);
        tma_load_2d(st + kF8WTile, &tm_x, &bars->full[s], (kb0 + i) * 128, n0);
        issued = i + 1;
      }
      // never leave the CTA with copies in flight into its shared memory
      for (int i = max(0, issued - C::kStages); i < issued; ++i)
        mbar_wait(&bars->full[i % C::kStages], (i / C::kStages) & 1, a.err, 50ull * 1000 * 1000);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, NT);
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % C::kStages, b = i & 1;
        if (!mbar_wait(&bars->full[s], (i / C::kStages) & 1, a.err)) { ok = false; break; }
        if (i >= 2 && !mbar_wait(&bars->accempty[b], ((i >> 1) - 1) & 1, a.err)) { ok = false; break; }
        tc_fence_after();
        uint8_t* st = smem + s * C::kStage;
        const uint64_t ad = sw128_desc(st), bd = sw128_desc(st + kF8WTile);
#pragma unroll
        for (int k = 0; k < 4; ++k)   // 4 x K32 per block: +32 B along K in both operands
          mma_f8(tmem + NT * b, ad + 2 * k, bd + 2 * k, idesc, k ? 1u : 0u);
        mma_commit(&bars->empty[s]);
        mma_commit(&bars->accfull[b]);
      }
      if (!ok) {
        set_error(a.err, kErrTimeout);
        bars->abort = 1;
      }
    }
  } else {
    // ------------------------------------------------------------ promotion + epilogue
    // Thread = (weight row m = TMEM lane, column group). Per K block: acc += block partial x the
    // row's weight multiplier for that block; the per-token activation scale is the same for
    // every block and is applied once at the end.
    const int q = warp & 3;                       // TMEM lane quarter this warp may access
    const int part = (warp - 2) >> 2;             // which column group
    const int m = 32 * q + lane;                  // weight row within the tile
    const int mg = m0 + m;
    const int c0 = part * C::kCols;               // first column of this thread
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16) + c0;
    const float* wsrow = a.wscale + (size_t)min(mg, a.N - 1) * kblocks;
    float acc[C::kCols];
#pragma unroll
    for (int j = 0; j < C::kCols; ++j) acc[j] = 0.f;
    bool ok = true;
    float sw_next = nk > 0 ? __ldg(wsrow + kb0) : 0.f;
    for (int i = 0; i < nk; ++i) {
      const int b = i & 1;
      const float sw = sw_next;
      if (i + 1 < nk) sw_next = __ldg(wsrow + kb0 + i + 1);
      if (!mbar_wait(&bars->accfull[b], (i >> 1) & 1, a.err)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < C::kCols / 32; ++c) {
        float v[32];
        tmem_ld32(trow + NT * b + 32 * c, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[32 * c + e] = fmaf(v[e], sw, acc[32 * c + e]);
      }
      if constexpr (C::kCols % 32) {
        float v[16];
        tmem_ld16(trow + NT * b + C::kCols - 16, v);
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[C::kCols - 16 + e] = fmaf(v[e], sw, acc[C::kCols - 16 + e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->accempty[b]);
    }
    if (!ok) {
      set_error(a.err, kErrTimeout);
      bars->abort = 1;
    }
    const bool valid = __all_sync(0xffffffffu, ok && !(*(volatile int*)&bars->abort));
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    bool store = true;
    if (splits > 1) {
      float* pp = a.ws + ((size_t)tile * splits + split) * NT * 128;
#pragma unroll
      for (int j = 0; j < C::kCols; ++j) pp[(c0 + j) * 128 + m] = valid ? acc[j] : 0.f;
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(32 * PW) : "memory");
      if (threadIdx.x == 64) {
        const int old = atomicAdd(&a.counters[tile], 1);
        bars->last = (old == splits - 1);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * PW) : "memory");
      store = bars->last != 0;
      if (store) {
        __threadfence();
        if (threadIdx.x == 64) a.counters[tile] = 0;   // self-cleaning for the next call
#pragma unroll
        for (int j = 0; j < C::kCols; ++j) acc[j] = 0.f;
        for (int sp = 0; sp < splits; ++sp) {
          const float* p = a.ws + ((size_t)tile * splits + sp) * NT * 128;
#pragma unroll
          for (int j = 0; j < C::kCols; ++j) acc[j] += __ldcg(p + (c0 + j) * 128 + m);
        }
      }
    }
    if (store && mg < a.N) {
#pragma unroll
      for (int j = 0; j < C::kCols; ++j) {
        const int n = n0 + c0 + j;
        if (n < a.T) {
          const float v = acc[j] * __ldg(a.xscale + n);
          const size_t o = (size_t)n * a.ldo + mg;
          if (a.mode == kGemmStoreF32) static_cast<float*>(a.out)[o] = v;
          else if (a.mode == kGemmStoreBF16) static_cast<__nv_bfloat16*>(a.out)[o] = f2bf(v);
          else static_cast<float*>(a.out)[o] += v;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// One 256-thread CTA per token row: row amax -> scale = amax / 448 (one per token), codes =
// x / scale in E4M3 (saturating). Two passes over the row (the second from L1/L2).
__global__ void __launch_bounds__(256) quant_fp8_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                             int K, uint8_t* __restrict__ xq, float* __restrict__ xs) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const __nv_bfloat16* row = x + (size_t)t * ldx;
  float amax = 0.f;
  for (int k = 8 * threadIdx.x; k < K; k += 8 * 256) {
    float f[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + k), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
  }
  amax = block_max(amax, red);
  const float inv = amax > 0.f ? 448.f / amax : 0.f;
  for (int k = 8 * threadIdx.x; k < K; k += 8 * 256) {
    float f[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(row + k), f);
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_fp8x2_storage_t lo =
          __nv_cvt_float2_to_fp8x2(make_float2(f[4 * h] * inv, f[4 * h + 1] * inv), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi =
          __nv_cvt_float2_to_fp8x2(make_float2(f[4 * h + 2] * inv, f[4 * h + 3] * inv), __NV_SATFINITE, __NV_E4M3);
      w[h] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint2*>(xq + (size_t)t * K + k) = make_uint2(w[0], w[1]);
  }
  if (threadIdx.x == 0) xs[t] = amax / 448.f;
}

PFN_cuTensorMapEncodeTiled_v12000 f8_encode_fn() {
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

// [rows, cols] bytes (row stride `stride` bytes) in 128-byte-wide SW128 boxes of box_rows rows
bool f8_map(CUtensorMap* m, const void* p, uint64_t cols, uint64_t rows, uint64_t stride, uint32_t box_rows) {
  auto fn = f8_encode_fn();
  if (!fn) return false;
  memset(m, 0, sizeof(*m));
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(p), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, int PW, int CPS>
const char* launch_nt(const GemmF8Args& a, dim3 grid, cudaStream_t st) {
  using C = F8Cfg<NT, PW, CPS>;
  CUtensorMap tw, tx;
  if (!f8_map(&tw, a.wq, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.w_row_bytes, 128))
    return "gemm_fp8: cuTensorMapEncodeTiled failed for the weights";
  if (!f8_map(&tx, a.xq, (uint64_t)a.K, (uint64_t)a.T, (uint64_t)a.K, NT))
    return "gemm_fp8: cuTensorMapEncodeTiled failed for the activations";
  static unsigned long long attr_done = 0;
  if (!set_max_smem_per_device(gemm_fp8_kernel<NT, PW, CPS>, C::kSmem, attr_done))
    return "gemm_fp8: cudaFuncSetAttribute(max dynamic smem) failed";
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, gemm_fp8_kernel<NT, PW, CPS>, tw, tx, a) != cudaSuccess) return "gemm_fp8: launch failed";
  return nullptr;
}

}  // namespace

int gemm_fp8_token_tile(int T) { return T <= 32 ? 32 : (T <= 64 ? 64 : (T <= 128 ? 128 : 256)); }

int gemm_fp8_splits(int N, int K, int T) {
  const int nt = gemm_fp8_token_tile(T);
  const int tiles = ((N + 127) / 128) * ((T + nt - 1) / nt);
  const int kblocks = K / 128;
  int s = 148 / tiles;
  const int max_s = kblocks / 4 > 0 ? kblocks / 4 : 1;   // four K blocks per split at least
  s = s < 1 ? 1 : (s > max_s ? max_s : s);
  // no empty split: the last one must own at least one block
  const int kper = (kblocks + s - 1) / s;
  return (kblocks + kper - 1) / kper;
}

size_t gemm_fp8_workspace_floats(int N, int T, int splits) {
  const int nt = gemm_fp8_token_tile(T);
  const size_t tiles = (size_t)((N + 127) / 128) * ((T + nt - 1) / nt);
  return splits > 1 ? tiles * splits * nt * 128 : 0;
}

size_t gemm_fp8_counters(int N, int T) {
  const int nt = gemm_fp8_token_tile(T);
  return (size_t)((N + 127) / 128) * ((T + nt - 1) / nt);
}

const char* launch_quant_fp8_rows(const void* x, int64_t ldx, int T, int K, void* xq, float* xs, cudaStream_t st) {
  if (K % 128 || T < 1) return "quant_fp8_rows: K must be a multiple of 128";
  if (reinterpret_cast<uintptr_t>(x) % 16 || ldx % 8 || reinterpret_cast<uintptr_t>(xq) % 16)
    return "quant_fp8_rows: misaligned operands";
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)T);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, quant_fp8_rows_kernel, static_cast<const __nv_bfloat16*>(x), ldx, K,
                         static_cast<uint8_t*>(xq), xs) != cudaSuccess)
    return "quant_fp8_rows: launch failed";
  return nullptr;
}

const char* launch_gemm_fp8(const GemmF8Args& a, cudaStream_t st) {
  if (a.K % 128 || a.N < 1 || a.T < 1) return "gemm_fp8: K must be a multiple of 128";
  if (!a.wq || !a.xq || !a.wscale || !a.xscale || !a.out || !a.err) return "gemm_fp8: null operand";
  if (reinterpret_cast<uintptr_t>(a.wq) % 16 || reinterpret_cast<uintptr_t>(a.xq) % 16 || a.w_row_bytes % 16)
    return "gemm_fp8: codes must be 16-byte aligned with 16-byte-multiple row strides";
  if (a.mode != kGemmStoreF32 && a.mode != kGemmStoreBF16 && a.mode != kGemmResidualF32)
    return "gemm_fp8: store / residual modes only";
  const int nt = gemm_fp8_token_tile(a.T);
  const int kblocks = a.K / 128;
  if (a.splits < 1 || a.splits > kblocks) return "gemm_fp8: bad split count";
  const int kper = (kblocks + a.splits - 1) / a.splits;
  if ((a.splits - 1) * kper >= kblocks) return "gemm_fp8: a split would own no K block";
  if (a.splits > 1 && (!a.ws || !a.counters)) return "gemm_fp8: split-K needs workspace and counters";
  dim3 grid((a.N + 127) / 128, (a.T + nt - 1) / nt, a.splits);
  // grids of more than one wave of single CTAs (wide decode projections) run two CTAs per SM
  const long long ctas = (long long)grid.x * grid.y * grid.z;
  switch (nt) {
    case 32: return ctas > 148 ? launch_nt<32, 8, 2>(a, grid, st) : launch_nt<32, 8, 1>(a, grid, st);
    case 64: return ctas > 148 ? launch_nt<64, 8, 2>(a, grid, st) : launch_nt<64, 8, 1>(a, grid, st);
    case 128: return launch_nt<128, 16, 1>(a, grid, st);
    default: return launch_nt<256, 16, 1>(a, grid, st);
  }
}

}  // namespace air
