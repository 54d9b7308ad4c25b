// Paged attention, tensor-core variant (head_dim 128, GQA group <= 8).
//
// Same contract as paged_attn_kernel (attention.cu): CTA = (KV head, query row, split),
// four warps, online softmax, partial (max, sum, o) per split merged by attn_merge_kernel.
// The G query heads of the group are the 16-row A operand of m16n8k16 bf16 MMAs (rows >= G
// are zero), so both S = Q K^T and O += P V run on the tensor pipe and the per-key work
// is a handful of instructions. Each warp streams its own 16-key chunks of K and V with
// cp.async into an XOR-swizzled shared buffer (double buffered) and feeds the MMAs with
// ldmatrix (.trans for V). The S accumulators are reused directly as the P operand
// (FlashAttention-2 register layout).
//
// F8 (fp8 KV pool, kv_f8.cuh): the cp.async ring holds the raw 144-byte rows (codes + scale);
// before its MMAs a warp converts its chunk to f16 (exact for E4M3) in one swizzled K|V tile
// pair, runs the same MMAs in f16, multiplies each key's score by its K scale and each key's
// softmax weight by its V scale.
#include "common.cuh"
#include "attention.h"
#include "kv_f8.cuh"

namespace air {

namespace {

constexpr int kD = 128;
constexpr int kRow = kD * 2;           // bytes per K/V row
constexpr int kKeys = 16;              // keys per warp chunk
constexpr int kWarpsM = 4;
constexpr int kTile = kKeys * kRow;    // 4 KB: one K or V chunk
constexpr int kF8Row = kv_f8_row_bytes(kD);     // 144 B fp8 row
constexpr int kF8Tile = kKeys * kF8Row;          // 2304 B: one raw fp8 K or V chunk
// shared bytes per warp: 2 stages x (K, V) bf16 tiles, or one f16 tile pair + 2 raw fp8 stages
template <bool F8>
__host__ __device__ constexpr int warp_bytes() { return F8 ? 2 * kTile + 4 * kF8Tile : 4 * kTile; }

AIR_DEVICE uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 16-byte chunk c of key row t lives at t*256 + ((c ^ (t & 7)) * 16): conflict-free ldmatrix.
AIR_DEVICE uint32_t swz(uint32_t base, int t, int c) { return base + t * kRow + ((c ^ (t & 7)) << 4); }

AIR_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0 source bytes -> zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
AIR_DEVICE void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
AIR_DEVICE void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

AIR_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
AIR_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
AIR_DEVICE void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
AIR_DEVICE void mma16816_h(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
AIR_DEVICE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
AIR_DEVICE uint32_t pack_h16(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <bool F8>
AIR_DEVICE void mma_kv(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (F8) mma16816_h(c, a, b0, b1);
  else mma16816(c, a, b0, b1);
}
template <bool F8>
AIR_DEVICE uint32_t pack_kv(float lo, float hi) {
  if constexpr (F8) return pack_h16(lo, hi);
  else return pack_bf16(lo, hi);
}

AIR_DEVICE bool visible(int t, const AttnRows& rows, int r, int ctx) {
  if (t >= ctx) return false;
  if (rows.window > 0 && t < ctx - rows.window) return false;
  if (rows.tree_base) {
    const int tb = rows.tree_base[r];
    if (t >= tb) {
      const int k = t - tb;
      if (k >= 64) return false;
      return (rows.tree_mask[r] >> k) & 1ull;
    }
  }
  return true;
}

// merge buffer [warps][16][128] f32 (32 KB), aliased onto the tile ring after the key loop
constexpr int kMergeBytes = kWarpsM * 16 * kD * 4;
template <bool F8>
__host__ __device__ constexpr int smem_total() {
  return kWarpsM * warp_bytes<F8>() > kMergeBytes ? kWarpsM * warp_bytes<F8>() : kMergeBytes;
}

// three CTAs (12 warps) per SM: 64 KB (bf16) / 68 KB (F8) of shared memory each
template <int G, bool F8>
__global__ void __launch_bounds__(kWarpsM * 32, 3)
paged_attn_mma_kernel(const float* __restrict__ q, const uint8_t* __restrict__ kv,
                      const int* __restrict__ block_tables, int max_blocks, AttnRows rows, int n_heads,
                      int n_kv, int block_size, int64_t num_blocks, int n_splits, int split_tokens,
                      float scale, float* __restrict__ part_o, float2* __restrict__ part_ml,
                      float* __restrict__ out, int* err) {
  static_assert(G >= 1 && G <= 8, "GQA group (rows 8..15 of the MMA are padding)");
  extern __shared__ __align__(128) uint8_t smem[];
  // per warp: 2 stages x (K tile + V tile)
  __shared__ float red_m[kWarpsM][16], red_l[kWarpsM][16];
  float* red_o = reinterpret_cast<float*>(smem);  // [warps][16][128], over the tiles once the loop is done

  const int h = blockIdx.x, r = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = rows.row_seq ? rows.row_seq[r] : r;
  const int ctx = rows.ctx_len[r];
  // at least 64 keys per split: shorter splits cost more in fixed work and merge than they save
  const int st = split_tokens > 0 ? split_tokens
                                  : max(64, ((ctx + n_splits - 1) / n_splits + kKeys - 1) / kKeys * kKeys);
  int t_begin = split * st;
  const int t_end = min(ctx, t_begin + st);
  if (rows.window > 0) t_begin = max(t_begin, ((ctx - rows.window) / kKeys) * kKeys);

  // ---- Q fragments (rows = heads of the group, zero-padded to 16) ----
  uint32_t qa[8][4];
  {
    const int r0 = lane >> 2, cpair = (lane & 3) * 2;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {       // rows r0 / r0 + 8
        const int hrow = r0 + 8 * half;
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {           // cols +0 / +8
          float x0 = 0.f, x1 = 0.f;
          if (hrow < G) {
            const float* qp = q + ((size_t)r * n_heads + h * G + hrow) * kD + kk * 16 + cpair + 8 * kh;
            x0 = qp[0] * scale;
            x1 = qp[1] * scale;
          }
          qa[kk][half + 2 * kh] = pack_kv<F8>(x0, x1);
        }
      }
    }
  }

  const int* bt = block_tables + (size_t)seq * max_blocks;
  constexpr int kRowB = F8 ? kF8Row : kRow;
  constexpr int kChunks = kRowB / 16;                 // 16-byte chunks per row: 16 or 9
  const size_t head_stride = (size_t)block_size * kRowB;
  const size_t kv_stride = (size_t)n_kv * head_stride;
  const size_t blk_stride = 2 * kv_stride;
  const uint32_t wbase = smem_addr(smem) + warp * warp_bytes<F8>();  // bf16: [stage][K|V]
  uint8_t* const wgen = smem + warp * warp_bytes<F8>();
  // F8: raw rows of stage sidx at wbase + 2 kTile + sidx * 2 kF8Tile (K, then V)

  // issue the cp.async loads of one 16-key chunk starting at key t0 into stage sidx
  auto load_chunk = [&](int t0, int sidx) {
    const uint32_t kb = F8 ? wbase + 2 * kTile + sidx * 2 * kF8Tile : wbase + sidx * 2 * kTile;
    const uint32_t vb = kb + (F8 ? kF8Tile : kTile);
#pragma unroll
    for (int it = 0; it < (kKeys * kChunks + 31) / 32; ++it) {
      const int idx = it * 32 + lane;
      if (kKeys * kChunks % 32 != 0 && idx >= kKeys * kChunks) continue;
      const int key = idx / kChunks, c = idx % kChunks;
      const int t = t0 + key;
      bool ok = t < t_end;
      const uint8_t* src = kv;
      if (ok) {
        const int b = bt[t / block_size];
        if (b < 0 || b >= num_blocks) {
          set_error(err, kErrBounds);
          ok = false;
        } else {
          src = kv + (size_t)b * blk_stride + h * head_stride + (size_t)(t % block_size) * kRowB + c * 16;
        }
      }
      const uint32_t dk = F8 ? kb + key * kF8Row + c * 16 : swz(kb, key, c);
      const uint32_t dv = F8 ? vb + key * kF8Row + c * 16 : swz(vb, key, c);
      cp_async16(dk, src, ok);
      cp_async16(dv, ok ? src + kv_stride : kv, ok);
    }
    cp_commit();
  };

  float o[16][4];
#pragma unroll
  for (int nd = 0; nd < 16; ++nd)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[nd][j] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;   // for head row lane/4

  const int stride = kWarpsM * kKeys;
  int t0 = t_begin + warp * kKeys;
  int sidx = 0;
  if (t0 < t_end) load_chunk(t0, 0);
  for (; t0 < t_end; t0 += stride, sidx ^= 1) {
    const bool more = t0 + stride < t_end;
    if (more) load_chunk(t0 + stride, sidx ^ 1);
    if (more) cp_wait<1>(); else cp_wait<0>();
    __syncwarp();
    const uint32_t kb = F8 ? wbase : wbase + sidx * 2 * kTile, vb = kb + kTile;
    float ksc[2][2], vsc[2][2];   // F8: scales of this lane's keys (lane&3)*2 + {0,1} (+8)
    if constexpr (F8) {
      const uint8_t* raw = wgen + 2 * kTile + sidx * 2 * kF8Tile;
#pragma unroll
      for (int it = 0; it < 4; ++it) {              // 16 keys x 8 code chunks, K and V
        const int u = it * 32 + lane, key = u >> 3, cc = u & 7;
#pragma unroll
        for (int kvi = 0; kvi < 2; ++kvi) {
          const uint4 c = *reinterpret_cast<const uint4*>(raw + kvi * kF8Tile + key * kF8Row + cc * 16);
          uint4 lo, hi;
          e4m3x16_to_h16(c, lo, hi);
          const uint32_t tb = kvi ? vb : kb;
          *reinterpret_cast<uint4*>(wgen + (swz(tb, key, 2 * cc) - wbase)) = lo;
          *reinterpret_cast<uint4*>(wgen + (swz(tb, key, 2 * cc + 1) - wbase)) = hi;
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int key = nt * 8 + (lane & 3) * 2 + j;
          ksc[nt][j] = *reinterpret_cast<const float*>(raw + key * kF8Row + kD);
          vsc[nt][j] = *reinterpret_cast<const float*>(raw + kF8Tile + key * kF8Row + kD);
        }
      __syncwarp();
    }
    // ---- S = Q K^T for 16 keys: two n8 tiles ----
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {
        const int mi = lane >> 3;
        const int key = nt * 8 + (lane & 7);
        const int c = 2 * (kk + (mi >> 1)) + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(swz(kb, key, c), b0, b1, b2, b3);
        mma_kv<F8>(s[nt], qa[kk], b0, b1);
        mma_kv<F8>(s[nt], qa[kk + 1], b2, b3);
      }
    }
    // ---- mask + online softmax for head row lane/4 (keys (lane&3)*2 + {0,1} (+8)) ----
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int t = t0 + nt * 8 + (lane & 3) * 2 + j;
        if constexpr (F8) s[nt][j] *= ksc[nt][j];
        if (!visible(t, rows, r, ctx) || t >= t_end) s[nt][j] = -INFINITY;
        else s[nt][j] = soft_cap(s[nt][j], rows.softcap);
        mx = fmaxf(mx, s[nt][j]);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mnew = fmaxf(m_run, mx);
    const float alpha = (mnew == -INFINITY) ? 1.f : __expf(m_run - mnew);
    float p[2][2], psum = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        p[nt][j] = (s[nt][j] == -INFINITY) ? 0.f : __expf(s[nt][j] - mnew);
        psum += p[nt][j];
      }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    l_run = l_run * alpha + psum;
    m_run = mnew;
#pragma unroll
    for (int nd = 0; nd < 16; ++nd) {
      o[nd][0] *= alpha;
      o[nd][1] *= alpha;
    }
    // P as the A operand: rows 8..15 (padding heads) are zero
    uint32_t pa[4];
    if constexpr (F8) {
      pa[0] = pack_h16(p[0][0] * vsc[0][0], p[0][1] * vsc[0][1]);
      pa[2] = pack_h16(p[1][0] * vsc[1][0], p[1][1] * vsc[1][1]);
    } else {
      pa[0] = pack_bf16(p[0][0], p[0][1]);
      pa[2] = pack_bf16(p[1][0], p[1][1]);
    }
    pa[1] = 0u;
    pa[3] = 0u;
    // ---- O += P V: 16 n8 tiles over the 128 dims ----
#pragma unroll
    for (int nd = 0; nd < 16; nd += 2) {
      const int mi = lane >> 3;
      const int key = (mi & 1) * 8 + (lane & 7);
      const int c = nd + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(swz(vb, key, c), b0, b1, b2, b3);
      mma_kv<F8>(o[nd], pa, b0, b1);
      mma_kv<F8>(o[nd + 1], pa, b2, b3);
    }
    __syncwarp();
  }
  cp_wait<0>();
  __syncthreads();     // every warp is done with its tiles before red_o overwrites them

  // ---- merge the 4 warps (head rows < G) ----
  const int hr = lane >> 2;
  if ((lane & 3) == 0 && hr < 16) {
    red_m[warp][hr] = m_run;
    red_l[warp][hr] = l_run;
  }
#pragma unroll
  for (int nd = 0; nd < 16; ++nd) {
    const int d0 = nd * 8 + (lane & 3) * 2;
    red_o[(warp * 16 + hr) * kD + d0] = o[nd][0];
    red_o[(warp * 16 + hr) * kD + d0 + 1] = o[nd][1];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const int g = i / kD, d = i % kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarpsM; ++w) M = fmaxf(M, red_m[w][g]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsM; ++w) {
      const float f = (red_m[w][g] == -INFINITY) ? 0.f : __expf(red_m[w][g] - M);
      L += red_l[w][g] * f;
      O += red_o[(w * 16 + g) * kD + d] * f;
    }
    const int head = h * G + g;
    if (n_splits == 1) {
      out[((size_t)r * n_heads + head) * kD + d] = L > 0.f ? O / L : 0.f;
    } else {
      const size_t pi = ((size_t)r * n_heads + head) * n_splits + split;
      part_o[pi * kD + d] = O;
      if (d == 0) part_ml[pi] = make_float2(M, L);
    }
  }
}

template <int G, bool F8>
void launch_gf(const AttnArgs& a, cudaStream_t st) {
  // bf16: 64 KB tiles; F8: 68 KB tiles (the merge buffer reuses them)
  const int smem = smem_total<F8>();
  static unsigned long long attr_done = 0;
  set_max_smem_per_device(paged_attn_mma_kernel<G, F8>, smem, attr_done);
  dim3 grid(a.n_kv, a.n_rows, a.n_splits);
  paged_attn_mma_kernel<G, F8><<<grid, kWarpsM * 32, smem, st>>>(
      a.q, (const uint8_t*)a.kv, a.block_tables, a.max_blocks, a.rows, a.n_heads, a.n_kv,
      a.block_size, a.num_blocks, a.n_splits, a.split_tokens, a.scale, a.part_o, a.part_ml, a.out, a.err);
}

template <int G>
void launch_g(const AttnArgs& a, cudaStream_t st) {
  if (a.kv_fp8) launch_gf<G, true>(a, st);
  else launch_gf<G, false>(a, st);
}

}  // namespace

bool launch_paged_attention_mma(const AttnArgs& a, cudaStream_t st) {
  if (a.head_dim != kD) return false;
  switch (a.n_heads / a.n_kv) {
    case 1: launch_g<1>(a, st); return true;
    case 2: launch_g<2>(a, st); return true;
    case 4: launch_g<4>(a, st); return true;
    case 8: launch_g<8>(a, st); return true;
    default: return false;
  }
}

}  // namespace air
