// Query-tiled paged attention for prefill (head_dim 128): FlashAttention-2 style.
//
// The decode kernel (attention_mma.cu) gives every query row its own CTA, so a T-token
// prompt streams each key T times. Here a CTA owns one KV head and a tile of 16 consecutive
// query rows; its G warps (one per query head of the GQA group) share every 64-key K/V tile
// loaded into shared memory (cp.async, double buffered, XOR-swizzled for ldmatrix), so each
// key is read once per 16 queries. Per warp and key tile: S = Q K^T as 8 x 8 m16n8k16 bf16
// MMAs (16 query rows x 64 keys), causal / window masking per row, online softmax in
// registers, and O += P V with the S accumulators reused as the P operand (16 x 128 fp32
// accumulators per warp).
//
// Rows of a tile that belong to different sequences (a prompt boundary inside the tile) are
// handled as consecutive groups: the CTA runs the key loop once per group against that
// group's block table with the other rows masked. Speculative-tree rows keep the per-row
// kernel. Reference: flash-attention prefill in src/ops.rs:458-508 (GQA at :514-568).
//
// F8 (fp8 KV pool, kv_f8.cuh): the cp.async ring holds raw 144-byte rows; after each tile
// lands the CTA converts it to one f16 K|V tile pair (exact), runs the MMAs in f16 and applies
// the per-key K scale to the scores and the V scale to the softmax weights.
#include "common.cuh"
#include "attention.h"
#include "kv_f8.cuh"

namespace air {

namespace {

constexpr int kD = 128;
constexpr int kRow = kD * 2;            // bytes per K/V row
constexpr int kQT = 16;                 // query rows per CTA
constexpr int kKT = 64;                 // keys per tile
constexpr int kTileBytes = kKT * kRow;  // 16 KB (K or V)
constexpr int kF8Row = kv_f8_row_bytes(kD);   // 144 B
constexpr int kF8Tile = kKT * kF8Row;          // 9 KB raw fp8 K or V tile
// bf16: 2 stages x (K, V); F8: one f16 (K, V) pair + 2 raw stages x (K, V)
template <bool F8>
__host__ __device__ constexpr int smem_bytes() { return F8 ? 2 * kTileBytes + 4 * kF8Tile : 4 * kTileBytes; }

AIR_DEVICE uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
AIR_DEVICE uint32_t swz(uint32_t base, int t, int c) { return base + t * kRow + ((c ^ (t & 7)) << 4); }

AIR_DEVICE void cp16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
AIR_DEVICE void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
AIR_DEVICE void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
AIR_DEVICE void ldsm4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
AIR_DEVICE void ldsm4t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
AIR_DEVICE void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
AIR_DEVICE void mma_h(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <bool F8>
AIR_DEVICE void mmak(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (F8) mma_h(c, a, b0, b1);
  else mma(c, a, b0, b1);
}
template <bool F8>
AIR_DEVICE uint32_t pk(float lo, float hi) {
  if constexpr (F8) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

template <int G, bool F8>
__global__ void __launch_bounds__(G * 32, G == 4 ? 3 : 1)
prefill_attn_kernel(const float* __restrict__ q, const uint8_t* __restrict__ kv,
                    const int* __restrict__ block_tables, int max_blocks, AttnRows rows, int R, int n_heads,
                    int n_kv, int block_size, int64_t num_blocks, float scale, float* __restrict__ out,
                    __nv_bfloat16* __restrict__ out_bf16, int* err) {
  extern __shared__ __align__(128) uint8_t smem[];   // [2 stages][K | V] tiles
  __shared__ int s_seq[kQT], s_ctx[kQT];
  const int h = blockIdx.x, r0 = blockIdx.y * kQT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = h * G + warp;
  if (threadIdx.x < kQT) {
    const int r = r0 + threadIdx.x;
    s_seq[threadIdx.x] = r < R ? (rows.row_seq ? rows.row_seq[r] : r) : -1;
    s_ctx[threadIdx.x] = r < R ? rows.ctx_len[r] : 0;
  }
  __syncthreads();

  // this thread's two query rows (MMA rows lane/4 and lane/4 + 8)
  const int qr[2] = {lane >> 2, (lane >> 2) + 8};
  // ---- Q fragments of this warp's head, pre-scaled ----
  uint32_t qa[8][4];
  {
    const int cpair = (lane & 3) * 2;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
      for (int half = 0; half < 2; ++half)
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
          const int r = r0 + qr[half];
          float x0 = 0.f, x1 = 0.f;
          if (r < R) {
            const float* qp = q + ((size_t)r * n_heads + head) * kD + kk * 16 + cpair + 8 * kh;
            x0 = qp[0] * scale;
            x1 = qp[1] * scale;
          }
          qa[kk][half + 2 * kh] = pk<F8>(x0, x1);
        }
  }
  constexpr int kRowB = F8 ? kF8Row : kRow;
  constexpr int kChunks = kRowB / 16;
  const size_t head_stride = (size_t)block_size * kRowB;
  const size_t kv_stride = (size_t)n_kv * head_stride;
  const size_t blk_stride = 2 * kv_stride;
  const uint32_t sbase = saddr(smem);

  int done_mask = 0;     // rows already written by an earlier group
  for (int grp = 0; grp < kQT; ++grp) {
    // leader of the next group: the first row not handled yet (uniform across the CTA)
    int lead = -1;
    for (int i = 0; i < kQT; ++i)
      if (!((done_mask >> i) & 1) && s_seq[i] >= 0) { lead = i; break; }
    if (lead < 0) break;
    const int seq = s_seq[lead];
    int gmask = 0, kmax = 0, kmin_ctx = 1 << 30;
    for (int i = 0; i < kQT; ++i)
      if (s_seq[i] == seq) {
        gmask |= 1 << i;
        kmax = max(kmax, s_ctx[i]);
        kmin_ctx = min(kmin_ctx, s_ctx[i]);
      }
    done_mask |= gmask;
    const int t_lo = rows.window > 0 ? max(0, (kmin_ctx - rows.window) / kKT * kKT) : 0;
    const int* bt = block_tables + (size_t)seq * max_blocks;
    bool in_g[2];
    int ctx[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      in_g[i] = (gmask >> qr[i]) & 1;
      ctx[i] = s_ctx[qr[i]];
    }

    auto load_tile = [&](int t0, int stage) {
      const uint32_t kb = F8 ? sbase + 2 * kTileBytes + stage * 2 * kF8Tile : sbase + stage * 2 * kTileBytes;
      const uint32_t vb = kb + (F8 ? kF8Tile : kTileBytes);
      for (int idx = threadIdx.x; idx < kKT * kChunks; idx += G * 32) {
        const int key = idx / kChunks, c = idx % kChunks;
        const int t = t0 + key;
        bool ok = t < kmax;
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
        cp16(F8 ? kb + key * kF8Row + c * 16 : swz(kb, key, c), src, ok);
        cp16(F8 ? vb + key * kF8Row + c * 16 : swz(vb, key, c), ok ? src + kv_stride : kv, ok);
      }
      cp_commit();
    };

    float o[16][4];
#pragma unroll
    for (int nd = 0; nd < 16; ++nd)
#pragma unroll
      for (int j = 0; j < 4; ++j) o[nd][j] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

    int stage = 0;
    load_tile(t_lo, 0);
    for (int t0 = t_lo; t0 < kmax; t0 += kKT, stage ^= 1) {
      const bool more = t0 + kKT < kmax;
      if (more) load_tile(t0 + kKT, stage ^ 1);
      if (more) cp_wait<1>(); else cp_wait<0>();
      __syncthreads();
      const uint32_t kb = F8 ? sbase : sbase + stage * 2 * kTileBytes, vb = kb + kTileBytes;
      const uint8_t* raw = smem + 2 * kTileBytes + stage * 2 * kF8Tile;   // F8 only
      if constexpr (F8) {
        for (int u = threadIdx.x; u < 2 * kKT * 8; u += G * 32) {   // (K|V) x 64 keys x 8 chunks
          const int kvi = u / (kKT * 8), key = (u / 8) % kKT, cc = u % 8;
          const uint4 c = *reinterpret_cast<const uint4*>(raw + kvi * kF8Tile + key * kF8Row + cc * 16);
          uint4 lo, hi;
          e4m3x16_to_h16(c, lo, hi);
          const uint32_t tb = kvi ? vb : kb;
          *reinterpret_cast<uint4*>(smem + (swz(tb, key, 2 * cc) - sbase)) = lo;
          *reinterpret_cast<uint4*>(smem + (swz(tb, key, 2 * cc + 1) - sbase)) = hi;
        }
        __syncthreads();
      }
      // ---- S = Q K^T: 16 rows x 64 keys ----
      float s[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk += 2) {
          const int mi = lane >> 3;
          const int key = nt * 8 + (lane & 7);
          const int c = 2 * (kk + (mi >> 1)) + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldsm4(swz(kb, key, c), b0, b1, b2, b3);
          mmak<F8>(s[nt], qa[kk], b0, b1);
          mmak<F8>(s[nt], qa[kk + 1], b2, b3);
        }
      }
      // ---- mask + online softmax (rows qr[0], qr[1]) ----
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = j >> 1;
          const int t = t0 + nt * 8 + (lane & 3) * 2 + (j & 1);
          const bool vis = in_g[i] && t < ctx[i] && !(rows.window > 0 && t < ctx[i] - rows.window);
          if constexpr (F8)
            s[nt][j] *= *reinterpret_cast<const float*>(raw + (nt * 8 + (lane & 3) * 2 + (j & 1)) * kF8Row + kD);
          s[nt][j] = vis ? soft_cap(s[nt][j], rows.softcap) : -INFINITY;
          mx[i] = fmaxf(mx[i], s[nt][j]);
        }
      float alpha[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
        const float mnew = fmaxf(m_run[i], mx[i]);
        alpha[i] = (mnew == -INFINITY) ? 1.f : __expf(m_run[i] - mnew);
        m_run[i] = mnew;
      }
      float psum[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = j >> 1;
          const float p = (s[nt][j] == -INFINITY) ? 0.f : __expf(s[nt][j] - m_run[i]);
          s[nt][j] = p;
          psum[i] += p;
        }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        psum[i] += __shfl_xor_sync(0xffffffffu, psum[i], 1);
        psum[i] += __shfl_xor_sync(0xffffffffu, psum[i], 2);
        l_run[i] = l_run[i] * alpha[i] + psum[i];
      }
#pragma unroll
      for (int nd = 0; nd < 16; ++nd) {
        o[nd][0] *= alpha[0];
        o[nd][1] *= alpha[0];
        o[nd][2] *= alpha[1];
        o[nd][3] *= alpha[1];
      }
      // ---- O += P V: four 16-key steps, 16 n8 tiles over the 128 dims ----
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        uint32_t pa[4];
        if constexpr (F8) {
          float vs[2][2];     // V scales of keys kt*16 + {0, 8} + (lane&3)*2 + {0, 1}
#pragma unroll
          for (int x = 0; x < 2; ++x)
#pragma unroll
            for (int y = 0; y < 2; ++y)
              vs[x][y] = *reinterpret_cast<const float*>(
                  raw + kF8Tile + ((2 * kt + x) * 8 + (lane & 3) * 2 + y) * kF8Row + kD);
          pa[0] = pk<F8>(s[2 * kt][0] * vs[0][0], s[2 * kt][1] * vs[0][1]);
          pa[1] = pk<F8>(s[2 * kt][2] * vs[0][0], s[2 * kt][3] * vs[0][1]);
          pa[2] = pk<F8>(s[2 * kt + 1][0] * vs[1][0], s[2 * kt + 1][1] * vs[1][1]);
          pa[3] = pk<F8>(s[2 * kt + 1][2] * vs[1][0], s[2 * kt + 1][3] * vs[1][1]);
        } else {
          pa[0] = pk<F8>(s[2 * kt][0], s[2 * kt][1]);
          pa[1] = pk<F8>(s[2 * kt][2], s[2 * kt][3]);
          pa[2] = pk<F8>(s[2 * kt + 1][0], s[2 * kt + 1][1]);
          pa[3] = pk<F8>(s[2 * kt + 1][2], s[2 * kt + 1][3]);
        }
#pragma unroll
        for (int nd = 0; nd < 16; nd += 2) {
          const int mi = lane >> 3;
          const int key = kt * 16 + (mi & 1) * 8 + (lane & 7);
          const int c = nd + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm4t(swz(vb, key, c), b0, b1, b2, b3);
          mmak<F8>(o[nd], pa, b0, b1);
          mmak<F8>(o[nd + 1], pa, b2, b3);
        }
      }
      __syncthreads();      // every warp is done with this stage before it is refilled
    }
    cp_wait<0>();
    // ---- write this group's rows ----
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = r0 + qr[i];
      if (!in_g[i] || r >= R) continue;
      const float inv = l_run[i] > 0.f ? 1.f / l_run[i] : 0.f;
      float* orow = out + ((size_t)r * n_heads + head) * kD;
#pragma unroll
      for (int nd = 0; nd < 16; ++nd) {
        const int d = nd * 8 + (lane & 3) * 2;
        const float v0 = o[nd][2 * i] * inv, v1 = o[nd][2 * i + 1] * inv;
        *reinterpret_cast<float2*>(orow + d) = make_float2(v0, v1);
        if (out_bf16) {
          __nv_bfloat16* ob = out_bf16 + ((size_t)r * n_heads + head) * kD + d;
          *reinterpret_cast<__nv_bfloat162*>(ob) = __floats2bfloat162_rn(v0, v1);
        }
      }
    }
    __syncthreads();
  }
}

template <int G, bool F8>
void launch_gf(const AttnArgs& a, cudaStream_t st) {
  constexpr int smem = smem_bytes<F8>();    // 64 KB (bf16) / 68 KB (F8)
  static unsigned long long attr_done = 0;
  set_max_smem_per_device(prefill_attn_kernel<G, F8>, smem, attr_done);
  dim3 grid(a.n_kv, (a.n_rows + kQT - 1) / kQT);
  prefill_attn_kernel<G, F8><<<grid, G * 32, smem, st>>>(
      a.q, (const uint8_t*)a.kv, a.block_tables, a.max_blocks, a.rows, a.n_rows, a.n_heads, a.n_kv,
      a.block_size, a.num_blocks, a.scale, a.out, (__nv_bfloat16*)a.out_bf16, a.err);
}

template <int G>
void launch_g(const AttnArgs& a, cudaStream_t st) {
  if (a.kv_fp8) launch_gf<G, true>(a, st);
  else launch_gf<G, false>(a, st);
}

}  // namespace

bool launch_prefill_attention(const AttnArgs& a, cudaStream_t st) {
  if (a.head_dim != kD || a.rows.tree_base != nullptr || a.n_splits != 1 || a.out_q != nullptr) return false;
  switch (a.n_heads / a.n_kv) {
    case 1: launch_g<1>(a, st); return true;
    case 2: launch_g<2>(a, st); return true;
    case 4: launch_g<4>(a, st); return true;
    case 8: launch_g<8>(a, st); return true;
    default: return false;
  }
}

}  // namespace air
