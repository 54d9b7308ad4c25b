// torch <-> kernel adapter for the air_rs CUDA extension (module air_rs._C).
// Every launch goes to the current torch CUDA stream, so all ops are capturable in CUDA
// graphs; no op allocates device memory (callers own every buffer, including scratch).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "kernels.h"
#include "gemv_tiled.h"
#include "attention.h"
#include "sampler.h"
#include "misc.h"
#include "gemm_tc.h"
#include "comm.h"
#include "moe.h"

void register_gemm_tc(pybind11::module_& m);
void register_comm(pybind11::module_& m);
void register_gds(pybind11::module_& m);
void register_kv_push(pybind11::module_& m);
void register_ssm(pybind11::module_& m);
air::PeerPush peer_push_from_meta(const at::Tensor& meta);

using at::Tensor;
using c10::optional;

namespace {

template <typename T = void>
T* ptr(const optional<Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}
template <typename T = void>
T* ptr(const Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void post_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

void rmsnorm_quant(optional<Tensor> x, optional<Tensor> x_bf16, optional<Tensor> w, double w_offset,
                   double eps, int64_t B, int64_t K, optional<Tensor> q, optional<Tensor> ds,
                   optional<Tensor> y_bf16, optional<Tensor> bias, int64_t layer) {
  TORCH_CHECK(K % 32 == 0, "rmsnorm_quant: K must be a multiple of 32");
  air::launch_rmsnorm_quant(ptr<float>(x), ptr(x_bf16), ptr<float>(w), (float)w_offset, ptr<float>(bias),
                            (int)layer, (int)B,
                            (int)K, (float)eps, ptr<int8_t>(q), ptr<float2>(ds), ptr(y_bf16), stream());
  post_launch("rmsnorm_quant");
}

void gemv(int64_t fmt, Tensor data, optional<Tensor> scales, int64_t row_bytes, int64_t N, int64_t K,
          int64_t B, Tensor xq, Tensor xds, int64_t mode, optional<Tensor> out_f32,
          optional<Tensor> out_bf16, int64_t ld_out, optional<Tensor> resid,
          optional<Tensor> w2_data, optional<Tensor> w2_scales, optional<Tensor> rope_cs,
          optional<Tensor> positions, optional<Tensor> slots, optional<Tensor> kv,
          optional<Tensor> q_out, int64_t n_heads, int64_t n_kv, int64_t head_dim,
          int64_t block_size, int64_t rot_dim, optional<Tensor> err, int64_t splits,
          optional<Tensor> ws, optional<Tensor> counters, optional<Tensor> push_meta,
          optional<Tensor> out_q, optional<Tensor> out_ds, optional<Tensor> norm_w, double norm_offset,
          optional<Tensor> ss_out, optional<Tensor> ss_in, int64_t norm_k, double eps, int64_t act) {
  check_cuda(data, "gemv weight");
  TORCH_CHECK(B >= 1 && B <= 8, "gemv: batch must be in [1, 8]");
  TORCH_CHECK(K % 32 == 0, "gemv: K must be a multiple of 32");
  if (fmt == air::kFmtQ4K) TORCH_CHECK(K % 256 == 0 && row_bytes % 16 == 0, "gemv q4k: bad K");
  air::GemvWeight w{(int)fmt, data.data_ptr(), ptr(scales), row_bytes};
  air::GemvEpiParams ep{};
  ep.mode = (int)mode;
  ep.out_f32 = ptr<float>(out_f32);
  ep.out_bf16 = ptr(out_bf16);
  ep.ld_out = ld_out;
  ep.resid = ptr<float>(resid);
  ep.w2 = air::GemvWeight{(int)fmt, ptr(w2_data), ptr(w2_scales), row_bytes};
  ep.rope_cs = ptr<float2>(rope_cs);
  ep.positions = ptr<int>(positions);
  ep.slots = ptr<int64_t>(slots);
  ep.kv_cache = ptr(kv);
  ep.num_blocks = kv.has_value() ? kv->size(0) : 0;
  ep.q_out = ptr<float>(q_out);
  ep.n_heads = (int)n_heads;
  ep.n_kv = (int)n_kv;
  ep.head_dim = (int)head_dim;
  ep.block_size = (int)block_size;
  ep.rot_dim = (int)rot_dim;
  ep.err = ptr<int>(err);
  ep.act = (int)act;
  if (mode == air::kEpiSwiGLU) TORCH_CHECK(ep.w2.data, "gemv swiglu: w2 required");
  if (norm_w.has_value()) {
    TORCH_CHECK(mode == air::kEpiResidual && fmt == air::kFmtQ4K && out_q.has_value() && out_ds.has_value() &&
                    ss_out.has_value() && out_q->size(1) == N && norm_w->numel() >= N &&
                    ss_out->numel() >= B * (N / 32),
                "gemv: the fused RMSNorm producer is a residual epilogue of the tiled Q4_K path with "
                "out_q [B, N], out_ds and ss_out [B, N / 32]");
    ep.norm_w = ptr<float>(norm_w);
    ep.norm_offset = (float)norm_offset;
    ep.ss_out = ptr<float>(ss_out);
    ep.out_q = ptr<int8_t>(out_q);
    ep.out_ds = ptr<float2>(out_ds);
    ep.q_k = (int)N;
  }
  if (ss_in.has_value()) {
    TORCH_CHECK(fmt == air::kFmtQ4K && norm_k > 0 && norm_k % 32 == 0 && ss_in->numel() >= B * (norm_k / 32),
                "gemv: ss_in (fused RMSNorm partial sums [B, norm_k / 32]) needs the tiled Q4_K path");
    ep.ss_in = ptr<float>(ss_in);
    ep.norm_k = (int)norm_k;
    ep.eps = (float)eps;
  }
  if (out_q.has_value() && !norm_w.has_value()) {
    TORCH_CHECK(mode == air::kEpiSwiGLU && fmt == air::kFmtQ4K && out_ds.has_value(),
                "gemv: quantised output is a SwiGLU epilogue of the tiled Q4_K path");
    TORCH_CHECK(out_q->dim() == 2 && out_q->size(0) >= B && out_q->size(1) % 32 == 0 && out_q->size(1) >= N &&
                    out_q->size(1) <= (N + 127) / 128 * 128 && out_q->is_contiguous(),
                "gemv: out_q must be int8 [>=B, q_k], q_k % 32 == 0, N <= q_k <= N rounded up to 128");
    ep.out_q = ptr<int8_t>(out_q);
    ep.out_ds = ptr<float2>(out_ds);
    ep.q_k = (int)out_q->size(1);
  }
  if (mode == air::kEpiPeerPush) {
    TORCH_CHECK(push_meta.has_value() && fmt == air::kFmtQ4K, "gemv peer push: Q4_K tiled weights and push meta");
    ep.push = peer_push_from_meta(*push_meta);
    TORCH_CHECK(N == ep.push.row_len && B * ep.push.row_len <= ep.push.slot_elems,
                "gemv peer push: output [B, N] must fit the receive slot, N = its row length");
  }
  if (mode == air::kEpiResidual) TORCH_CHECK(ep.resid, "gemv residual: resid required");
  if (mode == air::kEpiQKVRope)
    TORCH_CHECK(ep.kv_cache && ep.q_out && ep.rope_cs && ep.positions && ep.slots,
                "gemv qkv: rope/kv/q buffers required");
  if (mode == air::kEpiQKVRope && kv)
    TORCH_CHECK(kv->scalar_type() == at::kBFloat16, "gemv qkv: the fused KV write needs a bf16 pool "
                "(fp8 pools take the rope_kv kernel)");
  if (fmt == air::kFmtQ4K) TORCH_CHECK(data.dim() == 4, "gemv q4k: expects the tiled device layout");
  // the tiled kernel handles every Q4_K case except the QKV epilogue of head_dim != 128
  if (fmt == air::kFmtQ4K && !(mode == air::kEpiQKVRope && head_dim != 128)) {
    TORCH_CHECK(data.dim() == 4, "gemv q4k: expects the tiled device layout [N/128, K/256, 128, 144]");
    TORCH_CHECK(ep.err, "gemv q4k: an error word is required (bounded waits report into it)");
    const int s = (int)std::max<int64_t>(1, splits);
    TORCH_CHECK(ws.has_value() && counters.has_value(), "gemv q4k: needs ws and counters");
    TORCH_CHECK((size_t)ws->numel() >= air::gemv_tiled_workspace_floats((int)N, s, (int)mode), "gemv: ws too small");
    TORCH_CHECK((size_t)counters->numel() >= air::gemv_tiled_counters((int)N), "gemv: counters too small");
    air::GemvTiledScratch sc{ptr<float>(ws), ptr<int>(counters)};
    const char* e = air::launch_gemv_tiled(w, (int)N, (int)K, (int)B, ptr<int8_t>(xq), ptr<float2>(xds), ep, sc,
                                           s, stream());
    TORCH_CHECK(e == nullptr, e ? e : "");
  } else {
    air::launch_gemv(w, (int)N, (int)K, (int)B, ptr<int8_t>(xq), ptr<float2>(xds), ep, stream());
  }
  post_launch("gemv");
}

void paged_attention(Tensor q, Tensor kv, Tensor block_tables, optional<Tensor> row_seq,
                     Tensor ctx_len, optional<Tensor> tree_base, optional<Tensor> tree_mask,
                     int64_t window, int64_t n_rows, int64_t n_heads, int64_t n_kv, int64_t head_dim,
                     int64_t block_size, int64_t n_splits, int64_t split_tokens, double scale,
                     optional<Tensor> part_o, optional<Tensor> part_ml, Tensor out,
                     optional<Tensor> out_q, optional<Tensor> out_ds, optional<Tensor> err,
                     optional<Tensor> out_bf16, double softcap) {
  check_cuda(q, "q");
  check_cuda(kv, "kv");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt, "block_tables must be int32");
  air::AttnArgs a{};
  a.q = ptr<float>(q);
  a.kv = kv.data_ptr();
  a.kv_fp8 = kv.scalar_type() == at::kByte ? 1 : 0;
  if (a.kv_fp8) {
    TORCH_CHECK(kv.size(-1) == head_dim + 16, "paged_attention: fp8 KV rows are head_dim + 16 bytes");
  } else {
    TORCH_CHECK(kv.scalar_type() == at::kBFloat16, "paged_attention: KV pool is bf16 or uint8 (fp8 rows)");
  }
  a.block_tables = ptr<int>(block_tables);
  a.max_blocks = (int)block_tables.size(1);
  a.rows = air::AttnRows{ptr<int>(row_seq), ptr<int>(ctx_len), ptr<int>(tree_base),
                         ptr<unsigned long long>(tree_mask), (int)window, (float)softcap};
  a.n_rows = (int)n_rows;
  a.n_heads = (int)n_heads;
  a.n_kv = (int)n_kv;
  a.head_dim = (int)head_dim;
  a.block_size = (int)block_size;
  a.num_blocks = kv.size(0);
  a.n_splits = (int)n_splits;
  a.split_tokens = (int)split_tokens;
  a.scale = (float)scale;
  a.part_o = ptr<float>(part_o);
  a.part_ml = ptr<float2>(part_ml);
  a.out = ptr<float>(out);
  a.out_q = ptr<int8_t>(out_q);
  a.out_ds = ptr<float2>(out_ds);
  a.out_bf16 = ptr(out_bf16);
  TORCH_CHECK(!a.out_bf16 || n_splits > 1, "paged_attention: out_bf16 needs the split merge (n_splits > 1)");
  a.err = ptr<int>(err);
  if (n_splits > 1) TORCH_CHECK(a.part_o && a.part_ml, "paged_attention: split scratch required");
  TORCH_CHECK(n_splits <= 256, "paged_attention: at most 256 splits");
  TORCH_CHECK(air::launch_paged_attention(a, stream()), "paged_attention: unsupported head_dim/GQA");
  post_launch("paged_attention");
}

void sampler(Tensor logits, int64_t B, int64_t V, optional<Tensor> counts, optional<Tensor> count_row,
             optional<Tensor> mask,
             optional<Tensor> temperature, optional<Tensor> penalty, optional<Tensor> top_k,
             optional<Tensor> top_p, int64_t seed, optional<Tensor> step, Tensor out_tokens,
             optional<Tensor> out_prob, optional<Tensor> part) {
  check_cuda(logits, "logits");
  air::SamplerArgs a{ptr<uint8_t>(counts), ptr<int>(count_row), ptr<uint32_t>(mask), ptr<float>(temperature),
                     ptr<float>(penalty), ptr<int>(top_k), ptr<float>(top_p),
                     (unsigned long long)seed, ptr<long long>(step), ptr<int>(out_tokens),
                     ptr<float>(out_prob)};
  if (part.has_value()) {
    TORCH_CHECK(part->dtype() == torch::kFloat32 && part->is_contiguous() &&
                    (size_t)part->numel() >= (size_t)B * air::sampler_chunks((int)V) * 4,
                "sampler: part scratch must be float32 [B * sampler_chunks(V) * 4]");
    a.part = reinterpret_cast<float4*>(part->data_ptr<float>());
  }
  air::launch_sampler(ptr<float>(logits), (int)B, (int)V, logits.stride(0), a, stream());
  post_launch("sampler");
}

// partial pass over a vocabulary shard: columns [v_off, v_off + V) of a V_total vocabulary
void sampler_partial(Tensor logits, int64_t B, int64_t V, int64_t nch, int64_t v_off, int64_t V_total,
                     optional<Tensor> counts, optional<Tensor> count_row, optional<Tensor> mask,
                     optional<Tensor> penalty, Tensor part) {
  check_cuda(logits, "logits");
  TORCH_CHECK(v_off % 32 == 0 && v_off + V <= V_total, "sampler_partial: shard [v_off, v_off+V) of V_total, v_off % 32 == 0");
  TORCH_CHECK(nch >= air::sampler_chunks((int)V) && nch > 0, "sampler_partial: nch < sampler_chunks(V)");
  TORCH_CHECK(part.dtype() == torch::kFloat32 && part.is_contiguous() && (size_t)part.numel() >= (size_t)B * nch * 4,
              "sampler_partial: part must be float32 [B * nch * 4]");
  air::SamplerArgs a{ptr<uint8_t>(counts), ptr<int>(count_row), ptr<uint32_t>(mask), nullptr,
                     ptr<float>(penalty), nullptr, nullptr, 0ull, nullptr, nullptr, nullptr};
  a.part = reinterpret_cast<float4*>(part.data_ptr<float>());
  a.v_off = (int)v_off;
  a.v_total = (int)V_total;
  air::launch_sampler_partial(ptr<float>(logits), (int)B, (int)V, (int)nch, logits.stride(0), a, stream());
  post_launch("sampler_partial");
}

void sampler_greedy_merge(Tensor part_all, int64_t W, int64_t B, int64_t nch, Tensor out_tokens,
                          optional<Tensor> out_prob, optional<Tensor> step) {
  check_cuda(part_all, "part_all");
  TORCH_CHECK(part_all.dtype() == torch::kFloat32 && part_all.is_contiguous() &&
                  (size_t)part_all.numel() >= (size_t)W * B * nch * 4,
              "sampler_greedy_merge: part_all must be float32 [W, B, nch, 4]");
  air::launch_sampler_greedy_merge(reinterpret_cast<const float4*>(part_all.data_ptr<float>()), (int)W, (int)B,
                                   (int)nch, ptr<int>(out_tokens), ptr<float>(out_prob), ptr<long long>(step),
                                   stream());
  post_launch("sampler_greedy_merge");
}

void count_tokens(Tensor counts, Tensor tokens, int64_t n, int64_t per_row,
                  optional<Tensor> count_row) {
  air::launch_count_tokens(ptr<uint8_t>(counts), (int)counts.size(1), ptr<int>(tokens), (int)n,
                           (int)per_row, ptr<int>(count_row), stream());
  post_launch("count_tokens");
}

void embed(int64_t fmt, Tensor table, optional<Tensor> scales, int64_t row_bytes, int64_t K,
           Tensor ids, int64_t n, int64_t vocab, optional<Tensor> out_f32, optional<Tensor> out_bf16,
           double mult, optional<Tensor> err) {
  air::launch_embed((int)fmt, table.data_ptr(), ptr(scales), row_bytes, (int)K, ptr<int>(ids), (int)n,
                    vocab, ptr<float>(out_f32), ptr(out_bf16), (float)mult, ptr<int>(err), stream());
  post_launch("embed");
}

void dequant(int64_t fmt, Tensor w, optional<Tensor> scales, int64_t row_bytes, int64_t N, int64_t K,
             Tensor out) {
  TORCH_CHECK(out.scalar_type() == at::kBFloat16, "dequant: out must be bf16");
  air::launch_dequant((int)fmt, w.data_ptr(), ptr(scales), row_bytes, (int)N, (int)K, out.data_ptr(),
                      stream());
  post_launch("dequant");
}

void rope_kv(Tensor qkv, int64_t T, Tensor rope_cs, Tensor positions, Tensor slots, Tensor kv,
             Tensor q_out, int64_t n_heads, int64_t n_kv, int64_t head_dim, int64_t block_size,
             int64_t rot_dim, optional<Tensor> err, optional<Tensor> bias) {
  air::RopeKvArgs a{ptr<float2>(rope_cs), ptr<int>(positions), ptr<int64_t>(slots), kv.data_ptr(),
                    ptr<float>(q_out), (int)n_heads, (int)n_kv, (int)head_dim, (int)block_size,
                    (int)rot_dim, kv.size(0), ptr<int>(err), ptr<float>(bias),
                    kv.scalar_type() == at::kByte ? 1 : 0};
  if (a.kv_fp8) {
    TORCH_CHECK(kv.size(-1) == head_dim + 16 && head_dim % 64 == 0 && head_dim <= 512,
                "rope_kv: fp8 KV rows are head_dim + 16 bytes, head_dim a multiple of 64 (<= 512)");
  }
  air::launch_rope_kv(qkv.data_ptr(), qkv.scalar_type() == at::kBFloat16, (int)T, a, stream());
  post_launch("rope_kv");
}

void swiglu(Tensor gu, int64_t T, int64_t F, int64_t up_off, int64_t ld_out, optional<Tensor> out_bf16,
            optional<Tensor> out_f32, int64_t act) {
  air::launch_swiglu(gu.data_ptr(), gu.scalar_type() == at::kBFloat16, (int)T, (int)F, gu.stride(0), up_off,
                     ld_out, ptr(out_bf16),
                     ptr<float>(out_f32), (int)act, stream());
  post_launch("swiglu");
}

void residual_add(Tensor resid, Tensor y, int64_t n) {
  air::launch_residual_add(ptr<float>(resid), y.data_ptr(), y.scalar_type() == at::kBFloat16, n, stream());
  post_launch("residual_add");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "air_rs sm_100a kernels";
  m.def("moe_route", [](Tensor x, int64_t T, Tensor router, int64_t k, bool normalize, Tensor cw,
                        optional<Tensor> ids, optional<Tensor> wts) {
    TORCH_CHECK(x.is_cuda() && router.is_cuda() && cw.is_cuda(), "moe_route: CUDA tensors");
    TORCH_CHECK(router.scalar_type() == torch::kFloat && router.dim() == 2, "moe_route: router fp32 [E, H]");
    const int E = (int)router.size(0), H = (int)router.size(1);
    TORCH_CHECK(E <= 256 && k >= 1 && k <= 8 && k <= E, "moe_route: E <= 256, 1 <= k <= 8");
    TORCH_CHECK(x.size(-1) >= H && x.stride(-1) == 1, "moe_route: x rows");
    TORCH_CHECK(cw.scalar_type() == torch::kFloat && cw.numel() >= T * E, "moe_route: cw [T, E] fp32");
    air::launch_moe_route(x.data_ptr(), x.scalar_type() == torch::kBFloat16, x.stride(0), (int)T, H,
                          router.data_ptr<float>(), E, (int)k, normalize, cw.data_ptr<float>(), ptr<int>(ids),
                          ptr<float>(wts), stream());
    post_launch("moe_route");
  });
  m.def("moe_combine", [](Tensor x, Tensor y, Tensor cw, int64_t e, int64_t E, int64_t T) {
    TORCH_CHECK(x.is_cuda() && y.is_cuda() && x.scalar_type() == torch::kFloat && y.scalar_type() == torch::kFloat,
                "moe_combine: fp32 CUDA");
    TORCH_CHECK(x.is_contiguous() && y.stride(-1) == 1, "moe_combine: layouts");
    air::launch_moe_combine(x.data_ptr<float>(), y.data_ptr<float>(), y.stride(0), cw.data_ptr<float>(), (int)e,
                            (int)E, (int)T, (int)x.size(1), stream());
    post_launch("moe_combine");
  });
  m.def("moe_select_grouped", [](Tensor cw, Tensor experts, int64_t T, Tensor idx, Tensor wts, Tensor count,
                                  Tensor pos) {
    const int G = (int)experts.numel();
    TORCH_CHECK(cw.is_cuda() && cw.scalar_type() == torch::kFloat && cw.dim() == 2, "moe_select_grouped: cw [T, E]");
    TORCH_CHECK(experts.is_cuda() && experts.scalar_type() == torch::kInt && idx.numel() >= G * T &&
                    wts.numel() >= G * T && count.numel() >= G && pos.numel() >= G * T,
                "moe_select_grouped: buffers of G * T rows");
    air::launch_moe_select_grouped(cw.data_ptr<float>(), experts.data_ptr<int>(), G, (int)cw.size(1), (int)T,
                                   idx.data_ptr<int>(), wts.data_ptr<float>(), count.data_ptr<int>(),
                                   pos.data_ptr<int>(), stream());
    post_launch("moe_select_grouped");
  });
  m.def("moe_gather_grouped", [](Tensor x, Tensor idx, Tensor count, int64_t G, int64_t T, Tensor xg) {
    const int64_t H = x.size(1);
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && xg.scalar_type() == at::kBFloat16 && H % 8 == 0 &&
                    x.stride(0) % 8 == 0 && xg.size(1) == H && xg.size(0) >= G * T && xg.is_contiguous(),
                "moe_gather_grouped: bf16 rows");
    air::launch_moe_gather_grouped(x.data_ptr(), x.stride(0), (int)H, idx.data_ptr<int>(), count.data_ptr<int>(),
                                   (int)G, (int)T, xg.data_ptr(), stream());
    post_launch("moe_gather_grouped");
  });
  m.def("moe_scatter_grouped", [](Tensor out, Tensor y, Tensor pos, Tensor wts, int64_t G, int64_t T) {
    TORCH_CHECK(out.scalar_type() == torch::kFloat && y.scalar_type() == torch::kFloat && out.is_contiguous() &&
                    y.size(0) >= G * T && y.stride(1) == 1, "moe_scatter_grouped: fp32 out / y");
    air::launch_moe_scatter_grouped(out.data_ptr<float>(), y.data_ptr<float>(), y.stride(0), (int)out.size(1),
                                    pos.data_ptr<int>(), wts.data_ptr<float>(), (int)G, (int)T, stream());
    post_launch("moe_scatter_grouped");
  });
  m.def("moe_select", [](Tensor cw, int64_t e, int64_t T, Tensor idx, Tensor wts, Tensor count) {
    TORCH_CHECK(cw.is_cuda() && cw.scalar_type() == torch::kFloat && cw.dim() == 2, "moe_select: cw [T, E] fp32");
    TORCH_CHECK(idx.numel() >= T && wts.numel() >= T && count.numel() >= 1, "moe_select: buffers");
    air::launch_moe_select(cw.data_ptr<float>(), (int)e, (int)cw.size(1), (int)T, idx.data_ptr<int>(),
                           wts.data_ptr<float>(), count.data_ptr<int>(), stream());
    post_launch("moe_select");
  });
  m.def("moe_gather", [](Tensor x, Tensor idx, Tensor count, int64_t cap, Tensor xg) {
    TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && xg.scalar_type() == torch::kBFloat16 && x.stride(1) == 1,
                "moe_gather: bf16 rows");
    const int H = (int)x.size(1);
    TORCH_CHECK(H % 8 == 0 && x.stride(0) % 8 == 0 && xg.size(1) == H && xg.size(0) >= cap, "moe_gather: shapes");
    air::launch_moe_gather(x.data_ptr(), x.stride(0), H, idx.data_ptr<int>(), count.data_ptr<int>(), (int)cap,
                           xg.data_ptr(), stream());
    post_launch("moe_gather");
  });
  m.def("moe_scatter", [](Tensor out, Tensor y, Tensor idx, Tensor wts, Tensor count, int64_t cap) {
    TORCH_CHECK(out.scalar_type() == torch::kFloat && y.scalar_type() == torch::kFloat && out.is_contiguous(),
                "moe_scatter: fp32");
    air::launch_moe_scatter(out.data_ptr<float>(), y.data_ptr<float>(), y.stride(0), (int)out.size(1),
                            idx.data_ptr<int>(), wts.data_ptr<float>(), count.data_ptr<int>(), (int)cap, stream());
    post_launch("moe_scatter");
  });
  m.def("rmsnorm_quant", &rmsnorm_quant);
  m.def("gemv", &gemv);
  m.def("gemv_tiled_splits", [](int64_t N, int64_t K, int64_t mode) { return air::gemv_tiled_splits((int)N, (int)K, (int)mode); });
  m.def("gemv_tiled_workspace", [](int64_t N, int64_t splits, int64_t mode) {
    return (int64_t)air::gemv_tiled_workspace_floats((int)N, (int)splits, (int)mode); });
  m.def("gemv_tiled_counters", [](int64_t N) { return (int64_t)air::gemv_tiled_counters((int)N); });
  m.def("paged_attention", &paged_attention);
  m.def("sampler", &sampler);
  m.def("sampler_partial", &sampler_partial);
  m.def("sampler_greedy_merge", &sampler_greedy_merge);
  m.def("sampler_chunks", [](int64_t V) { return (int64_t)air::sampler_chunks((int)V); });
  m.def("count_tokens", &count_tokens);
  m.def("embed", &embed);
  m.def("dequant", &dequant);
  m.def("rope_kv", &rope_kv);
  m.def("swiglu", &swiglu);
  m.def("residual_add", &residual_add);
  register_gemm_tc(m);
  register_kv_push(m);
  register_ssm(m);
  register_comm(m);
  register_gds(m);
}
