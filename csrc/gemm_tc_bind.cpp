#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include "gemm_tc.h"

using at::Tensor;
using c10::optional;

air::PeerPush peer_push_from_meta(const Tensor& meta);

namespace {

void gemm_q(int64_t fmt, Tensor w, optional<Tensor> scales, int64_t row_bytes, int64_t N, int64_t K,
            Tensor x, Tensor out, int64_t mode, int64_t splits, optional<Tensor> ws,
            optional<Tensor> counters, optional<Tensor> err, optional<Tensor> dbg,
            optional<Tensor> row_count, optional<Tensor> push_meta, optional<Tensor> rope_cs,
            optional<Tensor> positions, optional<Tensor> slots, optional<Tensor> kv, optional<Tensor> q_out,
            optional<Tensor> qkv_bias, int64_t n_heads, int64_t n_kv, int64_t block_size, int64_t rot_dim) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2, "gemm_q: x must be 2-D bf16 CUDA");
  TORCH_CHECK(x.stride(1) == 1 && out.stride(1) == 1, "gemm_q: rows must be contiguous");
  TORCH_CHECK(x.size(1) == K, "gemm_q: x has ", x.size(1), " columns, expected K=", K);
  if (mode == air::kGemmPeerPush) {
    TORCH_CHECK(push_meta.has_value(), "gemm_q peer push: push meta required");
  } else if (mode == air::kGemmQkvRope) {
    TORCH_CHECK(rope_cs.has_value() && positions.has_value() && slots.has_value() && kv.has_value() &&
                    q_out.has_value(), "gemm_q qkv rope: rope table, positions, slots, kv and q_out required");
    TORCH_CHECK(N == (n_heads + 2 * n_kv) * 128 && rot_dim > 0 && rot_dim <= 128 && rot_dim % 2 == 0,
                "gemm_q qkv rope: N must be (n_heads + 2 n_kv) x 128 (head_dim 128)");
    TORCH_CHECK(kv->scalar_type() == at::kBFloat16 && kv->is_contiguous() && q_out->is_contiguous() &&
                    q_out->scalar_type() == at::kFloat && positions->numel() >= x.size(0) &&
                    slots->numel() >= x.size(0) && slots->scalar_type() == at::kLong,
                "gemm_q qkv rope: bf16 contiguous kv, fp32 q_out, int64 slots covering the rows");
    TORCH_CHECK(!qkv_bias.has_value() || qkv_bias->numel() >= N, "gemm_q qkv rope: bias too short");
  } else if (mode == air::kGemmStoreBF16) {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "gemm_q: out must be bf16");
  } else {
    TORCH_CHECK(out.scalar_type() == at::kFloat, "gemm_q: out must be f32");
  }
  air::GemmArgs a{};
  a.N = (int)N;
  a.K = (int)K;
  a.T = (int)x.size(0);
  a.mode = (int)mode;
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.splits = (int)std::max<int64_t>(1, splits);
  if (a.splits > 1) {
    TORCH_CHECK(ws.has_value() && counters.has_value(), "gemm_q: split-K needs ws and counters");
    TORCH_CHECK((size_t)ws->numel() >= air::gemm_q_workspace_floats(a.N, a.K, a.T, (int)fmt, a.splits),
                "gemm_q: workspace too small");
    TORCH_CHECK((size_t)counters->numel() >= air::gemm_q_counters(a.N, a.T), "gemm_q: counters too small");
    a.ws = ws->data_ptr<float>();
    a.counters = counters->data_ptr<int>();
  }
  TORCH_CHECK(err.has_value(), "gemm_q: an error word is required (bounded waits report into it)");
  a.err = err->data_ptr<int>();
  a.dbg = dbg.has_value() ? (long long*)dbg->data_ptr<int64_t>() : nullptr;
  a.row_count = row_count.has_value() ? row_count->data_ptr<int>() : nullptr;
  a.wscales = (scales.has_value() && scales->defined()) ? scales->data_ptr() : nullptr;
  if (mode == air::kGemmQkvRope) {
    a.rope.cs = static_cast<const float2*>(rope_cs->data_ptr());
    a.rope.positions = positions->data_ptr<int>();
    a.rope.slots = slots->data_ptr<int64_t>();
    a.rope.kv = kv->data_ptr();
    a.rope.q_out = q_out->data_ptr<float>();
    a.rope.bias = qkv_bias.has_value() ? qkv_bias->data_ptr<float>() : nullptr;
    a.rope.n_heads = (int)n_heads;
    a.rope.n_kv = (int)n_kv;
    a.rope.block_size = (int)block_size;
    a.rope.rot_dim = (int)rot_dim;
    a.rope.num_blocks = kv->size(0);
  }
  if (mode == air::kGemmPeerPush) {
    a.push = peer_push_from_meta(*push_meta);
    TORCH_CHECK(a.N == a.push.row_len && (int64_t)a.T * a.push.row_len <= a.push.slot_elems,
                "gemm_q peer push: output [T, N] must fit the receive slot with N = its row length");
  }
  const char* e = air::launch_gemm_q((int)fmt, w.data_ptr(), row_bytes, x.data_ptr(), x.stride(0), a,
                                     at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == nullptr, e ? e : "");
  cudaError_t ce = cudaGetLastError();
  TORCH_CHECK(ce == cudaSuccess, "gemm_q launch: ", cudaGetErrorString(ce));
}

}  // namespace

void register_gemm_tc(pybind11::module_& m) {
  m.def("gemm_q", &gemm_q);
  m.def("gemm_q_splits", [](int64_t N, int64_t K, int64_t T, int64_t fmt) {
    return air::gemm_q_splits((int)N, (int)K, (int)T, (int)fmt);
  });
  m.def("gemm_q_workspace", [](int64_t N, int64_t K, int64_t T, int64_t fmt, int64_t splits) {
    return (int64_t)air::gemm_q_workspace_floats((int)N, (int)K, (int)T, (int)fmt, (int)splits);
  });
  m.def("gemm_q_counters", [](int64_t N, int64_t T) { return (int64_t)air::gemm_q_counters((int)N, (int)T); });
}
