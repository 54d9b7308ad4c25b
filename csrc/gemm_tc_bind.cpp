#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <vector>
#include <torch/csrc/utils/pybind.h>
#include "gemm_tc.h"

using at::Tensor;
using c10::optional;

air::PeerPush peer_push_from_meta(const Tensor& meta);

namespace {

void gemm_q(int64_t fmt, Tensor w, optional<Tensor> scales, int64_t row_bytes, int64_t N, int64_t K,
            Tensor x, Tensor out, int64_t mode, int64_t splits, optional<Tensor> ws,
            optional<Tensor> counters, optional<Tensor> err, optional<Tensor> dbg,
            optional<Tensor> row_count, optional<Tensor> push_meta) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2, "gemm_q: x must be 2-D bf16 CUDA");
  TORCH_CHECK(x.stride(1) == 1 && out.stride(1) == 1, "gemm_q: rows must be contiguous");
  TORCH_CHECK(x.size(1) == K, "gemm_q: x has ", x.size(1), " columns, expected K=", K);
  if (mode == air::kGemmPeerPush) {
    TORCH_CHECK(push_meta.has_value(), "gemm_q peer push: push meta required");
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

// Grouped GEMM over G <= 8 weights of one shape (routed experts): x [G * rows, K] bf16,
// out [G * rows, N] (f32 or bf16), row_counts [G] int32 on the device.
void gemm_q_grouped(int64_t fmt, std::vector<Tensor> ws, std::vector<optional<Tensor>> scales, int64_t row_bytes,
                    int64_t N, int64_t K, Tensor x, int64_t rows, Tensor out, Tensor row_counts, Tensor err) {
  const int G = (int)ws.size();
  TORCH_CHECK(G >= 1 && G <= air::kGemmMaxGroups, "gemm_q_grouped: 1..8 weights");
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.size(0) >= G * rows &&
                  x.size(1) == K && x.stride(1) == 1, "gemm_q_grouped: x must be bf16 [G * rows, K]");
  TORCH_CHECK(out.size(0) >= G * rows && out.size(1) >= N && out.stride(1) == 1, "gemm_q_grouped: out [G * rows, N]");
  TORCH_CHECK(row_counts.is_cuda() && row_counts.scalar_type() == at::kInt && row_counts.numel() >= G,
              "gemm_q_grouped: int32 row counts per group");
  const void* wp[air::kGemmMaxGroups] = {};
  const void* sp[air::kGemmMaxGroups] = {};
  for (int g = 0; g < G; ++g) {
    wp[g] = ws[g].data_ptr();
    sp[g] = (g < (int)scales.size() && scales[g].has_value()) ? scales[g]->data_ptr() : nullptr;
  }
  air::GemmArgs a{};
  a.N = (int)N;
  a.K = (int)K;
  a.mode = out.scalar_type() == at::kBFloat16 ? air::kGemmStoreBF16 : air::kGemmStoreF32;
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.splits = 1;
  a.err = err.data_ptr<int>();
  a.row_count = row_counts.data_ptr<int>();
  const char* e = air::launch_gemm_q_grouped((int)fmt, wp, sp, G, row_bytes, x.data_ptr(), x.stride(0), (int)rows, a,
                                             at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == nullptr, e ? e : "");
  cudaError_t ce = cudaGetLastError();
  TORCH_CHECK(ce == cudaSuccess, "gemm_q_grouped launch: ", cudaGetErrorString(ce));
}

}  // namespace

void register_gemm_tc(pybind11::module_& m) {
  m.def("gemm_q", &gemm_q);
  m.def("gemm_q_grouped", &gemm_q_grouped);
  m.def("gemm_q_splits", [](int64_t N, int64_t K, int64_t T, int64_t fmt) {
    return air::gemm_q_splits((int)N, (int)K, (int)T, (int)fmt);
  });
  m.def("gemm_q_workspace", [](int64_t N, int64_t K, int64_t T, int64_t fmt, int64_t splits) {
    return (int64_t)air::gemm_q_workspace_floats((int)N, (int)K, (int)T, (int)fmt, (int)splits);
  });
  m.def("gemm_q_counters", [](int64_t N, int64_t T) { return (int64_t)air::gemm_q_counters((int)N, (int)T); });
}
