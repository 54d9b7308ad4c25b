#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <vector>
#include <torch/csrc/utils/pybind.h>
#include "gemm_tc.h"
#include "gemm_fp8.h"

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

// W8A8 FP8: activation codes + one scale per token from bf16 rows.
void quant_fp8_rows(Tensor x, Tensor xq, Tensor xs) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "quant_fp8_rows: x must be 2-D bf16 with contiguous rows");
  const int64_t T = x.size(0), K = x.size(1);
  TORCH_CHECK(xq.is_contiguous() && xq.numel() >= T * K && xq.element_size() == 1, "quant_fp8_rows: xq [T, K] bytes");
  TORCH_CHECK(xs.is_contiguous() && xs.scalar_type() == at::kFloat && xs.numel() >= T,
              "quant_fp8_rows: xs f32 [T]");
  const char* e = air::launch_quant_fp8_rows(x.data_ptr(), x.stride(0), (int)T, (int)K, xq.data_ptr(),
                                             xs.data_ptr<float>(), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == nullptr, e ? e : "");
  cudaError_t ce = cudaGetLastError();
  TORCH_CHECK(ce == cudaSuccess, "quant_fp8_rows launch: ", cudaGetErrorString(ce));
}

// W8A8 FP8 tensor-core GEMM: out [T, N] (f32 / bf16 store, or f32 residual add).
void gemm_fp8(Tensor wq, Tensor wscale, int64_t row_bytes, int64_t N, int64_t K, Tensor xq, Tensor xs, Tensor out,
              int64_t mode, int64_t splits, optional<Tensor> ws, optional<Tensor> counters, Tensor err) {
  TORCH_CHECK(wq.is_cuda() && xq.is_cuda() && wscale.scalar_type() == at::kFloat && xs.scalar_type() == at::kFloat,
              "gemm_fp8: CUDA codes and f32 scales");
  TORCH_CHECK(K % 128 == 0 && xq.is_contiguous() && xq.dim() == 2 && xq.size(1) == K, "gemm_fp8: xq [T, K]");
  const int64_t T = xq.size(0);
  TORCH_CHECK(wscale.numel() >= N * (K / 128) && xs.numel() >= T, "gemm_fp8: scale shapes");
  TORCH_CHECK(out.stride(1) == 1 && out.size(0) >= T && out.size(1) >= N, "gemm_fp8: out [T, N] with contiguous rows");
  TORCH_CHECK(out.scalar_type() == (mode == air::kGemmStoreBF16 ? at::kBFloat16 : at::kFloat),
              "gemm_fp8: out must be bf16 for the bf16 store, else f32");
  air::GemmF8Args a{};
  a.N = (int)N;
  a.K = (int)K;
  a.T = (int)T;
  a.mode = (int)mode;
  a.wq = wq.data_ptr();
  a.w_row_bytes = row_bytes;
  a.wscale = wscale.data_ptr<float>();
  a.xq = xq.data_ptr();
  a.xscale = xs.data_ptr<float>();
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.splits = (int)std::max<int64_t>(1, splits);
  if (a.splits > 1) {
    TORCH_CHECK(ws.has_value() && counters.has_value(), "gemm_fp8: split-K needs ws and counters");
    TORCH_CHECK((size_t)ws->numel() >= air::gemm_fp8_workspace_floats(a.N, a.T, a.splits), "gemm_fp8: workspace too small");
    TORCH_CHECK((size_t)counters->numel() >= air::gemm_fp8_counters(a.N, a.T), "gemm_fp8: counters too small");
    a.ws = ws->data_ptr<float>();
    a.counters = counters->data_ptr<int>();
  }
  a.err = err.data_ptr<int>();
  const char* e = air::launch_gemm_fp8(a, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == nullptr, e ? e : "");
  cudaError_t ce = cudaGetLastError();
  TORCH_CHECK(ce == cudaSuccess, "gemm_fp8 launch: ", cudaGetErrorString(ce));
}

}  // namespace

void register_gemm_tc(pybind11::module_& m) {
  m.def("gemm_fp8", &gemm_fp8);
  m.def("quant_fp8_rows", &quant_fp8_rows);
  m.def("gemm_fp8_splits", [](int64_t N, int64_t K, int64_t T) { return air::gemm_fp8_splits((int)N, (int)K, (int)T); });
  m.def("gemm_fp8_workspace", [](int64_t N, int64_t T, int64_t splits) {
    return (int64_t)air::gemm_fp8_workspace_floats((int)N, (int)T, (int)splits);
  });
  m.def("gemm_fp8_counters", [](int64_t N, int64_t T) { return (int64_t)air::gemm_fp8_counters((int)N, (int)T); });
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
