// torch adapter of the fused tensor-parallel all-reduce (comm.h): symmetric receive
// buffers (cudaMalloc'd here so an IPC handle covers exactly the buffer), CUDA IPC handle
// export/import between the ranks' processes, and the producer/consumer launches.
//
// Pointer tables travel as int64 CPU tensors ("meta"):
//   push meta  : data[8], epoch, slot_elems, world, rank, row_len, shard
//   reduce meta: rs, ag, ag_peer[8], epoch, done, err, slot_elems, world, rank, timeout_ns, shard
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cstring>
#include <vector>
#include <torch/csrc/utils/pybind.h>

#include "comm.h"

using at::Tensor;
using c10::optional;

namespace {

void ck(cudaError_t e, const char* what) { TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e)); }

Tensor comm_alloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  ck(cudaMalloc(&p, bytes), "comm_alloc");
  ck(cudaMemset(p, 0, bytes), "comm_alloc memset");
  ck(cudaDeviceSynchronize(), "comm_alloc sync");
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  return torch::from_blob(p, {bytes}, [](void* q) { cudaFree(q); }, opts);
}

pybind11::bytes ipc_handle(const Tensor& t) {
  cudaIpcMemHandle_t h;
  ck(cudaIpcGetMemHandle(&h, t.data_ptr()), "cudaIpcGetMemHandle");
  return pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(const std::string& handle, int64_t device) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}

// Lets kernels on `device` dereference pointers into `peer`'s memory (same process).
bool enable_peer_access(int64_t device, int64_t peer) {
  int ok = 0;
  ck(cudaDeviceCanAccessPeer(&ok, (int)device, (int)peer), "cudaDeviceCanAccessPeer");
  if (!ok) return false;
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaError_t e = cudaDeviceEnablePeerAccess((int)peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return true;
  }
  ck(e, "cudaDeviceEnablePeerAccess");
  return true;
}

void ipc_close(int64_t ptr) { ck(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle"); }

// reduce meta: rs, ag, ag_peer[8], epoch, done, err, slot_elems, world, rank, timeout_ns, shard
air::TPReduceRank reduce_rank_from_meta(const Tensor& meta, int64_t* slot, int* world, int64_t* timeout,
                                        int64_t* shard) {
  TORCH_CHECK(meta.device().is_cpu() && meta.scalar_type() == torch::kLong && meta.numel() >= 18, "reduce meta");
  const int64_t* m = meta.data_ptr<int64_t>();
  air::TPReduceRank r{};
  r.rs = reinterpret_cast<const uint2*>(m[0]);
  r.ag = reinterpret_cast<const uint2*>(m[1]);
  for (int i = 0; i < air::kMaxPeers; ++i) r.ag_peer[i] = reinterpret_cast<uint2*>(m[2 + i]);
  r.epoch = reinterpret_cast<int*>(m[10]);
  r.done = reinterpret_cast<int*>(m[11]);
  r.err = reinterpret_cast<int*>(m[12]);
  *slot = m[13];
  *world = (int)m[14];
  r.rank = (int)m[15];
  *timeout = m[16];
  *shard = m[17];
  return r;
}

// x[b] += sum of the ranks' partials, then RMSNorm (+ Q8A / bf16 outputs). One meta (and one
// x / q / ds / y) per rank handled by this launch: a real TP group passes one; the
// single-GPU emulation of a group passes all of them, so the two-shot exchange between ranks
// happens inside one launch.
void tp_reduce_norm(const std::vector<Tensor>& metas, const std::vector<Tensor>& xs, optional<Tensor> w,
                    double w_offset, double eps, int64_t B, int64_t K, const std::vector<optional<Tensor>>& qs,
                    const std::vector<optional<Tensor>>& dss, const std::vector<optional<Tensor>>& ys,
                    bool two_shot, optional<Tensor> bias, int64_t layer) {
  const int n = (int)metas.size();
  TORCH_CHECK(n >= 1 && n <= air::kMaxPeers && (int)xs.size() == n, "tp_reduce_norm: 1..8 ranks, one x each");
  TORCH_CHECK(qs.empty() || (int)qs.size() == n, "tp_reduce_norm: q per rank");
  TORCH_CHECK(dss.empty() || (int)dss.size() == n, "tp_reduce_norm: ds per rank");
  TORCH_CHECK(ys.empty() || (int)ys.size() == n, "tp_reduce_norm: y per rank");
  TORCH_CHECK(K % 32 == 0 && K <= 16384, "tp_reduce_norm: K must be a multiple of 32, <= 16384");
  // two-shot CTAs wait for the other ranks' CTAs of the same launch (emulated group) or of
  // the peers' launches: every CTA must be resident at once (one 1024-thread CTA per SM)
  TORCH_CHECK(B >= 1 && (!two_shot || B * n <= 148), "tp_reduce_norm: two-shot needs B x ranks-in-launch <= 148");
  auto p = [](const optional<Tensor>& t) { return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr; };
  air::TPReduceArgs a{};
  a.n_local = n;
  for (int i = 0; i < n; ++i) {
    int64_t slot, timeout, shard;
    int world;
    a.r[i] = reduce_rank_from_meta(metas[i], &slot, &world, &timeout, &shard);
    a.slot_elems = slot;
    a.world = world;
    a.timeout_ns = timeout;
    a.shard = two_shot ? shard : 0;
    TORCH_CHECK(B * K <= slot, "tp_reduce_norm: B*K exceeds the receive slot");
    TORCH_CHECK(!two_shot || (shard > 0 && shard % 32 == 0 && shard * world >= K),
                "tp_reduce_norm: two-shot needs a positive shard, a multiple of 32, covering K");
    const Tensor& x = xs[i];
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat && x.is_contiguous() && x.numel() >= B * K,
                "x must be contiguous fp32 CUDA [B, K]");
    a.r[i].x = x.data_ptr<float>();
    a.r[i].q = qs.empty() ? nullptr : static_cast<int8_t*>(p(qs[i]));
    a.r[i].ds = dss.empty() ? nullptr : static_cast<float2*>(p(dss[i]));
    a.r[i].y_bf16 = ys.empty() ? nullptr : p(ys[i]);
    TORCH_CHECK((a.r[i].q == nullptr) == (a.r[i].ds == nullptr), "tp_reduce_norm: q and ds go together");
  }
  a.w = static_cast<const float*>(p(w));
  a.w_offset = (float)w_offset;
  a.bias = static_cast<const float*>(p(bias));
  a.layer = (int)layer;
  a.eps = (float)eps;
  a.B = (int)B;
  a.K = (int)K;
  air::launch_tp_reduce_norm(a, at::cuda::getCurrentCUDAStream());
  ck(cudaGetLastError(), "tp_reduce_norm");
}

// NVLS consumer of one rank. meta (int64, CPU): multicast partial region, local flags,
// flags of ranks 0..7 (mapped here), epoch, done, err, world, rank, timeout_ns, slot_elems.
void tp_reduce_norm_nvls(const Tensor& meta, const Tensor& x, optional<Tensor> w, double w_offset, double eps,
                         int64_t B, int64_t K, optional<Tensor> q, optional<Tensor> ds, optional<Tensor> y,
                         optional<Tensor> bias, int64_t layer) {
  TORCH_CHECK(meta.device().is_cpu() && meta.scalar_type() == torch::kLong && meta.numel() >= 17, "nvls meta");
  const int64_t* m = meta.data_ptr<int64_t>();
  TORCH_CHECK(K % 32 == 0 && K <= 16384 && B >= 1 && B * K <= m[16], "tp_reduce_norm_nvls: B x K must fit the slot");
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat && x.is_contiguous() && x.numel() >= B * K,
              "x must be contiguous fp32 CUDA [B, K]");
  TORCH_CHECK(m[0] != 0 && m[0] % 16 == 0, "tp_reduce_norm_nvls: multicast address");
  auto p = [](const optional<Tensor>& t) { return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr; };
  air::TPReduceArgs a{};
  a.n_local = 1;
  a.nvls = 1;
  a.world = (int)m[13];
  TORCH_CHECK(a.world >= 1 && a.world <= air::kMaxPeers && m[14] >= 0 && m[14] < a.world, "nvls meta: world/rank");
  a.timeout_ns = m[15];
  a.slot_elems = m[16];
  air::TPReduceRank& r = a.r[0];
  r.mc = reinterpret_cast<const float*>(m[0]);
  r.flags = reinterpret_cast<int*>(m[1]);
  for (int i = 0; i < air::kMaxPeers; ++i) r.flags_peer[i] = reinterpret_cast<int*>(m[2 + i]);
  r.epoch = reinterpret_cast<int*>(m[10]);
  r.done = reinterpret_cast<int*>(m[11]);
  r.err = reinterpret_cast<int*>(m[12]);
  r.rank = (int)m[14];
  r.x = x.data_ptr<float>();
  r.q = static_cast<int8_t*>(p(q));
  r.ds = static_cast<float2*>(p(ds));
  r.y_bf16 = p(y);
  TORCH_CHECK((r.q == nullptr) == (r.ds == nullptr), "tp_reduce_norm_nvls: q and ds go together");
  a.w = static_cast<const float*>(p(w));
  a.w_offset = (float)w_offset;
  a.bias = static_cast<const float*>(p(bias));
  a.layer = (int)layer;
  a.eps = (float)eps;
  a.B = (int)B;
  a.K = (int)K;
  air::launch_tp_reduce_norm(a, at::cuda::getCurrentCUDAStream());
  ck(cudaGetLastError(), "tp_reduce_norm_nvls");
}

}  // namespace

// push meta: data[8], epoch, slot_elems, world, rank, row_len, shard
air::PeerPush peer_push_from_meta(const Tensor& meta) {
  TORCH_CHECK(meta.device().is_cpu() && meta.scalar_type() == torch::kLong && meta.numel() >= 14, "push meta");
  const int64_t* m = meta.data_ptr<int64_t>();
  air::PeerPush p{};
  for (int i = 0; i < air::kMaxPeers; ++i) p.data[i] = reinterpret_cast<uint2*>(m[i]);
  p.epoch = reinterpret_cast<const int*>(m[8]);
  p.slot_elems = m[9];
  p.world = (int)m[10];
  p.rank = (int)m[11];
  p.row_len = m[12];
  p.shard = m[13];
  TORCH_CHECK(p.world >= 1 && p.world <= air::kMaxPeers && p.rank >= 0 && p.rank < p.world, "push meta: world/rank");
  TORCH_CHECK(p.row_len > 0 && p.shard >= 0 && (p.shard == 0 || p.shard * p.world >= p.row_len),
              "push meta: row length / shard");
  return p;
}

void register_comm(pybind11::module_& m) {
  m.def("comm_alloc", &comm_alloc);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("enable_peer_access", &enable_peer_access);
  m.def("peer_buffer_bytes", [](int64_t w, int64_t s) { return air::peer_buffer_bytes((int)w, s); });
  m.def("tp_reduce_norm", &tp_reduce_norm);
  m.def("tp_reduce_norm_nvls", &tp_reduce_norm_nvls);
  m.def("peer_push", [](const Tensor& meta, const Tensor& src, int64_t B, int64_t N, int64_t ld) {
    TORCH_CHECK(src.is_cuda() && src.scalar_type() == torch::kFloat, "peer_push: fp32 CUDA source");
    const air::PeerPush p = peer_push_from_meta(meta);
    TORCH_CHECK(N == p.row_len && B * p.row_len <= p.slot_elems, "peer_push: [B, N] must fit the receive slot, N = row length");
    air::launch_peer_push(p, src.data_ptr<float>(), (int)B, (int)N, ld, at::cuda::getCurrentCUDAStream());
    ck(cudaGetLastError(), "peer_push");
  });
}
