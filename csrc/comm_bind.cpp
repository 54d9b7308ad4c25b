// torch adapter of the fused tensor-parallel all-reduce (comm.h): symmetric receive
// buffers (cudaMalloc'd here so an IPC handle covers exactly the buffer), CUDA IPC handle
// export/import between the ranks' processes, and the producer/consumer launches.
//
// Pointer tables travel as int64 CPU tensors ("meta"):
//   push meta  : data[8], epoch, slot_elems, world, rank
//   reduce meta: data, epoch, done, err, slot_elems, world, timeout_ns
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cstring>

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

void reduce_rmsnorm_quant(const Tensor& meta, Tensor x, optional<Tensor> w, double w_offset, double eps, int64_t B,
                          int64_t K, optional<Tensor> q, optional<Tensor> ds, optional<Tensor> y_bf16) {
  TORCH_CHECK(meta.device().is_cpu() && meta.scalar_type() == torch::kLong && meta.numel() >= 7, "reduce meta");
  TORCH_CHECK(K % 32 == 0 && K <= 16384, "reduce_rmsnorm_quant: K must be a multiple of 32, <= 16384");
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat && x.is_contiguous(), "x must be contiguous fp32 CUDA");
  const int64_t* m = meta.data_ptr<int64_t>();
  air::PeerReduce r{};
  r.data = reinterpret_cast<const uint2*>(m[0]);
  r.epoch = reinterpret_cast<int*>(m[1]);
  r.done = reinterpret_cast<int*>(m[2]);
  r.err = reinterpret_cast<int*>(m[3]);
  r.slot_elems = m[4];
  r.world = (int)m[5];
  r.timeout_ns = m[6];
  TORCH_CHECK(B * K <= r.slot_elems, "reduce_rmsnorm_quant: B*K exceeds the receive slot");
  auto p = [](const optional<Tensor>& t) { return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr; };
  air::launch_reduce_rmsnorm_quant(r, x.data_ptr<float>(), static_cast<const float*>(p(w)), (float)w_offset,
                                   (int)B, (int)K, (float)eps, static_cast<int8_t*>(p(q)), static_cast<float2*>(p(ds)),
                                   p(y_bf16), at::cuda::getCurrentCUDAStream());
  ck(cudaGetLastError(), "reduce_rmsnorm_quant");
}

}  // namespace

air::PeerPush peer_push_from_meta(const Tensor& meta) {
  TORCH_CHECK(meta.device().is_cpu() && meta.scalar_type() == torch::kLong && meta.numel() >= 12, "push meta");
  const int64_t* m = meta.data_ptr<int64_t>();
  air::PeerPush p{};
  for (int i = 0; i < air::kMaxPeers; ++i) p.data[i] = reinterpret_cast<uint2*>(m[i]);
  p.epoch = reinterpret_cast<const int*>(m[8]);
  p.slot_elems = m[9];
  p.world = (int)m[10];
  p.rank = (int)m[11];
  TORCH_CHECK(p.world >= 1 && p.world <= air::kMaxPeers && p.rank >= 0 && p.rank < p.world, "push meta: world/rank");
  return p;
}

void register_comm(pybind11::module_& m) {
  m.def("comm_alloc", &comm_alloc);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("enable_peer_access", &enable_peer_access);
  m.def("peer_buffer_bytes", [](int64_t w, int64_t s) { return air::peer_buffer_bytes((int)w, s); });
  m.def("reduce_rmsnorm_quant", &reduce_rmsnorm_quant);
  m.def("peer_push", [](const Tensor& meta, const Tensor& src, int64_t B, int64_t N, int64_t ld) {
    TORCH_CHECK(src.is_cuda() && src.scalar_type() == torch::kFloat, "peer_push: fp32 CUDA source");
    const air::PeerPush p = peer_push_from_meta(meta);
    TORCH_CHECK(B * ld <= p.slot_elems, "peer_push: B*ld exceeds the receive slot");
    air::launch_peer_push(p, src.data_ptr<float>(), (int)B, (int)N, ld, at::cuda::getCurrentCUDAStream());
    ck(cudaGetLastError(), "peer_push");
  });
}
