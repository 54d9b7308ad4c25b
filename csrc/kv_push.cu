// Prefill -> decode KV hand-off over NVLink: one launch copies every (layer, block) pair of
// a sequence from this GPU's paged KV pool straight into the decode GPU's pool (mapped here
// through CUDA IPC) and raises one completion flag per pair in the decode GPU's memory; the
// decode side runs kv_wait on its compute stream (bounded) before the first decode step.
// Reference: src/pd_disagg.rs PrefillNode::prefill_and_send / DecodeNode::recv_and_prepare
// (TCP frames of int8-quantised blocks there).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "comm.cuh"
#include "sm100.cuh"

namespace air {
namespace {

// Grid (n_blocks, n_layers), 256 threads: CTA copies one block_bytes chunk with 16-byte
// vector loads / peer stores, then (fence, barrier) flags[layer * flag_stride + dst_block] = tag.
__global__ void __launch_bounds__(256)
kv_push_kernel(const uint8_t* __restrict__ src, int64_t src_layer_stride, uint8_t* dst, int64_t dst_layer_stride,
               int64_t block_bytes, const int* __restrict__ src_blocks, const int* __restrict__ dst_blocks,
               int* flags, int64_t flag_stride, int tag, int64_t src_nb, int64_t dst_nb, int* err) {
  const int i = blockIdx.x, l = blockIdx.y;
  const int sb = src_blocks[i], db = dst_blocks[i];
  if (sb < 0 || sb >= src_nb || db < 0 || db >= dst_nb) {
    if (threadIdx.x == 0) set_error(err, kErrBounds);
    return;
  }
  const uint4* s = reinterpret_cast<const uint4*>(src + l * src_layer_stride + (int64_t)sb * block_bytes);
  uint4* d = reinterpret_cast<uint4*>(dst + l * dst_layer_stride + (int64_t)db * block_bytes);
  const int64_t n = block_bytes / 16;
  for (int64_t k = threadIdx.x; k < n; k += blockDim.x) d[k] = __ldcg(s + k);
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) st_release_sys(flags + l * flag_stride + db, tag);
}

// One thread per (layer, block) flag; bounded wait; status 0 = all arrived, 2 = timeout.
__global__ void kv_wait_kernel(const int* flags, int64_t flag_stride, const int* __restrict__ dst_blocks,
                               int n_blocks, int n_layers, int tag, int64_t timeout_ns, int* status) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_blocks * n_layers) return;
  const int l = idx / n_blocks, b = dst_blocks[idx % n_blocks];
  const int* f = flags + l * flag_stride + b;
  if (ld_acquire_sys(f) == tag) return;
  const uint64_t t0 = sm100::global_ns();
  for (uint32_t it = 1;; ++it) {
    if (ld_acquire_sys(f) == tag) return;
    if ((it & 63) == 0 && sm100::global_ns() - t0 > (uint64_t)timeout_ns) {
      atomicCAS(status, 0, (int)kErrTimeout);
      return;
    }
  }
}

}  // namespace
}  // namespace air

using at::Tensor;

// src / dst: the two pools' base addresses (dst may be a peer mapping); layer strides and
// block size in bytes; block id lists as int32 CUDA tensors (same length).
void kv_push(int64_t src, int64_t src_layer_stride, int64_t src_nb, int64_t dst, int64_t dst_layer_stride,
             int64_t dst_nb, int64_t block_bytes, int64_t n_layers, Tensor src_blocks, Tensor dst_blocks,
             int64_t flags, int64_t flag_stride, int64_t tag, Tensor err) {
  TORCH_CHECK(src_blocks.is_cuda() && dst_blocks.is_cuda() && src_blocks.scalar_type() == torch::kInt &&
                  dst_blocks.scalar_type() == torch::kInt && src_blocks.numel() == dst_blocks.numel(),
              "kv_push: int32 CUDA block lists of equal length");
  TORCH_CHECK(block_bytes % 16 == 0 && src % 16 == 0 && dst % 16 == 0 && src_layer_stride % 16 == 0 &&
                  dst_layer_stride % 16 == 0, "kv_push: 16-byte alignment");
  const int nb = (int)src_blocks.numel();
  if (nb == 0) return;
  air::kv_push_kernel<<<dim3(nb, (unsigned)n_layers), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint8_t*>(src), src_layer_stride, reinterpret_cast<uint8_t*>(dst), dst_layer_stride,
      block_bytes, src_blocks.data_ptr<int>(), dst_blocks.data_ptr<int>(), reinterpret_cast<int*>(flags), flag_stride,
      (int)tag, src_nb, dst_nb, err.data_ptr<int>());
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "kv_push launch");
}

void kv_wait(int64_t flags, int64_t flag_stride, Tensor dst_blocks, int64_t n_layers, int64_t tag,
             double timeout_s, Tensor status) {
  const int nb = (int)dst_blocks.numel();
  const int n = nb * (int)n_layers;
  if (n == 0) return;
  air::kv_wait_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const int*>(flags), flag_stride, dst_blocks.data_ptr<int>(), nb, (int)n_layers, (int)tag,
      (int64_t)(timeout_s * 1e9), status.data_ptr<int>());
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "kv_wait launch");
}

void register_kv_push(pybind11::module_& m) {
  m.def("kv_push", &kv_push);
  m.def("kv_wait", &kv_wait);
}
