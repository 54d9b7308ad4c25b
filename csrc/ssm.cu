// Gated delta rule recurrence on the GPU (the DeltaNet layers of Qwen3.6-style hybrids;
// reference src/gated_deltanet.rs and the Metal deltanet_recurrence kernel):
//   S_t = alpha_t S_{t-1} (I - beta_t k_t k_t^T) + beta_t v_t k_t^T,   o_t = S_t q_t
// One CTA per (batch, head); the state S [dv, dk] lives in registers for the whole sequence:
// four threads per state row, each holding dk/4 columns, so the row products S k and S q are
// four-lane shuffle reductions and a token costs two broadcast reads of k_t and q_t.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"

namespace air {
namespace {

template <int DK>
__global__ void __launch_bounds__(512)
gated_delta_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                   const float* __restrict__ alpha, const float* __restrict__ beta, float* __restrict__ state,
                   float* __restrict__ out, int L, int DV) {
  constexpr int J = DK / 4;
  __shared__ float sk[DK], sq[DK];
  const int bh = blockIdx.x, t = threadIdx.x;
  const int i = t >> 2, p = t & 3;
  const bool row = i < DV;
  float S[J];
  float* st = state + ((size_t)bh * DV + (row ? i : 0)) * DK + p * J;
#pragma unroll
  for (int j = 0; j < J; ++j) S[j] = row ? st[j] : 0.f;
  for (int l = 0; l < L; ++l) {
    const size_t tok = (size_t)bh * L + l;
    for (int x = t; x < DK; x += blockDim.x) {
      sk[x] = k[tok * DK + x];
      sq[x] = q[tok * DK + x];
    }
    __syncthreads();
    const float a = alpha[tok], b = beta[tok];
    const float vi = row ? v[tok * DV + i] : 0.f;
    float d = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) d += S[j] * sk[p * J + j];
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    float o = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const float kj = sk[p * J + j];
      S[j] = a * (S[j] - b * d * kj) + b * vi * kj;
      o += S[j] * sq[p * J + j];
    }
    o += __shfl_xor_sync(0xffffffffu, o, 1);
    o += __shfl_xor_sync(0xffffffffu, o, 2);
    if (row && p == 0) out[tok * DV + i] = o;
    __syncthreads();                    // sk / sq are overwritten by the next token
  }
  if (row) {
#pragma unroll
    for (int j = 0; j < J; ++j) st[j] = S[j];
  }
}

}  // namespace
}  // namespace air

using at::Tensor;

// q, k [BH, L, dk], v [BH, L, dv], alpha, beta [BH, L] (fp32, contiguous); state [BH, dv, dk]
// is read as the initial state and overwritten with the final one; out [BH, L, dv].
void gated_delta(Tensor q, Tensor k, Tensor v, Tensor alpha, Tensor beta, Tensor state, Tensor out) {
  for (const Tensor* x : {&q, &k, &v, &alpha, &beta, &state, &out})
    TORCH_CHECK(x->is_cuda() && x->scalar_type() == torch::kFloat && x->is_contiguous(),
                "gated_delta: contiguous fp32 CUDA tensors");
  const int64_t BH = q.size(0), L = q.size(1), DK = q.size(2), DV = v.size(2);
  TORCH_CHECK(k.sizes() == q.sizes() && v.size(0) == BH && v.size(1) == L && alpha.numel() == BH * L &&
                  beta.numel() == BH * L && state.numel() == BH * DV * DK && out.numel() == BH * L * DV,
              "gated_delta: shape mismatch");
  TORCH_CHECK((DK == 64 || DK == 128) && DV >= 8 && DV <= 128 && DV % 8 == 0,
              "gated_delta: dk in {64, 128}, dv a multiple of 8 up to 128");
  if (BH == 0 || L == 0) return;
  const int threads = (int)DV * 4;
  auto st = at::cuda::getCurrentCUDAStream();
  if (DK == 128)
    air::gated_delta_kernel<128><<<(unsigned)BH, threads, 0, st>>>(
        q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), alpha.data_ptr<float>(),
        beta.data_ptr<float>(), state.data_ptr<float>(), out.data_ptr<float>(), (int)L, (int)DV);
  else
    air::gated_delta_kernel<64><<<(unsigned)BH, threads, 0, st>>>(
        q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), alpha.data_ptr<float>(),
        beta.data_ptr<float>(), state.data_ptr<float>(), out.data_ptr<float>(), (int)L, (int)DV);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "gated_delta launch");
}

void register_ssm(pybind11::module_& m) {
  m.def("gated_delta", &gated_delta);
}
