// Mixture-of-experts routing and combine kernels (reference src/moe.rs:163-300).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace air {

// Per token: logits = router[E, H] . x[t] (fp32 router), softmax over E, top-k, optional
// renormalisation of the selected weights. Writes the dense combine matrix cw[T, E]
// (zero for unselected experts) and optionally ids/weights [T, k]. E <= 256, k <= 8.
void launch_moe_route(const void* x, bool x_bf16, int64_t ldx, int T, int H, const float* router, int E, int k,
                      bool normalize, float* cw, int* ids, float* wts, cudaStream_t st);

// x[t, :] += cw[t, e] * y[t, :]   (y fp32 [T, ldy])
void launch_moe_combine(float* x, const float* y, int64_t ldy, const float* cw, int e, int E, int T, int H,
                        cudaStream_t st);

}  // namespace air
