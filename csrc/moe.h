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

// Routed-expert grouping (per expert e): select the tokens with cw[t, e] > 0 (in token order)
// into idx / wts / *count; gather their bf16 rows into xg [cap, H]; scatter-add
// wts[i] * y[i] back into out[idx[i]] (fp32 [T, H]). Kernels past *count do nothing, so the
// launches have a fixed shape (graph capturable).
void launch_moe_select(const float* cw, int e, int E, int T, int* idx, float* wts, int* count, cudaStream_t st);
void launch_moe_gather(const void* x, int64_t ldx, int H, const int* idx, const int* count, int cap, void* xg,
                       cudaStream_t st);
void launch_moe_scatter(float* out, const float* y, int64_t ldy, int H, const int* idx, const float* wts,
                        const int* count, int cap, cudaStream_t st);

// Grouped over G local experts (ids in `experts`, device int32): packed buffers of G * T rows,
// group g at rows [g * T, g * T + T). pos[g * T + t] = packed row of token t in group g or -1.
// The scatter sums every group's weighted output per token in group order.
void launch_moe_select_grouped(const float* cw, const int* experts, int G, int E, int T, int* idx, float* wts,
                               int* count, int* pos, cudaStream_t st);
void launch_moe_gather_grouped(const void* x, int64_t ldx, int H, const int* idx, const int* count, int G, int T,
                               void* xg, cudaStream_t st);
void launch_moe_scatter_grouped(float* out, const float* y, int64_t ldy, int H, const int* pos, const float* wts,
                                int G, int T, cudaStream_t st);

}  // namespace air
