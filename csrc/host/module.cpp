// air_rs._host: the CPU-side native runtime (no CUDA dependency, so it also loads on
// machines without a GPU): paged-KV bookkeeping, the batch scheduler core, and the STRIX
// VRAM budget arena and host staging-buffer pool.
#ifdef AIR_HOST_NO_TORCH
#include <pybind11/pybind11.h>
#define TORCH_EXTENSION_NAME _host
#else
#include <torch/extension.h>
#endif

void register_host_kv(pybind11::module_& m);
void register_arena(pybind11::module_& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "air_rs native host runtime";
  register_host_kv(m);
  register_arena(m);
}
