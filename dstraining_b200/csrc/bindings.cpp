// Python module for the sm_100a kernels (dstraining_b200._C).
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <mutex>

#include "common.h"

namespace dst {

int* status_ptr() {
  static int* ptrs[64] = {nullptr};
  static std::mutex mu;
  int dev;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    C10_CUDA_CHECK(cudaMalloc(&ptrs[dev], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(ptrs[dev], 0, sizeof(int)));
  }
  return ptrs[dev];
}

}  // namespace dst

// Read and clear the device status word (synchronises the device).
static int64_t read_status(bool clear) {
  int* p = dst::status_ptr();
  int v = 0;
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  C10_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  return v;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "dstraining_b200 sm_100a kernels";
  m.def("read_status", &read_status, "read (and optionally clear) the device status word", py::arg("clear") = true);
  m.def("num_sms", &dst::num_sms);
  register_gemm(m);
  register_norm(m);
  register_embed(m);
  register_adam(m);
  register_ce(m);
  register_attn_tc(m);
  register_symm(m);
  register_tp(m);
}
