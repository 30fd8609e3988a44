// Per-device status word written by kernels whose bounded waits gave up (see common.cuh).
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace mykb {

int* device_status() {
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (ptrs[dev] == nullptr) {
    C10_CUDA_CHECK(cudaMalloc(&ptrs[dev], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(ptrs[dev], 0, sizeof(int)));
  }
  return ptrs[dev];
}

// Returns the status word of the current device and clears it (synchronises the device).
int64_t take_status() {
  int* d = device_status();
  int h = 0;
  C10_CUDA_CHECK(cudaMemcpy(&h, d, sizeof(int), cudaMemcpyDeviceToHost));
  if (h != 0) C10_CUDA_CHECK(cudaMemset(d, 0, sizeof(int)));
  return h;
}

}  // namespace mykb
