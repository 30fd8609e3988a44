// Per-device status word written by kernels whose bounded waits gave up (see common.cuh).
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace mykb {

namespace {
std::mutex g_pool_mu;  // guards the per-device lazily created buffers below
}

int* device_status() {
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  TORCH_CHECK(dev >= 0 && dev < 64, "device index out of range");
  std::lock_guard<std::mutex> lock(g_pool_mu);
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

// Split-K / split-KV kernels count arriving CTAs on "tickets" that the last CTA resets to
// zero, so one zeroed pool per device serves every launch.  Each launch takes the next
// `count` tickets of a ring of kTicketPool; a region comes round again only after
// kTicketPool tickets of later launches, long after its own launch has finished.
int* ticket_region(int count) {
  constexpr int kTicketPool = 1 << 20;
  static int* pools[64] = {nullptr};
  static int next[64] = {0};
  TORCH_CHECK(count > 0 && count <= kTicketPool / 4, "ticket_region: too many tickets (", count, ")");
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  TORCH_CHECK(dev >= 0 && dev < 64, "device index out of range");
  std::lock_guard<std::mutex> lock(g_pool_mu);
  if (pools[dev] == nullptr) {
    C10_CUDA_CHECK(cudaMalloc(&pools[dev], sizeof(int) * kTicketPool));
    C10_CUDA_CHECK(cudaMemset(pools[dev], 0, sizeof(int) * kTicketPool));
  }
  if (next[dev] + count > kTicketPool) next[dev] = 0;
  int* r = pools[dev] + next[dev];
  next[dev] += count;
  return r;
}

}  // namespace mykb
