// FlashAttention forward/backward on tcgen05 (sm_100a).  (kernels being written)
#include <torch/extension.h>

namespace mykb {
std::vector<torch::Tensor> fa_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, c10::optional<torch::Tensor> cu_q,
                                  c10::optional<torch::Tensor> cu_k, c10::optional<torch::Tensor> seqused_k,
                                  int64_t max_q, int64_t max_k, double scale, int64_t left, int64_t right) {
  TORCH_CHECK(false, "fa_fwd: not built yet");
}
std::vector<torch::Tensor> fa_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                  torch::Tensor out, torch::Tensor lse, c10::optional<torch::Tensor> cu_q,
                                  c10::optional<torch::Tensor> cu_k, int64_t max_q, int64_t max_k, double scale,
                                  int64_t left, int64_t right) {
  TORCH_CHECK(false, "fa_bwd: not built yet");
}
}  // namespace mykb
