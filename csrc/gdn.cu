// Gated DeltaNet kernels (sm_100a).  (kernels being written)
#include <torch/extension.h>

namespace mykb {
std::vector<torch::Tensor> conv1d_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> cu,
                                      c10::optional<torch::Tensor> init) { TORCH_CHECK(false, "conv1d_fwd: not built yet"); }
std::vector<torch::Tensor> conv1d_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w,
                                      c10::optional<torch::Tensor> cu, c10::optional<torch::Tensor> init) { TORCH_CHECK(false, "conv1d_bwd: not built yet"); }
std::vector<torch::Tensor> gdn_chunk_fwd_entry(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                               torch::Tensor beta, c10::optional<torch::Tensor> init,
                                               c10::optional<torch::Tensor> cu, bool per_channel) { TORCH_CHECK(false, "gdn: not built yet"); }
std::vector<torch::Tensor> gdn_chunk_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                         torch::Tensor g, torch::Tensor beta, c10::optional<torch::Tensor> init,
                                         c10::optional<torch::Tensor> cu, std::vector<torch::Tensor> saved,
                                         bool per_channel) { TORCH_CHECK(false, "gdn: not built yet"); }
std::vector<torch::Tensor> gdn_recurrent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                         torch::Tensor beta, c10::optional<torch::Tensor> init, bool per_channel) { TORCH_CHECK(false, "gdn: not built yet"); }
}  // namespace mykb
