// Python bindings of the sm_100a kernels (module myk_llm_b200._C).
#include <torch/extension.h>

namespace mykb {
void fp8_scaled_gemm(torch::Tensor a, torch::Tensor unit_sa, bool a_e5m2, torch::Tensor b, torch::Tensor unit_sb,
                     bool b_e5m2, torch::Tensor row_scale, torch::Tensor col_scale, torch::Tensor d);
torch::Tensor cast_bf16(torch::Tensor src);
void dp_reduce_sumsq_multimem(int64_t grad_mc, torch::Tensor own_grad, torch::Tensor offsets, torch::Tensor prefix,
                              torch::Tensor partial, int64_t total);
void dp_muon_apply_shards(torch::Tensor param_ptrs, torch::Tensor bf16_ptrs, torch::Tensor poffs,
                          torch::Tensor boffs, int64_t rows, int64_t cols, int64_t rows_per_rank, double decay,
                          double step_scale, torch::Tensor orth);
void cast_ranges_bf16(torch::Tensor src, torch::Tensor dst, torch::Tensor src_offsets, torch::Tensor prefix,
                      torch::Tensor dst_offsets, int64_t total);
int64_t take_status();
// gemm.cu
void gemm_gather(torch::Tensor a, torch::Tensor b, torch::Tensor d, bool a_mn, bool b_mn, bool accumulate,
                 torch::Tensor gw, torch::Tensor src_ptrs, int64_t src_offset, int64_t rows_per_rank, int64_t rank,
                 torch::Tensor ready, int64_t epoch);
void shard_gather(torch::Tensor w, torch::Tensor src_ptrs, int64_t src_offset, int64_t rows_per_rank, int64_t rank,
                  torch::Tensor ready, int64_t epoch);
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor d, c10::optional<torch::Tensor> c, bool a_mn, bool b_mn,
          double alpha, double beta, bool accumulate, bool symmetric);
// norm.cu
std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, c10::optional<std::vector<torch::Tensor>> add,
                                       double eps, c10::ScalarType out_dtype);
std::vector<torch::Tensor> rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd,
                                       c10::optional<torch::Tensor> dres, bool bf16_copy);
std::vector<torch::Tensor> gated_rmsnorm_fwd(torch::Tensor o, c10::optional<torch::Tensor> g, torch::Tensor w,
                                             double eps, int64_t act);
std::vector<torch::Tensor> gated_rmsnorm_bwd(torch::Tensor dy, torch::Tensor o, c10::optional<torch::Tensor> g,
                                             torch::Tensor w, torch::Tensor rstd, int64_t act);
// elementwise.cu
torch::Tensor swiglu_fwd(torch::Tensor gu);
torch::Tensor swiglu_bwd(torch::Tensor da, torch::Tensor gu);
torch::Tensor rope(torch::Tensor x, torch::Tensor cos_t, torch::Tensor sin_t, torch::Tensor pos, bool inverse);
std::vector<torch::Tensor> rope_qkv_fwd(torch::Tensor qkv, torch::Tensor cos_t, torch::Tensor sin_t, torch::Tensor pos,
                                        int64_t H, int64_t KV);
std::vector<torch::Tensor> split_cols(torch::Tensor x, std::vector<int64_t> widths);
torch::Tensor rope_qkv_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor cos_t, torch::Tensor sin_t,
                           torch::Tensor pos);
torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor w);
void embedding_bwd(torch::Tensor ids, torch::Tensor dout, torch::Tensor grad);
// fp8.cu
std::vector<torch::Tensor> fp8_quant_rows(torch::Tensor x, bool e5m2, bool pow2);
std::vector<torch::Tensor> fp8_quant_tensor(torch::Tensor x, bool e5m2);
std::vector<torch::Tensor> fp8_quant_cols_t(torch::Tensor x, bool e5m2, bool pow2);
// loss.cu
void ce_fwd_grad(torch::Tensor logits, torch::Tensor targets, double scale, double z_coef, int64_t ignore_index,
                 torch::Tensor ce_sum, torch::Tensor z_sum);
// optim.cu
void adamw_step(std::vector<torch::Tensor> params, std::vector<torch::Tensor> grads, std::vector<torch::Tensor> m,
                std::vector<torch::Tensor> v, int64_t step, double lr, double b1, double b2, double eps, double wd,
                c10::optional<torch::Tensor> gscale);
void muon_prepare(std::vector<torch::Tensor> grads, std::vector<torch::Tensor> bufs, double mu, bool nesterov,
                  torch::Tensor out, c10::optional<torch::Tensor> gscale);
void muon_apply(std::vector<torch::Tensor> params, torch::Tensor orth, double decay, double step_scale);
void frob_normalize_(torch::Tensor x, double eps);
// attention.cu
std::vector<torch::Tensor> fa_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, c10::optional<torch::Tensor> cu_q,
                                  c10::optional<torch::Tensor> cu_k, c10::optional<torch::Tensor> seqused_k,
                                  int64_t max_q, int64_t max_k, double scale, int64_t left, int64_t right);
std::vector<torch::Tensor> fa_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                  torch::Tensor out, torch::Tensor lse, c10::optional<torch::Tensor> cu_q,
                                  c10::optional<torch::Tensor> cu_k, int64_t max_q, int64_t max_k, double scale,
                                  int64_t left, int64_t right);
// gdn.cu
std::vector<torch::Tensor> conv1d_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> cu,
                                      c10::optional<torch::Tensor> init);
std::vector<torch::Tensor> conv1d_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w,
                                      c10::optional<torch::Tensor> cu, c10::optional<torch::Tensor> init);
std::vector<torch::Tensor> gdn_chunk_fwd_entry(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                               torch::Tensor beta, c10::optional<torch::Tensor> init,
                                               c10::optional<torch::Tensor> cu, bool per_channel);
std::vector<torch::Tensor> gdn_chunk_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                         torch::Tensor g, torch::Tensor beta, c10::optional<torch::Tensor> init,
                                         c10::optional<torch::Tensor> cu, std::vector<torch::Tensor> saved,
                                         c10::optional<torch::Tensor> dfinal, bool per_channel);
std::vector<torch::Tensor> gdn_recurrent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                                         torch::Tensor beta, c10::optional<torch::Tensor> init, bool per_channel);
torch::Tensor gdn_spec_window(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                              torch::Tensor state, torch::Tensor pq, torch::Tensor pk, torch::Tensor pv,
                              torch::Tensor pg, torch::Tensor pbeta, torch::Tensor pending, bool per_channel);
// attention_decode.cu
torch::Tensor fa_decode(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor seqused,
                        double scale, int64_t left, int64_t right);
void kv_append(torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor k, torch::Tensor v,
               torch::Tensor seqlens);
// mxfp8.cu
std::vector<torch::Tensor> mx_quantize(torch::Tensor x, bool e5m2, bool dim0, bool dim1);
void mx_gemm(torch::Tensor a, torch::Tensor sa, bool a_e5m2, torch::Tensor b, torch::Tensor sb, bool b_e5m2,
             torch::Tensor d, bool accumulate);
// gemm_skinny.cu
void gemm_skinny(torch::Tensor a, torch::Tensor w, torch::Tensor d);
// ngram.cu (fused hashed n-gram embedding)
std::vector<torch::Tensor> ngram_embed_fwd(torch::Tensor tokens, std::vector<torch::Tensor> tables,
                                           std::vector<int64_t> orders, int64_t context);
void ngram_embed_bwd(torch::Tensor rows, torch::Tensor dout, std::vector<torch::Tensor> grads);
std::vector<torch::Tensor> ngram_embed_fwd_shard(torch::Tensor tokens, torch::Tensor bases, int64_t order_stride,
                                                 int64_t rows_per_rank, int64_t buckets, int64_t dim,
                                                 std::vector<int64_t> orders, int64_t context);
void ngram_embed_bwd_shard(torch::Tensor rows, torch::Tensor dout, torch::Tensor bases, int64_t order_stride,
                           int64_t rows_per_rank, int64_t buckets);
void shard_sumsq(torch::Tensor g, torch::Tensor partial);
void mx_quantize_into(torch::Tensor x, bool e5m2, torch::Tensor q0, torch::Tensor s0, torch::Tensor q1,
                      torch::Tensor s1);
void mx_shard_gather(torch::Tensor bases, int64_t R, int64_t K, int64_t N, torch::Tensor q0, torch::Tensor s0,
                     torch::Tensor q1, torch::Tensor s1);
void shard_adamw(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr, double wd, double b1,
                 double b2, double eps, int64_t step, torch::Tensor partial_ptrs, int64_t world, double max_norm);
// ngram.cu
torch::Tensor ngram_stage(torch::Tensor ids, torch::Tensor W, torch::Tensor M, torch::Tensor V, torch::Tensor last,
                          int64_t step, double lr, double wd, double b1, double b2, double eps, bool rowwise,
                          bool catch_up, bool write_back);
void ngram_adam(torch::Tensor ids, torch::Tensor grad, torch::Tensor W, torch::Tensor M, torch::Tensor V,
                torch::Tensor last, int64_t step, double lr, double wd, double b1, double b2, double eps, bool rowwise);
// comm.cu
void peer_barrier(torch::Tensor flag_ptrs, int64_t rank, int64_t world, int64_t epoch);
void dp_reduce_sumsq(torch::Tensor grad_ptrs, int64_t rank, int64_t world, torch::Tensor offsets,
                     torch::Tensor prefix, torch::Tensor partial, int64_t total);
void dp_adamw_allgather(torch::Tensor param_ptrs, torch::Tensor grad_ptrs, int64_t rank, int64_t world,
                        torch::Tensor offsets, torch::Tensor prefix, torch::Tensor wd, torch::Tensor lr,
                        torch::Tensor m, torch::Tensor v, double b1, double b2, double eps, int64_t step,
                        torch::Tensor partial_ptrs, double extra_sq, double max_norm, torch::Tensor norm_out,
                        int64_t total);
void dp_muon_prepare(torch::Tensor grad_ptrs, int64_t rank, int64_t world, torch::Tensor offs, int64_t numel,
                     torch::Tensor mom, double mu, bool nesterov, torch::Tensor out, torch::Tensor partial_ptrs,
                     double extra_sq, double max_norm);
void dp_muon_apply_allgather(torch::Tensor param_ptrs, int64_t rank, int64_t world, torch::Tensor offs,
                             int64_t numel, double decay, double step_scale, torch::Tensor orth);
}  // namespace mykb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "myk_llm_b200 sm_100a kernels";
  m.def("take_status", &mykb::take_status, "read and clear the device status word");
  m.def("gemm", &mykb::gemm, "tcgen05 bf16 GEMM");
  m.def("gemm_gather", &mykb::gemm_gather, "tcgen05 bf16 GEMM with the all-gather of its sharded weight fused in");
  m.def("shard_gather", &mykb::shard_gather, "all-gather of a row-sharded bf16 weight over peer memory");
  m.def("rmsnorm_fwd", &mykb::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &mykb::rmsnorm_bwd);
  m.def("gated_rmsnorm_fwd", &mykb::gated_rmsnorm_fwd);
  m.def("gated_rmsnorm_bwd", &mykb::gated_rmsnorm_bwd);
  m.def("swiglu_fwd", &mykb::swiglu_fwd);
  m.def("swiglu_bwd", &mykb::swiglu_bwd);
  m.def("rope", &mykb::rope);
  m.def("rope_qkv_fwd", &mykb::rope_qkv_fwd);
  m.def("rope_qkv_bwd", &mykb::rope_qkv_bwd);
  m.def("split_cols", &mykb::split_cols);
  m.def("cast_bf16", &mykb::cast_bf16, "fp32 -> bf16 copy (round to nearest even)");
  m.def("fp8_quant_rows", &mykb::fp8_quant_rows);
  m.def("fp8_quant_tensor", &mykb::fp8_quant_tensor);
  m.def("fp8_quant_cols_t", &mykb::fp8_quant_cols_t);
  m.def("embedding_fwd", &mykb::embedding_fwd);
  m.def("embedding_bwd", &mykb::embedding_bwd);
  m.def("ce_fwd_grad", &mykb::ce_fwd_grad);
  m.def("adamw_step", &mykb::adamw_step);
  m.def("muon_prepare", &mykb::muon_prepare);
  m.def("muon_apply", &mykb::muon_apply);
  m.def("frob_normalize_", &mykb::frob_normalize_);
  m.def("fa_fwd", &mykb::fa_fwd);
  m.def("fa_bwd", &mykb::fa_bwd);
  m.def("conv1d_fwd", &mykb::conv1d_fwd);
  m.def("conv1d_bwd", &mykb::conv1d_bwd);
  m.def("gdn_chunk_fwd", &mykb::gdn_chunk_fwd_entry);
  m.def("gdn_chunk_bwd", &mykb::gdn_chunk_bwd);
  m.def("gdn_recurrent", &mykb::gdn_recurrent);
  m.def("gdn_spec_window", &mykb::gdn_spec_window);
  m.def("ngram_stage", &mykb::ngram_stage);
  m.def("ngram_embed_fwd", &mykb::ngram_embed_fwd, "hashed n-gram embedding: hash, gather and sum in one kernel");
  m.def("ngram_embed_fwd_shard", &mykb::ngram_embed_fwd_shard,
        "hashed n-gram embedding over row-sharded tables (peer loads from the owners' shards)");
  m.def("ngram_embed_bwd_shard", &mykb::ngram_embed_bwd_shard,
        "hashed n-gram embedding gradient added into the owners' gradient shards (peer reductions)");
  m.def("shard_sumsq", &mykb::shard_sumsq, "squared norm of an fp32 buffer added into a partial norm");
  m.def("mx_quantize_into", &mykb::mx_quantize_into, "MXFP8 quantisation (both copies) into given buffers");
  m.def("mx_shard_gather", &mykb::mx_shard_gather,
        "fp8 all-gather of a row-sharded MXFP8 weight from every rank's quantised shard (peer loads)");
  m.def("shard_adamw", &mykb::shard_adamw, "AdamW over a local shard with the global clip coefficient; zeroes the gradient");
  m.def("ngram_embed_bwd", &mykb::ngram_embed_bwd, "hashed n-gram embedding backward: scatter-add per order");
  m.def("gemm_skinny", &mykb::gemm_skinny);
  m.def("mx_quantize", &mykb::mx_quantize);
  m.def("mx_gemm", &mykb::mx_gemm);
  m.def("fp8_scaled_gemm", &mykb::fp8_scaled_gemm, "per-tensor / per-row scaled float8 GEMM on tcgen05");
  m.def("fa_decode", &mykb::fa_decode);
  m.def("kv_append", &mykb::kv_append);
  m.def("ngram_adam", &mykb::ngram_adam);
  m.def("peer_barrier", &mykb::peer_barrier);
  m.def("dp_reduce_sumsq", &mykb::dp_reduce_sumsq);
  m.def("dp_reduce_sumsq_multimem", &mykb::dp_reduce_sumsq_multimem,
        "gradient reduce-scatter + squared norm through NVSwitch multicast (multimem.ld_reduce)");
  m.def("dp_adamw_allgather", &mykb::dp_adamw_allgather);
  m.def("dp_muon_prepare", &mykb::dp_muon_prepare);
  m.def("dp_muon_apply_allgather", &mykb::dp_muon_apply_allgather);
  m.def("dp_muon_apply_shards", &mykb::dp_muon_apply_shards);
  m.def("cast_ranges_bf16", &mykb::cast_ranges_bf16);
}
