// Row-sharded hashed n-gram tables over NVLink peer memory (one process per GPU, torch
// symmetric memory).  Rank r owns rows [r R, (r + 1) R) of every order's table (fp32
// master, gradient, AdamW state); no rank holds a full table.
//
//   ngram_embed_fwd_shard  hash every order of every position, read the rows from their
//                          owners' shards (16-byte peer loads), sum them
//   ngram_embed_bwd_shard  add each position's output gradient into the owners' gradient
//                          rows (16-byte vector reductions on peer memory)
//   shard_sumsq            squared norm of this rank's gradient shard into the partial norm
//   shard_adamw            clip coefficient from every rank's partial norm, AdamW on this
//                          rank's rows, gradient rows zeroed for the next step
//
// So a step moves only the rows its tokens touch across NVLink (about 2 x tokens x orders
// x dim x 4 bytes), instead of reducing and gathering the whole tables.  The reference
// keeps the tables in FSDP2's root unit and all-gathers / reduce-scatters them in full
// (src/myk_llm/train/distributed.py:131).  Rows are addressed by the shared bucket function
// of ngram_hash.cuh.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "ngram_hash.cuh"

namespace mykb {

constexpr int kShardMaxOrders = 8;
constexpr int kShardMaxWorld = 8;

struct ShardTables {
  int64_t base[kShardMaxWorld];  // rank r's shard of order j starts at base[r] + j * order_stride (bytes)
  int64_t order_stride;          // bytes between consecutive orders' shards inside one rank's buffer
  int64_t rows_per_rank;
  int order[kShardMaxOrders];
  int k, world;
  __device__ __forceinline__ float* row(int j, int64_t r, int dim) const {
    const int owner = (int)(r / rows_per_rank);
    const int64_t local = r - (int64_t)owner * rows_per_rank;
    return reinterpret_cast<float*>(base[owner] + j * order_stride) + local * dim;
  }
};

// One warp per position: lanes 0..k-1 hash one order each; the warp sums the rows.
__global__ void __launch_bounds__(256)
ngram_embed_fwd_shard_kernel(const int64_t* __restrict__ tokens, int64_t batch, int64_t seq, int context,
                             int64_t buckets, ShardTables t, int dim, float* __restrict__ out,
                             int64_t* __restrict__ rows) {
  const int lane = threadIdx.x & 31;
  const int64_t n = batch * seq;
  for (int64_t pos = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; pos < n;
       pos += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t b = pos / seq, s = pos - b * seq;
    const int64_t* tok = tokens + b * (seq + context) + context + s;
    int64_t my = 0;
    if (lane < t.k) {
      my = ngram_bucket(tok, t.order[lane], buckets);
      rows[(int64_t)lane * n + pos] = my + lane * buckets;
    }
    const float4* src[kShardMaxOrders];
#pragma unroll
    for (int j = 0; j < kShardMaxOrders; ++j) {
      const int64_t r = __shfl_sync(0xffffffffu, my, j < t.k ? j : 0);
      src[j] = j < t.k ? reinterpret_cast<const float4*>(t.row(j, r, dim)) : nullptr;
    }
    float4* o4 = reinterpret_cast<float4*>(out + pos * dim);
    for (int c = lane; c < dim / 4; c += 32) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < t.k; ++j) {
        const float4 v = src[j][c];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      o4[c] = acc;
    }
  }
}

// One warp per position: the position's gradient row is added into every order's row of
// its owner with 16-byte reductions (performed at the owner's memory).
__global__ void __launch_bounds__(256)
ngram_embed_bwd_shard_kernel(const int64_t* __restrict__ rows, int64_t n, int64_t buckets, ShardTables g, int dim,
                             const float* __restrict__ dout) {
  const int lane = threadIdx.x & 31;
  for (int64_t pos = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; pos < n;
       pos += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const float4* d4 = reinterpret_cast<const float4*>(dout + pos * dim);
    for (int j = 0; j < g.k; ++j) {
      const int64_t r = rows[(int64_t)j * n + pos] - j * buckets;
      float4* dst = reinterpret_cast<float4*>(g.row(j, r, dim));
      for (int c = lane; c < dim / 4; c += 32) atomicAdd(dst + c, d4[c]);
    }
  }
}

__global__ void __launch_bounds__(256) shard_sumsq_kernel(const float4* __restrict__ g, int64_t n4,
                                                          float* __restrict__ partial) {
  __shared__ float red[8];
  float s = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = g[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(partial, t);
  }
}

// AdamW (torch.optim.AdamW, decoupled decay) over this rank's rows; the clip coefficient
// comes from every rank's partial squared norm (partial_ptrs[r] -> rank r's float).  The
// gradient rows are zeroed after they are read.
__global__ void __launch_bounds__(256)
shard_adamw_kernel(float4* __restrict__ p, float4* __restrict__ g, float4* __restrict__ m, float4* __restrict__ v,
                   int64_t n4, float lr, float wd, float b1, float b2, float eps, float bc1, float bc2_sqrt,
                   const int64_t* __restrict__ partial_ptrs, int world, float max_norm) {
  float sq = 0.f;
  for (int r = 0; r < world; ++r) sq += *reinterpret_cast<const volatile float*>(partial_ptrs[r]);
  const float coef = max_norm > 0.f ? fminf(1.f, max_norm / (sqrtf(sq) + 1e-6f)) : 1.f;
  const float decay = 1.f - lr * wd, step = lr / bc1;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 pp = p[i], gg = g[i], mm = m[i], vv = v[i];
    float* pa = reinterpret_cast<float*>(&pp);
    const float* ga = reinterpret_cast<const float*>(&gg);
    float* ma = reinterpret_cast<float*>(&mm);
    float* va = reinterpret_cast<float*>(&vv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gj = ga[e] * coef;
      ma[e] = ma[e] + (1.f - b1) * (gj - ma[e]);
      va[e] = b2 * va[e] + (1.f - b2) * gj * gj;
      pa[e] = pa[e] * decay - step * ma[e] / (sqrtf(va[e]) / bc2_sqrt + eps);
    }
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    g[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

static ShardTables shard_tables(const torch::Tensor& bases, int64_t order_stride_bytes, int64_t rows_per_rank,
                                const std::vector<int64_t>& orders) {
  TORCH_CHECK(bases.scalar_type() == at::kLong && bases.numel() >= 1 && bases.numel() <= kShardMaxWorld,
              "ngram shard: one int64 base address per rank, at most ", kShardMaxWorld);
  TORCH_CHECK(!orders.empty() && (int)orders.size() <= kShardMaxOrders, "ngram shard: 1..8 orders");
  auto b = bases.to(at::kCPU);
  ShardTables t{};
  t.world = (int)b.numel();
  for (int r = 0; r < t.world; ++r) {
    t.base[r] = b.data_ptr<int64_t>()[r];
    TORCH_CHECK(t.base[r] % 16 == 0, "ngram shard: 16-byte aligned shards");
  }
  TORCH_CHECK(order_stride_bytes % 16 == 0 && rows_per_rank > 0, "ngram shard: aligned order stride");
  t.order_stride = order_stride_bytes;
  t.rows_per_rank = rows_per_rank;
  t.k = (int)orders.size();
  for (int j = 0; j < t.k; ++j) {
    TORCH_CHECK(orders[j] >= 1 && orders[j] <= 32, "ngram shard: order out of range");
    t.order[j] = (int)orders[j];
  }
  return t;
}

// tokens (batch, context + seq) int64; bases: every rank's table buffer; returns the
// (batch * seq, dim) sums and the (orders, batch * seq) stacked row ids.
std::vector<torch::Tensor> ngram_embed_fwd_shard(torch::Tensor tokens, torch::Tensor bases, int64_t order_stride,
                                                 int64_t rows_per_rank, int64_t buckets, int64_t dim,
                                                 std::vector<int64_t> orders, int64_t context) {
  c10::cuda::CUDAGuard guard(tokens.device());
  TORCH_CHECK(tokens.is_cuda() && tokens.scalar_type() == at::kLong && tokens.dim() == 2 && tokens.is_contiguous(),
              "ngram_embed_fwd_shard: (batch, context + seq) int64 tokens");
  TORCH_CHECK(dim % 4 == 0, "ngram_embed_fwd_shard: dim must be a multiple of 4");
  ShardTables t = shard_tables(bases, order_stride, rows_per_rank, orders);
  TORCH_CHECK(rows_per_rank * t.world >= buckets, "ngram_embed_fwd_shard: shards do not cover the table");
  for (int j = 0; j < t.k; ++j) TORCH_CHECK(orders[j] - 1 <= context, "ngram_embed_fwd_shard: context too short");
  const int64_t batch = tokens.size(0), seq = tokens.size(1) - context, n = batch * seq;
  auto out = torch::empty({n, dim}, tokens.options().dtype(at::kFloat));
  auto rows = torch::empty({t.k, n}, tokens.options());
  if (n == 0) return {out, rows};
  const int blocks = (int)std::min<int64_t>((n * 32 + 255) / 256, 65535);
  ngram_embed_fwd_shard_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      tokens.data_ptr<int64_t>(), batch, seq, (int)context, buckets, t, (int)dim, out.data_ptr<float>(),
      rows.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {out, rows};
}

void ngram_embed_bwd_shard(torch::Tensor rows, torch::Tensor dout, torch::Tensor bases, int64_t order_stride,
                           int64_t rows_per_rank, int64_t buckets) {
  c10::cuda::CUDAGuard guard(dout.device());
  TORCH_CHECK(dout.is_cuda() && dout.scalar_type() == at::kFloat && dout.is_contiguous() && dout.dim() == 2,
              "ngram_embed_bwd_shard: fp32 contiguous (n, dim) dout");
  TORCH_CHECK(rows.scalar_type() == at::kLong && rows.is_contiguous() && rows.dim() == 2 &&
                  rows.size(1) == dout.size(0),
              "ngram_embed_bwd_shard: (orders, n) int64 rows");
  std::vector<int64_t> orders(rows.size(0), 1);
  ShardTables t = shard_tables(bases, order_stride, rows_per_rank, orders);
  const int64_t n = dout.size(0);
  const int dim = (int)dout.size(1);
  TORCH_CHECK(dim % 4 == 0, "ngram_embed_bwd_shard: dim must be a multiple of 4");
  if (n == 0) return;
  const int blocks = (int)std::min<int64_t>((n * 32 + 255) / 256, 65535);
  ngram_embed_bwd_shard_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      rows.data_ptr<int64_t>(), n, buckets, t, dim, dout.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void shard_sumsq(torch::Tensor g, torch::Tensor partial) {
  c10::cuda::CUDAGuard guard(g.device());
  TORCH_CHECK(g.is_cuda() && g.scalar_type() == at::kFloat && g.is_contiguous() && g.numel() % 4 == 0,
              "shard_sumsq: fp32 contiguous, multiple of 4 elements");
  const int64_t n4 = g.numel() / 4;
  if (n4 == 0) return;
  const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
  shard_sumsq_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(g.data_ptr<float>()), n4, partial.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void shard_adamw(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr, double wd, double b1,
                 double b2, double eps, int64_t step, torch::Tensor partial_ptrs, int64_t world, double max_norm) {
  c10::cuda::CUDAGuard guard(p.device());
  for (const auto& t : {p, g, m, v})
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == p.numel() &&
                    (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
                "shard_adamw: aligned fp32 contiguous tensors of one size");
  TORCH_CHECK(p.numel() % 4 == 0, "shard_adamw: multiple of 4 elements");
  const int64_t n4 = p.numel() / 4;
  if (n4 == 0) return;
  const float bc1 = 1.f - std::pow((float)b1, (float)step);
  const float bc2s = std::sqrt(1.f - std::pow((float)b2, (float)step));
  const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
  shard_adamw_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<float4*>(p.data_ptr<float>()), reinterpret_cast<float4*>(g.data_ptr<float>()),
      reinterpret_cast<float4*>(m.data_ptr<float>()), reinterpret_cast<float4*>(v.data_ptr<float>()), n4, (float)lr,
      (float)wd, (float)b1, (float)b2, (float)eps, bc1, bc2s, partial_ptrs.data_ptr<int64_t>(), (int)world,
      (float)max_norm);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
