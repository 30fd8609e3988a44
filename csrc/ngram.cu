// Lazy (sparse) Adam for the hashed n-gram tables: the rows a step touches are caught up
// and gathered in place (ngram_stage), and after backward Adam is applied to those rows
// in place (ngram_adam).  No compact copies of the moments are made: each kernel reads
// and writes the table rows directly, so a step moves 3 x rows x dim floats each way.
//
// The tables may live in device memory or in pinned host memory; for the latter the
// kernels address the host rows through their mapped device pointers (the same code
// path, so both placements give identical results).
//
// Catch-up (rows skipped for k steps get the k zero-gradient AdamW updates in closed
// form): w <- d^k (w - lr b m / (sqrt(v) + eps) * q (1 - q^k) / (1 - q)), q = beta1 /
// sqrt(beta2) / d, d = 1 - lr wd, b = sqrt(1 - beta2^(s-1)) / (1 - beta1^(s-1));
// m <- beta1^k m, v <- beta2^k v.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "ngram_hash.cuh"

namespace mykb {

struct NgramHyper {
  float lr, wd, b1, b2, eps;
  int step;
  bool rowwise;
};

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
  return t;
}

// One block per staged row.  catch_up: bring the row to the start of `step`; write_back:
// store the caught-up row into the tables (training) or only into `out` (reads).
__global__ void ngram_stage_kernel(const int64_t* __restrict__ ids, float* W, float* M, float* V,
                                   const int* __restrict__ last, float* __restrict__ out, int dim, NgramHyper hp,
                                   bool catch_up, bool write_back) {
  const int64_t id = ids[blockIdx.x];
  float* w = W + id * dim;
  float* o = out + (int64_t)blockIdx.x * dim;
  const int step = hp.step;
  if (!catch_up || step <= 1) {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) o[i] = w[i];
    return;
  }
  const float decay = 1.f - hp.lr * hp.wd;
  const float k = (float)max(step - 1 - last[id], 0);
  const float q = hp.b1 / sqrtf(hp.b2) / decay;
  const float drift = q * (1.f - powf(q, k)) / (1.f - q);
  const float bias = sqrtf(1.f - powf(hp.b2, (float)(step - 1))) / (1.f - powf(hp.b1, (float)(step - 1)));
  const float coef = drift * hp.lr * bias;
  const float dk = hp.wd != 0.f ? powf(decay, k) : 1.f;
  const float m1 = powf(hp.b1, k), v1 = powf(hp.b2, k);
  float* m = M + id * dim;
  if (hp.rowwise) {
    const float vr = V[id];
    const float den = sqrtf(vr) + hp.eps;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
      const float nw = (w[i] - coef * m[i] / den) * dk;
      o[i] = nw;
      if (write_back) {
        w[i] = nw;
        m[i] *= m1;
      }
    }
    __syncthreads();
    if (write_back && threadIdx.x == 0) V[id] = vr * v1;
  } else {
    float* v = V + id * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
      const float nw = (w[i] - coef * m[i] / (sqrtf(v[i]) + hp.eps)) * dk;
      o[i] = nw;
      if (write_back) {
        w[i] = nw;
        m[i] *= m1;
        v[i] *= v1;
      }
    }
  }
}

// AdamW (torch.optim.AdamW's rule, bias correction by the global step) on the staged
// rows with their compact gradients, in place; stamps last_step.
__global__ void ngram_adam_kernel(const int64_t* __restrict__ ids, const float* __restrict__ grad, float* W, float* M,
                                  float* V, int* last, int dim, NgramHyper hp) {
  __shared__ float red[32];
  const int64_t id = ids[blockIdx.x];
  const float* g = grad + (int64_t)blockIdx.x * dim;
  float* w = W + id * dim;
  float* m = M + id * dim;
  const float bias1 = 1.f - powf(hp.b1, (float)hp.step);
  const float sb2 = sqrtf(1.f - powf(hp.b2, (float)hp.step));
  const float dec = 1.f - hp.lr * hp.wd;
  const float step_size = hp.lr / bias1;
  if (hp.rowwise) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += g[i] * g[i];
    ss = block_sum(ss, red);
    const float vr = hp.b2 * V[id] + (1.f - hp.b2) * ss / dim;
    const float den = sqrtf(vr) / sb2 + hp.eps;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
      const float mi = m[i] + (1.f - hp.b1) * (g[i] - m[i]);
      m[i] = mi;
      w[i] = w[i] * dec - step_size * mi / den;
    }
    __syncthreads();
    if (threadIdx.x == 0) V[id] = vr;
  } else {
    float* v = V + id * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
      const float mi = m[i] + (1.f - hp.b1) * (g[i] - m[i]);
      const float vi = hp.b2 * v[i] + (1.f - hp.b2) * g[i] * g[i];
      m[i] = mi;
      v[i] = vi;
      w[i] = w[i] * dec - step_size * mi / (sqrtf(vi) / sb2 + hp.eps);
    }
  }
  if (threadIdx.x == 0) last[id] = hp.step;
}

// Device-addressable pointer of a tensor in device memory or in pinned host memory.
static void* device_view(const torch::Tensor& t) {
  if (t.is_cuda()) return t.data_ptr();
  TORCH_CHECK(t.is_pinned(), "ngram tables: host tensors must be pinned");
  void* dptr = nullptr;
  C10_CUDA_CHECK(cudaHostGetDevicePointer(&dptr, t.data_ptr(), 0));
  return dptr;
}

static NgramHyper hyper(double lr, double wd, double b1, double b2, double eps, int64_t step, bool rowwise) {
  return NgramHyper{(float)lr, (float)wd, (float)b1, (float)b2, (float)eps, (int)step, rowwise};
}

// ids (n,) int64 on the device; tables (rows, dim) fp32, moments, last_step int32.
torch::Tensor ngram_stage(torch::Tensor ids, torch::Tensor W, torch::Tensor M, torch::Tensor V, torch::Tensor last,
                          int64_t step, double lr, double wd, double b1, double b2, double eps, bool rowwise,
                          bool catch_up, bool write_back) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong, "ngram_stage: int64 ids on the device");
  TORCH_CHECK(W.scalar_type() == at::kFloat && W.is_contiguous() && M.is_contiguous() && V.is_contiguous() &&
                  last.scalar_type() == at::kInt,
              "ngram_stage: contiguous fp32 tables and int32 last_step");
  c10::cuda::CUDAGuard guard(ids.device());
  const int dim = W.size(1);
  auto out = torch::empty({ids.numel(), dim}, ids.options().dtype(at::kFloat));
  if (ids.numel() == 0) return out;
  ngram_stage_kernel<<<ids.numel(), 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), (float*)device_view(W), (float*)device_view(M), (float*)device_view(V),
      (const int*)device_view(last), out.data_ptr<float>(), dim, hyper(lr, wd, b1, b2, eps, step, rowwise), catch_up,
      write_back);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void ngram_adam(torch::Tensor ids, torch::Tensor grad, torch::Tensor W, torch::Tensor M, torch::Tensor V,
                torch::Tensor last, int64_t step, double lr, double wd, double b1, double b2, double eps, bool rowwise) {
  TORCH_CHECK(ids.is_cuda() && grad.is_cuda() && grad.scalar_type() == at::kFloat && grad.is_contiguous(),
              "ngram_adam: fp32 contiguous compact gradients on the device");
  c10::cuda::CUDAGuard guard(ids.device());
  const int dim = W.size(1);
  if (ids.numel() == 0) return;
  ngram_adam_kernel<<<ids.numel(), 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), grad.data_ptr<float>(), (float*)device_view(W), (float*)device_view(M),
      (float*)device_view(V), (int*)device_view(last), dim, hyper(lr, wd, b1, b2, eps, step, rowwise));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------------
// Hashed n-gram embedding, forward and backward in one kernel each.
//
// Row ids: for each order n (table k) and position t, the rolling hash of the n tokens
// ending at t (tokens[t], tokens[t-1], ...; missing left context is the sentinel id):
//   h = n;  for o in 0..n-1:  h = h * M[o % 4] + tok[t - o] + 1;  h ^= h >> 29  (wrapping
//   int64, arithmetic shift);  row = (h mod buckets, in [0, buckets)) + k * buckets.
// This is the bucket function of the reference model, so checkpoints' n-gram tables are
// addressed identically.  The forward writes the sum over orders of the rows (fp32) and
// the row ids (for the backward and for lazy tables); the backward scatter-adds the output
// gradient into every order's gradient rows.
// ------------------------------------------------------------------------------------
constexpr int kNgramMaxOrders = 8;

struct NgramTables {
  const float* table[kNgramMaxOrders];
  float* grad[kNgramMaxOrders];
  int order[kNgramMaxOrders];
  int k;
};

// One warp per position: lane 0..k-1 hash one order each, then the warp sums the rows with
// 16-byte loads.  tokens: (batch, context + seq) with `context` columns of left context.
__global__ void __launch_bounds__(256)
ngram_embed_fwd_kernel(const int64_t* __restrict__ tokens, int64_t batch, int64_t seq, int context, int64_t buckets,
                       NgramTables t, int dim, float* __restrict__ out, int64_t* __restrict__ rows) {
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
    const float4* src[kNgramMaxOrders];
#pragma unroll
    for (int j = 0; j < kNgramMaxOrders; ++j) {  // every lane takes part in every shuffle
      const int64_t r = __shfl_sync(0xffffffff, my, j < t.k ? j : 0);
      src[j] = j < t.k ? reinterpret_cast<const float4*>(t.table[j] + r * dim) : nullptr;
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

__global__ void __launch_bounds__(256)
ngram_embed_bwd_kernel(const int64_t* __restrict__ rows, int64_t n, int64_t buckets, NgramTables t, int dim,
                       const float* __restrict__ dout) {
  const int64_t total = n * dim;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pos = i / dim;
    const int c = (int)(i - pos * dim);
    const float g = dout[i];
    for (int j = 0; j < t.k; ++j) {
      const int64_t r = rows[(int64_t)j * n + pos] - j * buckets;
      atomicAdd(t.grad[j] + r * dim + c, g);
    }
  }
}

static NgramTables ngram_tables(const std::vector<torch::Tensor>& tabs, const std::vector<int64_t>& orders) {
  TORCH_CHECK(!tabs.empty() && tabs.size() == orders.size() && (int)tabs.size() <= kNgramMaxOrders,
              "ngram_embed: one table per order, at most 8");
  NgramTables t{};
  t.k = (int)tabs.size();
  for (int j = 0; j < t.k; ++j) {
    TORCH_CHECK(tabs[j].scalar_type() == at::kFloat && tabs[j].is_contiguous() && tabs[j].dim() == 2 &&
                    tabs[j].sizes() == tabs[0].sizes(),
                "ngram_embed: fp32 contiguous tables of one shape");
    t.table[j] = tabs[j].data_ptr<float>();
    t.order[j] = (int)orders[j];
    TORCH_CHECK(orders[j] >= 1 && orders[j] <= 32, "ngram_embed: order out of range");
  }
  return t;
}

// tokens: (batch, context + seq) int64.  Returns (batch * seq, dim) fp32 sums and the
// (orders, batch * seq) int64 stacked row ids.
std::vector<torch::Tensor> ngram_embed_fwd(torch::Tensor tokens, std::vector<torch::Tensor> tables,
                                           std::vector<int64_t> orders, int64_t context) {
  c10::cuda::CUDAGuard guard(tokens.device());
  TORCH_CHECK(tokens.scalar_type() == at::kLong && tokens.dim() == 2 && tokens.is_contiguous(),
              "ngram_embed: (batch, context + seq) int64 tokens");
  NgramTables t = ngram_tables(tables, orders);
  const int64_t batch = tokens.size(0), seq = tokens.size(1) - context;
  for (int j = 0; j < t.k; ++j) TORCH_CHECK(orders[j] - 1 <= context, "ngram_embed: context shorter than an order");
  const int dim = tables[0].size(1);
  TORCH_CHECK(dim % 4 == 0, "ngram_embed: dim must be a multiple of 4");
  const int64_t buckets = tables[0].size(0), n = batch * seq;
  auto out = torch::empty({n, dim}, tables[0].options());
  auto rows = torch::empty({t.k, n}, tokens.options());
  if (n == 0) return {out, rows};
  const int64_t warps = n;
  const int blocks = (int)std::min<int64_t>((warps * 32 + 255) / 256, 65535);
  ngram_embed_fwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      tokens.data_ptr<int64_t>(), batch, seq, (int)context, buckets, t, dim, out.data_ptr<float>(),
      rows.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {out, rows};
}

// Scatter-add of dout (n, dim) fp32 into every order's fp32 gradient table.
void ngram_embed_bwd(torch::Tensor rows, torch::Tensor dout, std::vector<torch::Tensor> grads) {
  c10::cuda::CUDAGuard guard(dout.device());
  TORCH_CHECK(dout.scalar_type() == at::kFloat && dout.is_contiguous(), "ngram_embed_bwd: fp32 contiguous dout");
  std::vector<int64_t> orders(grads.size(), 1);
  NgramTables t = ngram_tables(grads, orders);
  for (int j = 0; j < t.k; ++j) t.grad[j] = grads[j].data_ptr<float>();
  const int64_t n = dout.size(0);
  const int dim = dout.size(1);
  if (n == 0) return;
  const int64_t total = n * dim;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  ngram_embed_bwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      rows.data_ptr<int64_t>(), n, grads[0].size(0), t, dim, dout.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
