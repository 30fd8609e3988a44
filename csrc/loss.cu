// Cross-entropy + z-loss over a chunk of bf16 logits, producing the logits gradient in
// place (sm_100a).  One CTA per row:
//   pass 1: running max / rescaled sum over the row (online log-sum-exp, fp32)
//   pass 2: logits[j] <- (softmax_j * (1 + 2 z lse) - [j == target]) * scale
// Rows whose target is ignore_index get a zero gradient.  ce_sum += lse - logit[target] and
// z_sum += lse^2 over supervised rows (one atomic per CTA).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace mykb {

constexpr int kCeThreads = 512;

struct MaxSum {
  float m, s;
};

__device__ __forceinline__ MaxSum combine(MaxSum a, MaxSum b) {
  float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f};
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

__global__ void __launch_bounds__(kCeThreads)
ce_kernel(__nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ targets, int V, float scale, float z_coef,
          int64_t ignore_index, float* __restrict__ ce_sum, float* __restrict__ z_sum) {
  const int64_t row = blockIdx.x;
  __nv_bfloat16* lg = logits + row * V;
  const int64_t tgt = targets[row];
  const bool valid = tgt != ignore_index && tgt >= 0 && tgt < V;
  // pass 1
  MaxSum ms{-INFINITY, 0.f};
  const int nvec = (V % 8 == 0) ? V / 8 : 0;  // rows stay 16-byte aligned only when V % 8 == 0
  for (int i = threadIdx.x; i < nvec; i += kCeThreads) {
    uint4 raw = reinterpret_cast<const uint4*>(lg)[i];
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(p[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
    float m = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) m = fmaxf(m, v[j]);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += __expf(v[j] - m);
    ms = combine(ms, {m, s});
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += kCeThreads) ms = combine(ms, {__bfloat162float(lg[i]), 1.f});
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum other{__shfl_xor_sync(0xffffffff, ms.m, o), __shfl_xor_sync(0xffffffff, ms.s, o)};
    ms = combine(ms, other);
  }
  __shared__ MaxSum red[kCeThreads / 32];
  __shared__ float s_lse;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ms;
  __syncthreads();
  if (threadIdx.x == 0) {
    MaxSum t = red[0];
    for (int w = 1; w < kCeThreads / 32; ++w) t = combine(t, red[w]);
    s_lse = t.m + logf(t.s);
  }
  __syncthreads();
  const float lse = s_lse;
  if (threadIdx.x == 0 && valid) {
    const float tl = __bfloat162float(lg[tgt]);
    atomicAdd(ce_sum, lse - tl);
    atomicAdd(z_sum, lse * lse);
  }
  __syncthreads();  // the target logit is read before pass 2 overwrites it
  // pass 2
  const float factor = valid ? scale * (1.f + 2.f * z_coef * lse) : 0.f;
  for (int i = threadIdx.x; i < nvec; i += kCeThreads) {
    uint4 raw = reinterpret_cast<const uint4*>(lg)[i];
    __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(p[j]);
      float g0 = __expf(f.x - lse) * factor;
      float g1 = __expf(f.y - lse) * factor;
      const int c = i * 8 + 2 * j;
      if (valid && c == tgt) g0 -= scale;
      if (valid && c + 1 == tgt) g1 -= scale;
      p[j] = __floats2bfloat162_rn(g0, g1);
    }
    reinterpret_cast<uint4*>(lg)[i] = raw;
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += kCeThreads) {
    float g = __expf(__bfloat162float(lg[i]) - lse) * factor;
    if (valid && i == tgt) g -= scale;
    lg[i] = __float2bfloat16(g);
  }
}

void ce_fwd_grad(torch::Tensor logits, torch::Tensor targets, double scale, double z_coef, int64_t ignore_index,
                 torch::Tensor ce_sum, torch::Tensor z_sum) {
  c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.is_contiguous(), "ce: contiguous bf16 logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.numel() == logits.size(0), "ce: int64 targets per row");
  const int rows = logits.size(0), V = logits.size(1);
  if (rows == 0) return;
  ce_kernel<<<rows, kCeThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      (__nv_bfloat16*)logits.data_ptr(), targets.data_ptr<int64_t>(), V, (float)scale, (float)z_coef, ignore_index,
      ce_sum.data_ptr<float>(), z_sum.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
