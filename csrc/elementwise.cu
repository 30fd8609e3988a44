// Elementwise kernels (sm_100a): SwiGLU forward/backward, interleaved-pair RoPE (also fused
// over the QKV projection), token
// embedding gather / scatter-add.  All use 16-byte vector accesses on bf16 data.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace mykb {

struct alignas(16) bf16x8 {
  __nv_bfloat162 v[4];
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

// gu (rows, 2F): gate = gu[:, :F], up = gu[:, F:];  a = silu(gate) * up.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ a, int64_t rows,
                                  int F) {
  const int vec_per_row = F / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int c = (int)(i % vec_per_row) * 8;
    bf16x8 g = *reinterpret_cast<const bf16x8*>(gu + r * 2 * F + c);
    bf16x8 u = *reinterpret_cast<const bf16x8*>(gu + r * 2 * F + F + c);
    bf16x8 o;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 gf = __bfloat1622float2(g.v[j]);
      float2 uf = __bfloat1622float2(u.v[j]);
      o.v[j] = __floats2bfloat162_rn(silu_f(gf.x) * uf.x, silu_f(gf.y) * uf.y);
    }
    *reinterpret_cast<bf16x8*>(a + r * F + c) = o;
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ da, const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ dgu, int64_t rows, int F) {
  const int vec_per_row = F / 8;
  const int64_t total = rows * vec_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int c = (int)(i % vec_per_row) * 8;
    bf16x8 g = *reinterpret_cast<const bf16x8*>(gu + r * 2 * F + c);
    bf16x8 u = *reinterpret_cast<const bf16x8*>(gu + r * 2 * F + F + c);
    bf16x8 d = *reinterpret_cast<const bf16x8*>(da + r * F + c);
    bf16x8 dg, du;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 gf = __bfloat1622float2(g.v[j]);
      float2 uf = __bfloat1622float2(u.v[j]);
      float2 df = __bfloat1622float2(d.v[j]);
      float s0 = 1.f / (1.f + __expf(-gf.x)), s1 = 1.f / (1.f + __expf(-gf.y));
      float ds0 = s0 * (1.f + gf.x * (1.f - s0)), ds1 = s1 * (1.f + gf.y * (1.f - s1));
      dg.v[j] = __floats2bfloat162_rn(df.x * uf.x * ds0, df.y * uf.y * ds1);
      du.v[j] = __floats2bfloat162_rn(df.x * gf.x * s0, df.y * gf.y * s1);
    }
    *reinterpret_cast<bf16x8*>(dgu + r * 2 * F + c) = dg;
    *reinterpret_cast<bf16x8*>(dgu + r * 2 * F + F + c) = du;
  }
}

static int ew_grid(int64_t work, int threads) {
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t blocks = (work + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sms * 16));
}

torch::Tensor swiglu_fwd(torch::Tensor gu) {
  c10::cuda::CUDAGuard guard(gu.device());
  TORCH_CHECK(gu.scalar_type() == at::kBFloat16 && gu.is_contiguous(), "swiglu: contiguous bf16");
  const int F = gu.size(-1) / 2;
  TORCH_CHECK(F % 8 == 0, "swiglu: half width must be a multiple of 8");
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto a = torch::empty(sizes, gu.options());
  const int64_t rows = gu.numel() / (2 * F);
  if (rows == 0) return a;
  swiglu_fwd_kernel<<<ew_grid(rows * F / 8, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)a.data_ptr(), rows, F);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return a;
}

torch::Tensor swiglu_bwd(torch::Tensor da, torch::Tensor gu) {
  c10::cuda::CUDAGuard guard(gu.device());
  TORCH_CHECK(da.scalar_type() == at::kBFloat16 && da.is_contiguous(), "swiglu_bwd: contiguous bf16 grad");
  const int F = gu.size(-1) / 2;
  auto dgu = torch::empty_like(gu);
  const int64_t rows = gu.numel() / (2 * F);
  if (rows == 0) return dgu;
  swiglu_bwd_kernel<<<ew_grid(rows * F / 8, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)da.data_ptr(), (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)dgu.data_ptr(), rows,
      F);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dgu;
}

// ------------------------------------------------------------------------------ RoPE
// x (B, S, H, D) with arbitrary strides for B, S, H (unit stride along D); out is
// contiguous (B, S, H, D).  Pairs (2i, 2i+1) rotate by angle table[pos][2i].
// inverse=true applies the transpose rotation (the backward pass).
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            const int64_t* __restrict__ pos, int B, int S, int H, int D, int64_t sb, int64_t ss,
                            int64_t sh, int64_t table_len, bool inverse) {
  const int pairs = D / 2;
  const int64_t total = (int64_t)B * S * H * pairs;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(i % pairs);
    int64_t t = i / pairs;
    const int h = (int)(t % H);
    t /= H;
    const int s = (int)(t % S);
    const int b = (int)(t / S);
    int64_t ps = pos[(int64_t)b * S + s];
    ps = ps < 0 ? 0 : (ps >= table_len ? table_len - 1 : ps);
    const float c = cos_t[ps * D + 2 * p];
    const float sn = sin_t[ps * D + 2 * p];
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(x + b * sb + s * ss + h * sh + 2 * p);
    const float2 f = __bfloat1622float2(v);
    float o0, o1;
    if (!inverse) {
      o0 = f.x * c - f.y * sn;
      o1 = f.y * c + f.x * sn;
    } else {
      o0 = f.x * c + f.y * sn;
      o1 = f.y * c - f.x * sn;
    }
    *reinterpret_cast<__nv_bfloat162*>(y + (((int64_t)b * S + s) * H + h) * D + 2 * p) = __floats2bfloat162_rn(o0, o1);
  }
}

torch::Tensor rope(torch::Tensor x, torch::Tensor cos_t, torch::Tensor sin_t, torch::Tensor pos, bool inverse) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.dim() == 4 && x.stride(3) == 1 && x.scalar_type() == at::kBFloat16, "rope: bf16 (B,S,H,D), unit D stride");
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && cos_t.is_contiguous() && sin_t.is_contiguous(), "rope: fp32 tables");
  const int B = x.size(0), S = x.size(1), H = x.size(2), D = x.size(3);
  auto y = torch::empty({B, S, H, D}, x.options());
  const int64_t total = (int64_t)B * S * H * (D / 2);
  if (total == 0) return y;
  TORCH_CHECK(pos.is_contiguous() && pos.scalar_type() == at::kLong && pos.numel() == (int64_t)B * S, "rope: positions");
  rope_kernel<<<ew_grid(total, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), (__nv_bfloat16*)y.data_ptr(), cos_t.data_ptr<float>(),
      sin_t.data_ptr<float>(), pos.data_ptr<int64_t>(), B, S, H, D, x.stride(0), x.stride(1), x.stride(2),
      cos_t.size(0), inverse);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

// ------------------------------------------------------------------------ fused QKV RoPE
// Attention input in one pass.  Forward: rows of the QKV projection (q heads, then k heads,
// then v heads, row stride `rs` elements) -> rotated q (T, H, D), rotated k (T, KV, D) and
// v (T, KV, D), all contiguous.  Backward: dq, dk, dv -> the QKV gradient rows, with q / k
// rotated back.  Each thread moves one 16-byte vector (4 interleaved pairs); the cos / sin
// tables hold one fp32 value per element (pair values repeated), so a vector reads the
// 8 table entries at its own offset.
template <int D, bool BWD>
__global__ void rope_qkv_kernel(const __nv_bfloat16* __restrict__ src0, const __nv_bfloat16* __restrict__ src1,
                                const __nv_bfloat16* __restrict__ src2, __nv_bfloat16* __restrict__ dst0,
                                __nv_bfloat16* __restrict__ dst1, __nv_bfloat16* __restrict__ dst2,
                                const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                const int64_t* __restrict__ pos, uint32_t rows, int H, int KV, int64_t rs,
                                int64_t table_len) {
  constexpr int kVecPerHead = D / 8;
  const uint32_t vec_per_row = (uint32_t)(H + 2 * KV) * kVecPerHead;
  const uint64_t total = (uint64_t)rows * vec_per_row;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t t = (uint32_t)(i / vec_per_row);
    const uint32_t j = (uint32_t)(i - (uint64_t)t * vec_per_row);
    const int head = (int)(j / kVecPerHead);
    const int d0 = (int)(j % kVecPerHead) * 8;
    // source and destination of this vector
    const __nv_bfloat16* sp;
    __nv_bfloat16* dp;
    if (!BWD) {
      sp = src0 + (int64_t)t * rs + head * D + d0;
      if (head < H) dp = dst0 + ((int64_t)t * H + head) * D + d0;
      else if (head < H + KV) dp = dst1 + ((int64_t)t * KV + head - H) * D + d0;
      else dp = dst2 + ((int64_t)t * KV + head - H - KV) * D + d0;
    } else {
      if (head < H) sp = src0 + ((int64_t)t * H + head) * D + d0;
      else if (head < H + KV) sp = src1 + ((int64_t)t * KV + head - H) * D + d0;
      else sp = src2 + ((int64_t)t * KV + head - H - KV) * D + d0;
      dp = dst0 + (int64_t)t * rs + head * D + d0;
    }
    bf16x8 v = *reinterpret_cast<const bf16x8*>(sp);
    if (head < H + KV) {
      int64_t ps = pos[t];
      ps = ps < 0 ? 0 : (ps >= table_len ? table_len - 1 : ps);
      const float4 c0 = *reinterpret_cast<const float4*>(cos_t + ps * D + d0);
      const float4 c1 = *reinterpret_cast<const float4*>(cos_t + ps * D + d0 + 4);
      const float4 s0 = *reinterpret_cast<const float4*>(sin_t + ps * D + d0);
      const float4 s1 = *reinterpret_cast<const float4*>(sin_t + ps * D + d0 + 4);
      const float cs[4] = {c0.x, c0.z, c1.x, c1.z};
      const float sn[4] = {BWD ? -s0.x : s0.x, BWD ? -s0.z : s0.z, BWD ? -s1.x : s1.x, BWD ? -s1.z : s1.z};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(v.v[q]);
        v.v[q] = __floats2bfloat162_rn(f.x * cs[q] - f.y * sn[q], f.y * cs[q] + f.x * sn[q]);
      }
    }
    *reinterpret_cast<bf16x8*>(dp) = v;
  }
}

static void check_rope_tables(const torch::Tensor& cos_t, const torch::Tensor& sin_t, int D) {
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && cos_t.is_contiguous() && sin_t.is_contiguous() &&
                  cos_t.size(-1) == D && sin_t.sizes() == cos_t.sizes(),
              "rope_qkv: fp32 (positions, head_dim) tables");
}

template <bool BWD>
static void launch_rope_qkv(int D, const __nv_bfloat16* s0, const __nv_bfloat16* s1, const __nv_bfloat16* s2,
                            __nv_bfloat16* d0, __nv_bfloat16* d1, __nv_bfloat16* d2, const torch::Tensor& cos_t,
                            const torch::Tensor& sin_t, const torch::Tensor& pos, int64_t rows, int H, int KV,
                            int64_t rs) {
  const int64_t total = rows * (H + 2 * KV) * (D / 8);
  if (total == 0) return;
  TORCH_CHECK(rows < (int64_t)UINT32_MAX, "rope_qkv: too many rows");
  auto st = at::cuda::getCurrentCUDAStream();
  const unsigned grid = ew_grid(total, 256);
  if (D == 64)
    rope_qkv_kernel<64, BWD><<<grid, 256, 0, st>>>(s0, s1, s2, d0, d1, d2, cos_t.data_ptr<float>(),
                                                   sin_t.data_ptr<float>(), pos.data_ptr<int64_t>(), (uint32_t)rows,
                                                   H, KV, rs, cos_t.size(0));
  else if (D == 128)
    rope_qkv_kernel<128, BWD><<<grid, 256, 0, st>>>(s0, s1, s2, d0, d1, d2, cos_t.data_ptr<float>(),
                                                    sin_t.data_ptr<float>(), pos.data_ptr<int64_t>(), (uint32_t)rows,
                                                    H, KV, rs, cos_t.size(0));
  else
    TORCH_CHECK(false, "rope_qkv: head_dim 64 or 128");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// qkv (B, S, (H + 2 KV) D) bf16 with unit last stride -> [q (B,S,H,D), k (B,S,KV,D), v (B,S,KV,D)].
std::vector<torch::Tensor> rope_qkv_fwd(torch::Tensor qkv, torch::Tensor cos_t, torch::Tensor sin_t,
                                        torch::Tensor pos, int64_t H, int64_t KV) {
  c10::cuda::CUDAGuard guard(qkv.device());
  TORCH_CHECK(qkv.dim() == 3 && qkv.scalar_type() == at::kBFloat16 && qkv.stride(2) == 1 &&
                  qkv.stride(0) == qkv.size(1) * qkv.stride(1),
              "rope_qkv: bf16 (B, S, width) with unit last stride and uniformly strided rows");
  const int64_t B = qkv.size(0), S = qkv.size(1), D = qkv.size(2) / (H + 2 * KV);
  TORCH_CHECK(D * (H + 2 * KV) == qkv.size(2), "rope_qkv: width is not (H + 2 KV) * head_dim");
  TORCH_CHECK(qkv.stride(1) % 8 == 0 && reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0,
              "rope_qkv: rows must be 16-byte aligned");
  check_rope_tables(cos_t, sin_t, (int)D);
  TORCH_CHECK(pos.is_contiguous() && pos.scalar_type() == at::kLong && pos.numel() == B * S, "rope_qkv: positions");
  auto q = torch::empty({B, S, H, D}, qkv.options());
  auto k = torch::empty({B, S, KV, D}, qkv.options());
  auto v = torch::empty({B, S, KV, D}, qkv.options());
  auto bp = [](torch::Tensor& t) { return (__nv_bfloat16*)t.data_ptr(); };
  launch_rope_qkv<false>((int)D, (const __nv_bfloat16*)qkv.data_ptr(), nullptr, nullptr, bp(q), bp(k), bp(v), cos_t,
                         sin_t, pos, B * S, (int)H, (int)KV, qkv.stride(1));
  return {q, k, v};
}

// dq (B,S,H,D), dk, dv (B,S,KV,D) -> dqkv (B, S, (H + 2 KV) D), contiguous.
torch::Tensor rope_qkv_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor cos_t,
                           torch::Tensor sin_t, torch::Tensor pos) {
  c10::cuda::CUDAGuard guard(dq.device());
  dq = dq.contiguous();
  dk = dk.contiguous();
  dv = dv.contiguous();
  const int64_t B = dq.size(0), S = dq.size(1), H = dq.size(2), D = dq.size(3), KV = dk.size(2);
  TORCH_CHECK(dq.scalar_type() == at::kBFloat16 && dk.scalar_type() == at::kBFloat16 &&
                  dv.scalar_type() == at::kBFloat16 && dk.sizes() == dv.sizes(),
              "rope_qkv_bwd: bf16 gradients");
  check_rope_tables(cos_t, sin_t, (int)D);
  auto dqkv = torch::empty({B, S, (H + 2 * KV) * D}, dq.options());
  auto bp = [](const torch::Tensor& t) { return (__nv_bfloat16*)t.data_ptr(); };
  launch_rope_qkv<true>((int)D, bp(dq), bp(dk), bp(dv), bp(dqkv), nullptr, nullptr, cos_t, sin_t, pos, B * S, (int)H,
                        (int)KV, (H + 2 * KV) * D);
  return dqkv;
}

// ------------------------------------------------------------------------ column split
// x (rows, W) with unit last stride and row stride `rs` -> up to 4 contiguous outputs of
// widths w[i] (sum = W, each a multiple of 8): one 16-byte vector per thread.
struct SplitOut {
  __nv_bfloat16* ptr[4];
  int width[4];
  int n;
};

__global__ void split_cols_kernel(const __nv_bfloat16* __restrict__ x, int64_t rs, uint32_t rows, int W, SplitOut o) {
  const uint32_t vec_per_row = W / 8;
  const uint64_t total = (uint64_t)rows * vec_per_row;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t r = (uint32_t)(i / vec_per_row);
    int c = (int)(i - (uint64_t)r * vec_per_row) * 8;
    const bf16x8 v = *reinterpret_cast<const bf16x8*>(x + (int64_t)r * rs + c);
    int j = 0;
    while (j + 1 < o.n && c >= o.width[j]) c -= o.width[j++];
    *reinterpret_cast<bf16x8*>(o.ptr[j] + (int64_t)r * o.width[j] + c) = v;
  }
}

std::vector<torch::Tensor> split_cols(torch::Tensor x, std::vector<int64_t> widths) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 && x.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "split_cols: bf16 (rows, W) with 16-byte aligned rows");
  TORCH_CHECK(!widths.empty() && widths.size() <= 4, "split_cols: 1 to 4 parts");
  SplitOut o{};
  std::vector<torch::Tensor> outs;
  int64_t W = 0;
  for (size_t i = 0; i < widths.size(); ++i) {
    TORCH_CHECK(widths[i] > 0 && widths[i] % 8 == 0, "split_cols: widths must be positive multiples of 8");
    outs.push_back(torch::empty({x.size(0), widths[i]}, x.options()));
    o.ptr[i] = (__nv_bfloat16*)outs.back().data_ptr();
    o.width[i] = (int)widths[i];
    W += widths[i];
  }
  o.n = (int)widths.size();
  TORCH_CHECK(W == x.size(1), "split_cols: widths must sum to the row width");
  const int64_t total = x.size(0) * (W / 8);
  if (total > 0) {
    TORCH_CHECK(x.size(0) < (int64_t)UINT32_MAX, "split_cols: too many rows");
    split_cols_kernel<<<ew_grid(total, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        (const __nv_bfloat16*)x.data_ptr(), x.stride(0), (uint32_t)x.size(0), (int)W, o);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return outs;
}

// ------------------------------------------------------------------------ embedding
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ w,
                                     float* __restrict__ out, int64_t n, int dim, int64_t vocab) {
  const int v4 = dim / 4;
  const int64_t total = n * v4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / v4;
    const int c = (int)(i % v4);
    int64_t id = ids[r];
    float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
    if (id >= 0 && id < vocab) val = reinterpret_cast<const float4*>(w + id * dim)[c];
    reinterpret_cast<float4*>(out + r * dim)[c] = val;
  }
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dout_bf,
                                     const float* __restrict__ dout_f, float* __restrict__ grad, int64_t n, int dim,
                                     int64_t vocab) {
  const int64_t total = n * dim;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / dim;
    const int c = (int)(i % dim);
    const int64_t id = ids[r];
    if (id < 0 || id >= vocab) continue;
    const float g = dout_f != nullptr ? dout_f[i] : __bfloat162float(dout_bf[i]);
    atomicAdd(grad + id * dim + c, g);
  }
}

torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor w) {
  c10::cuda::CUDAGuard guard(w.device());
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && w.size(1) % 4 == 0, "embedding: fp32 table");
  const int64_t n = ids.numel();
  auto out = torch::empty({n, w.size(1)}, w.options());
  if (n == 0) return out;
  embedding_fwd_kernel<<<ew_grid(n * w.size(1) / 4, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), w.data_ptr<float>(), out.data_ptr<float>(), n, w.size(1), w.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void embedding_bwd(torch::Tensor ids, torch::Tensor dout, torch::Tensor grad) {
  c10::cuda::CUDAGuard guard(grad.device());
  TORCH_CHECK(grad.scalar_type() == at::kFloat && grad.is_contiguous(), "embedding_bwd: fp32 grad");
  const int64_t n = ids.numel();
  if (n == 0) return;
  const bool f32 = dout.scalar_type() == at::kFloat;
  embedding_bwd_kernel<<<ew_grid(n * grad.size(1), 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), f32 ? nullptr : (const __nv_bfloat16*)dout.data_ptr(),
      f32 ? dout.data_ptr<float>() : nullptr, grad.data_ptr<float>(), n, grad.size(1), grad.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------ fp32 -> bf16
// The bf16 compute copy of an fp32 master weight (once per optimizer step and weight):
// 16-byte loads, 8-byte stores, round to nearest even.
__global__ void __launch_bounds__(256) cast_bf16_kernel(const float4* __restrict__ src, uint2* __restrict__ dst,
                                                        int64_t n4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = src[i];
    dst[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

torch::Tensor cast_bf16(torch::Tensor src) {
  c10::cuda::CUDAGuard guard(src.device());
  TORCH_CHECK(src.scalar_type() == at::kFloat && src.is_contiguous(), "cast_bf16: contiguous fp32 input");
  auto out = torch::empty(src.sizes(), src.options().dtype(at::kBFloat16));
  const int64_t n = src.numel();
  if (n == 0) return out;
  TORCH_CHECK(n % 4 == 0 && reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0,
              "cast_bf16: 16-byte aligned input of a multiple of 4 elements");
  cast_bf16_kernel<<<ew_grid(n / 4, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(src.data_ptr<float>()), reinterpret_cast<uint2*>(out.data_ptr()), n / 4);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace mykb
