// Optimizer kernels (sm_100a):
//   adamw_step       one launch over any number of fp32 tensors (pointer table in device
//                    memory, chunk -> tensor lookup by binary search over prefix sums)
//   muon_prepare     momentum lerp, Nesterov blend and bf16 pack of a same-shape bucket
//   muon_apply       decoupled weight decay + orthogonalised update of a bucket
//   frob_normalize_  per-matrix Frobenius normalisation of a bf16 batch (Newton-Schulz input)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace mykb {

constexpr int kChunk = 4096;
constexpr int kOptThreads = 256;

struct TensorTable {
  const int64_t* prefix;  // [n+1] chunk prefix
  const int64_t* numel;   // [n]
  const int64_t* ptrs;    // [n * k] pointers, k per tensor
  int n;
};

__device__ __forceinline__ int find_tensor(const int64_t* prefix, int n, int64_t chunk) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= chunk) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <typename TG>
__global__ void __launch_bounds__(kOptThreads)
adamw_kernel(TensorTable tab, int64_t total_chunks, float lr, float b1, float b2, float eps, float wd, float bc1,
             float bc2_sqrt, const float* __restrict__ gscale) {
  // gradients are scaled on load (gradient clipping), so no separate pass rewrites them
  const float gs = gscale != nullptr ? *gscale : 1.f;
  for (int64_t chunk = blockIdx.x; chunk < total_chunks; chunk += gridDim.x) {
    const int t = find_tensor(tab.prefix, tab.n, chunk);
    const int64_t start = (chunk - tab.prefix[t]) * kChunk;
    const int64_t n = tab.numel[t];
    float* p = reinterpret_cast<float*>(tab.ptrs[4 * t + 0]);
    const TG* g = reinterpret_cast<const TG*>(tab.ptrs[4 * t + 1]);
    float* m = reinterpret_cast<float*>(tab.ptrs[4 * t + 2]);
    float* v = reinterpret_cast<float*>(tab.ptrs[4 * t + 3]);
    const int64_t end = min(n, start + kChunk);
    auto update = [&](float gi, float& pi, float& mi, float& vi) {
      gi *= gs;
      pi *= 1.f - lr * wd;
      mi += (1.f - b1) * (gi - mi);
      vi = b2 * vi + (1.f - b2) * gi * gi;
      pi -= (lr / bc1) * mi / (sqrtf(vi) / bc2_sqrt + eps);
    };
    // 16-byte accesses when every stream is aligned (tensors can be views at any offset of a
    // flat buffer, so this is checked per tensor), scalar ones otherwise and for the tail
    const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) &
                      15) == 0 && (reinterpret_cast<uintptr_t>(g) & (4 * sizeof(TG) - 1)) == 0;
    int64_t tail = start;
    if (vec) {
      const int64_t nv = (end - start) / 4;
      for (int64_t j = threadIdx.x; j < nv; j += kOptThreads) {
        const int64_t i = start + 4 * j;
        float4 pv = *reinterpret_cast<float4*>(p + i), mv = *reinterpret_cast<float4*>(m + i),
               vv = *reinterpret_cast<float4*>(v + i);
        float gv[4];
        if constexpr (sizeof(TG) == 4) {
          const float4 t = *reinterpret_cast<const float4*>(g + i);
          gv[0] = t.x, gv[1] = t.y, gv[2] = t.z, gv[3] = t.w;
        } else {
          const uint2 t = *reinterpret_cast<const uint2*>(g + i);
          const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.x));
          const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.y));
          gv[0] = a.x, gv[1] = a.y, gv[2] = b.x, gv[3] = b.y;
        }
        update(gv[0], pv.x, mv.x, vv.x);
        update(gv[1], pv.y, mv.y, vv.y);
        update(gv[2], pv.z, mv.z, vv.z);
        update(gv[3], pv.w, mv.w, vv.w);
        *reinterpret_cast<float4*>(p + i) = pv;
        *reinterpret_cast<float4*>(m + i) = mv;
        *reinterpret_cast<float4*>(v + i) = vv;
      }
      tail = start + 4 * nv;
    }
    for (int64_t i = tail + threadIdx.x; i < end; i += kOptThreads) {
      float gi;
      if constexpr (sizeof(TG) == 4) gi = g[i]; else gi = __bfloat162float(g[i]);
      float pi = p[i], mi = m[i], vi = v[i];
      update(gi, pi, mi, vi);
      p[i] = pi;
      m[i] = mi;
      v[i] = vi;
    }
  }
}

static int grid_for(int64_t chunks) {
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (int)std::max<int64_t>(1, std::min<int64_t>(chunks, (int64_t)sms * 8));
}

// Builds the device tables: prefix/numel/pointer arrays in one pinned host buffer, copied
// asynchronously on the current stream.
static torch::Tensor build_table(const std::vector<std::vector<torch::Tensor>>& lists, std::vector<int64_t>& numels,
                                 int64_t& total_chunks, torch::Device dev) {
  const int n = lists[0].size();
  const int k = lists.size();
  auto host = torch::empty({(int64_t)(n + 1) + n + (int64_t)n * k}, torch::dtype(torch::kLong).pinned_memory(true));
  int64_t* h = host.data_ptr<int64_t>();
  int64_t acc = 0;
  for (int i = 0; i < n; ++i) {
    h[i] = acc;
    const int64_t ne = lists[0][i].numel();
    numels.push_back(ne);
    acc += (ne + kChunk - 1) / kChunk;
    h[(n + 1) + i] = ne;
    for (int j = 0; j < k; ++j) {
      TORCH_CHECK(lists[j][i].is_contiguous() && lists[j][i].numel() == ne, "multi-tensor: mismatched tensor ", i);
      h[(n + 1) + n + (int64_t)i * k + j] = reinterpret_cast<int64_t>(lists[j][i].data_ptr());
    }
  }
  h[n] = acc;
  total_chunks = acc;
  auto d = host.to(dev, /*non_blocking=*/true);
  // keep the pinned buffer alive until the copy has run
  c10::cuda::CUDACachingAllocator::recordStream(d.storage().data_ptr(), at::cuda::getCurrentCUDAStream());
  return d;
}

// gscale: optional fp32 scalar on the device multiplying every gradient as it is read.
void adamw_step(std::vector<torch::Tensor> params, std::vector<torch::Tensor> grads, std::vector<torch::Tensor> m,
                std::vector<torch::Tensor> v, int64_t step, double lr, double b1, double b2, double eps, double wd,
                c10::optional<torch::Tensor> gscale) {
  if (params.empty()) return;
  const float* gsp = nullptr;
  if (gscale.has_value()) {
    TORCH_CHECK(gscale->scalar_type() == at::kFloat && gscale->numel() == 1 && gscale->is_cuda(),
                "adamw: gscale must be one fp32 value on the device");
    gsp = gscale->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(params[0].device());
  for (auto& p : params) TORCH_CHECK(p.scalar_type() == at::kFloat, "adamw: fp32 params");
  const bool g_bf16 = grads[0].scalar_type() == at::kBFloat16;
  for (auto& g : grads) TORCH_CHECK(g.scalar_type() == grads[0].scalar_type(), "adamw: one grad dtype per call");
  std::vector<int64_t> numels;
  int64_t chunks = 0;
  auto table = build_table({params, grads, m, v}, numels, chunks, params[0].device());
  const int n = params.size();
  TensorTable tab{table.data_ptr<int64_t>(), table.data_ptr<int64_t>() + n + 1,
                  table.data_ptr<int64_t>() + 2 * n + 1, n};
  const float bc1 = 1.f - (float)std::pow(b1, (double)step);
  const float bc2s = (float)std::sqrt(1.0 - std::pow(b2, (double)step));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (g_bf16)
    adamw_kernel<__nv_bfloat16><<<grid_for(chunks), kOptThreads, 0, st>>>(tab, chunks, lr, b1, b2, eps, wd, bc1, bc2s,
                                                                          gsp);
  else
    adamw_kernel<float><<<grid_for(chunks), kOptThreads, 0, st>>>(tab, chunks, lr, b1, b2, eps, wd, bc1, bc2s, gsp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  // keep the table alive until the kernel ran
  c10::cuda::CUDACachingAllocator::recordStream(table.storage().data_ptr(), at::cuda::getCurrentCUDAStream());
}

// ------------------------------------------------------------------------------ Muon
// Muon kernels over a bucket of same-shape tensors: blockIdx.y is the tensor, blocks in x
// stride over its elements.  VEC: 4 elements per access (16-byte fp32 / 8-byte bf16), used
// when every pointer of the bucket is aligned and numel is a multiple of 4.
__device__ __forceinline__ void load4f(const float* p, float (&v)[4]) {
  const float4 t = *reinterpret_cast<const float4*>(p);
  v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
}
__device__ __forceinline__ void load4b(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 t = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&t.y));
  v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
}
__device__ __forceinline__ void store4b(__nv_bfloat16* p, const float (&v)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
  uint2 t;
  t.x = *reinterpret_cast<uint32_t*>(&a);
  t.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = t;
}

template <bool VEC>
__global__ void muon_prepare_kernel(const int64_t* gptrs, const int64_t* mptrs, int n, int64_t numel, float mu,
                                    bool nesterov, bool g_bf16, __nv_bfloat16* __restrict__ out,
                                    const float* __restrict__ gscale) {
  const float gs = gscale != nullptr ? *gscale : 1.f;
  const int t = blockIdx.y;
  float* m = reinterpret_cast<float*>(mptrs[t]);
  const float* gf = reinterpret_cast<const float*>(gptrs[t]);
  const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(gptrs[t]);
  __nv_bfloat16* o = out + (int64_t)t * numel;
  constexpr int W = VEC ? 4 : 1;
  for (int64_t j = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) * W; j < numel; j += (int64_t)gridDim.x * blockDim.x * W) {
    float g[W], mv[W], u[W];
    if constexpr (VEC) {
      if (g_bf16) load4b(gb + j, g); else load4f(gf + j, g);
      load4f(m + j, mv);
    } else {
      g[0] = g_bf16 ? __bfloat162float(gb[j]) : gf[j];
      mv[0] = m[j];
    }
#pragma unroll
    for (int e = 0; e < W; ++e) {
      g[e] *= gs;
      mv[e] += (1.f - mu) * (g[e] - mv[e]);
      u[e] = nesterov ? g[e] + mu * (mv[e] - g[e]) : mv[e];
    }
    if constexpr (VEC) {
      *reinterpret_cast<float4*>(m + j) = make_float4(mv[0], mv[1], mv[2], mv[3]);
      store4b(o + j, u);
    } else {
      m[j] = mv[0];
      o[j] = __float2bfloat16(u[0]);
    }
  }
}

template <bool VEC>
__global__ void muon_apply_kernel(const int64_t* pptrs, int n, int64_t numel, float decay, float step_scale,
                                  const __nv_bfloat16* __restrict__ orth) {
  const int t = blockIdx.y;
  float* p = reinterpret_cast<float*>(pptrs[t]);
  const __nv_bfloat16* o = orth + (int64_t)t * numel;
  constexpr int W = VEC ? 4 : 1;
  for (int64_t j = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) * W; j < numel; j += (int64_t)gridDim.x * blockDim.x * W) {
    if constexpr (VEC) {
      float pv[4], ov[4];
      load4f(p + j, pv);
      load4b(o + j, ov);
#pragma unroll
      for (int e = 0; e < 4; ++e) pv[e] = pv[e] * (1.f - decay) + step_scale * ov[e];
      *reinterpret_cast<float4*>(p + j) = make_float4(pv[0], pv[1], pv[2], pv[3]);
    } else {
      p[j] = p[j] * (1.f - decay) + step_scale * __bfloat162float(o[j]);
    }
  }
}

static bool aligned16(const std::vector<torch::Tensor>& ts) {
  for (auto& t : ts)
    if (reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) return false;
  return true;
}

static dim3 bucket_grid(int64_t numel, int n, int width) {
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (numel / width + 255) / 256;
  const int64_t cap = std::max<int64_t>(1, (int64_t)sms * 8 / std::max(1, n));
  return dim3((unsigned)std::max<int64_t>(1, std::min(need, cap)), (unsigned)n);
}

static torch::Tensor ptr_table(const std::vector<std::vector<torch::Tensor>>& lists, torch::Device dev) {
  const int n = lists[0].size();
  auto host = torch::empty({(int64_t)lists.size() * n}, torch::dtype(torch::kLong).pinned_memory(true));
  int64_t* h = host.data_ptr<int64_t>();
  for (size_t j = 0; j < lists.size(); ++j)
    for (int i = 0; i < n; ++i) {
      TORCH_CHECK(lists[j][i].is_contiguous(), "muon: contiguous tensors required");
      h[j * n + i] = reinterpret_cast<int64_t>(lists[j][i].data_ptr());
    }
  auto d = host.to(dev, true);
  return d;
}

void muon_prepare(std::vector<torch::Tensor> grads, std::vector<torch::Tensor> bufs, double mu, bool nesterov,
                  torch::Tensor out, c10::optional<torch::Tensor> gscale) {
  if (grads.empty()) return;
  const float* gsp = nullptr;
  if (gscale.has_value()) {
    TORCH_CHECK(gscale->scalar_type() == at::kFloat && gscale->numel() == 1 && gscale->is_cuda(),
                "muon_prepare: gscale must be one fp32 value on the device");
    gsp = gscale->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(out.device());
  const int n = grads.size();
  const int64_t numel = grads[0].numel();
  TORCH_CHECK(out.numel() == n * numel && out.scalar_type() == at::kBFloat16, "muon_prepare: bad output");
  for (auto& b : bufs) TORCH_CHECK(b.scalar_type() == at::kFloat, "muon_prepare: fp32 momentum");
  const bool g_bf16 = grads[0].scalar_type() == at::kBFloat16;
  auto tab = ptr_table({grads, bufs}, out.device());
  TORCH_CHECK(n <= 65535, "muon_prepare: too many tensors in one bucket");
  const bool vec = numel % 4 == 0 && aligned16(bufs) && aligned16({out}) &&
                   [&] { for (auto& g : grads) if (reinterpret_cast<uintptr_t>(g.data_ptr()) % (g_bf16 ? 8 : 16)) return false; return true; }();
  auto st = at::cuda::getCurrentCUDAStream();
  if (vec)
    muon_prepare_kernel<true><<<bucket_grid(numel, n, 4), 256, 0, st>>>(
        tab.data_ptr<int64_t>(), tab.data_ptr<int64_t>() + n, n, numel, (float)mu, nesterov, g_bf16,
        (__nv_bfloat16*)out.data_ptr(), gsp);
  else
    muon_prepare_kernel<false><<<bucket_grid(numel, n, 1), 256, 0, st>>>(
        tab.data_ptr<int64_t>(), tab.data_ptr<int64_t>() + n, n, numel, (float)mu, nesterov, g_bf16,
        (__nv_bfloat16*)out.data_ptr(), gsp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  c10::cuda::CUDACachingAllocator::recordStream(tab.storage().data_ptr(), at::cuda::getCurrentCUDAStream());
}

void muon_apply(std::vector<torch::Tensor> params, torch::Tensor orth, double decay, double step_scale) {
  if (params.empty()) return;
  c10::cuda::CUDAGuard guard(orth.device());
  const int n = params.size();
  const int64_t numel = params[0].numel();
  for (auto& p : params) TORCH_CHECK(p.scalar_type() == at::kFloat, "muon_apply: fp32 params");
  auto tab = ptr_table({params}, orth.device());
  TORCH_CHECK(n <= 65535, "muon_apply: too many tensors in one bucket");
  const bool vec = numel % 4 == 0 && aligned16(params) && aligned16({orth});
  auto st = at::cuda::getCurrentCUDAStream();
  if (vec)
    muon_apply_kernel<true><<<bucket_grid(numel, n, 4), 256, 0, st>>>(
        tab.data_ptr<int64_t>(), n, numel, (float)decay, (float)step_scale, (const __nv_bfloat16*)orth.data_ptr());
  else
    muon_apply_kernel<false><<<bucket_grid(numel, n, 1), 256, 0, st>>>(
        tab.data_ptr<int64_t>(), n, numel, (float)decay, (float)step_scale, (const __nv_bfloat16*)orth.data_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  c10::cuda::CUDACachingAllocator::recordStream(tab.storage().data_ptr(), at::cuda::getCurrentCUDAStream());
}

// ------------------------------------------------------------- Frobenius normalisation
__global__ void sumsq_kernel(const __nv_bfloat16* __restrict__ x, int64_t per, float* __restrict__ out) {
  const int b = blockIdx.y;
  const __nv_bfloat16* xb = x + (int64_t)b * per;
  float s = 0.f;
  const int64_t per8 = (reinterpret_cast<uintptr_t>(xb) % 16 == 0) ? per / 8 : 0;  // 16-byte part
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per8; i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 u = reinterpret_cast<const uint4*>(xb)[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      s += f.x * f.x + f.y * f.y;
    }
  }
  for (int64_t i = per8 * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v = __bfloat162float(xb[i]);
    s += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(out + b, t);
  }
}

__global__ void scale_kernel(__nv_bfloat16* __restrict__ x, int64_t per, const float* __restrict__ ss, float eps) {
  const int b = blockIdx.y;
  __nv_bfloat16* xb = x + (int64_t)b * per;
  const float inv = 1.f / fmaxf(sqrtf(ss[b]), eps);
  const int64_t per8 = (reinterpret_cast<uintptr_t>(xb) % 16 == 0) ? per / 8 : 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per8; i += (int64_t)gridDim.x * blockDim.x) {
    uint4 u = reinterpret_cast<uint4*>(xb)[i];
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      h[e] = __floats2bfloat162_rn(f.x * inv, f.y * inv);
    }
    reinterpret_cast<uint4*>(xb)[i] = u;
  }
  for (int64_t i = per8 * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per;
       i += (int64_t)gridDim.x * blockDim.x)
    xb[i] = __float2bfloat16(__bfloat162float(xb[i]) * inv);
}

void frob_normalize_(torch::Tensor x, double eps) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 3, "frob_normalize_: bf16 (B, r, c)");
  const int B = x.size(0);
  const int64_t per = x.size(1) * x.size(2);
  auto ss = torch::zeros({B}, x.options().dtype(at::kFloat));
  dim3 grid((unsigned)std::max<int64_t>(1, std::min<int64_t>(std::max<int64_t>(64, 1184 / std::max(1, B)),
                                                               (per / 8 + 255) / 256)), B);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  sumsq_kernel<<<grid, 256, 0, st>>>((const __nv_bfloat16*)x.data_ptr(), per, ss.data_ptr<float>());
  scale_kernel<<<grid, 256, 0, st>>>((__nv_bfloat16*)x.data_ptr(), per, ss.data_ptr<float>(), (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
