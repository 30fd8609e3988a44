// RMSNorm family (sm_100a): plain, fused residual-add + RMSNorm, and the gated RMSNorm
// of the DeltaNet output.  One warp per row, 16-byte vector accesses, fp32 statistics.
//
//   y = x * rsqrt(mean(x^2) + eps) * w                           (rmsnorm)
//   s = x + u;  y = rmsnorm(s)                                   (add + rmsnorm, s returned)
//   y = rmsnorm(o) * w * act(g),  act = silu (GDN) or sigmoid (KDA)
//
// Width-64 rows (per-head norms at head_dim 64) use their own kernels, two elements per lane.
//
// Backward accumulates the weight gradient in registers per warp, reduces it across the
// block in shared memory and adds it to global memory once per block.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace mykb {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

// Load / store 4 consecutive elements.
template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&v)[4]) {
  float4 t = *reinterpret_cast<const float4*>(p);
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  uint2 t = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&t.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&t.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
}
template <typename T>
__device__ __forceinline__ void store4(T* p, const float (&v)[4]);
template <>
__device__ __forceinline__ void store4<float>(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
  uint2 t;
  t.x = *reinterpret_cast<uint32_t*>(&a);
  t.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = t;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

constexpr int kNormWarps = 8;

// NC = number of 4-element chunks per lane (H = NC * 128).
template <int NC, typename TX, typename TU, typename TY>
__global__ void __launch_bounds__(32 * kNormWarps)
rmsnorm_fwd_kernel(const TX* __restrict__ x, const TU* __restrict__ u, TX* __restrict__ s_out,
                   const float* __restrict__ w, TY* __restrict__ y, float* __restrict__ rstd, int rows, float eps) {
  constexpr int H = NC * 128;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int row = blockIdx.x * kNormWarps + warp; row < rows; row += gridDim.x * kNormWarps) {
    float v[NC][4];
    float ss = 0.f;
    const int64_t base = (int64_t)row * H;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int idx = (c * 32 + lane) * 4;
      load4<TX>(x + base + idx, v[c]);
      if (u != nullptr) {
        float t[4];
        load4<TU>(u + base + idx, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[c][i] += t[i];
        store4<TX>(s_out + base + idx, v[c]);
        if constexpr (sizeof(TX) == 2) {  // the stored sum is what backward sees: normalise that
          load4<TX>(s_out + base + idx, v[c]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) ss += v[c][i] * v[c][i];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / H + eps);
    if (lane == 0) rstd[row] = r;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int idx = (c * 32 + lane) * 4;
      float wv[4], o[4];
      load4<float>(w + idx, wv);
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = v[c][i] * r * wv[i];
      store4<TY>(y + base + idx, o);
    }
  }
}

template <int NC, typename TX, typename TY>
__global__ void __launch_bounds__(32 * kNormWarps)
rmsnorm_bwd_kernel(const TY* __restrict__ dy, const TX* __restrict__ x, const float* __restrict__ w,
                   const float* __restrict__ rstd, const TX* __restrict__ dres, TX* __restrict__ dx,
                   float* __restrict__ dw, int rows, __nv_bfloat16* __restrict__ dx_bf) {
  constexpr int H = NC * 128;
  __shared__ float sdw[H];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < H; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  float acc[NC][4];
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[c][i] = 0.f;

  for (int row = blockIdx.x * kNormWarps + warp; row < rows; row += gridDim.x * kNormWarps) {
    const int64_t base = (int64_t)row * H;
    const float r = rstd[row];
    float xh[NC][4], g[NC][4], t[NC][4];
    float dot = 0.f;
    // rows up to 1024 wide issue every load of the row (x, dy and the residual gradient)
    // before the row reduction, so they are in flight together (wider rows would spill);
    // the weights come from L1 each row
    constexpr bool kEarly = NC <= 8;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int idx = (c * 32 + lane) * 4;
      float xv[4], dv[4], wv[4];
      load4<TX>(x + base + idx, xv);
      load4<TY>(dy + base + idx, dv);
      if (kEarly && dres != nullptr) load4<TX>(dres + base + idx, t[c]);
      load4<float>(w + idx, wv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        xh[c][i] = xv[i] * r;
        g[c][i] = dv[i] * wv[i];
        dot += g[c][i] * xh[c][i];
        acc[c][i] += dv[i] * xh[c][i];
      }
    }
    dot = warp_sum(dot) / H;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int idx = (c * 32 + lane) * 4;
      float o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = r * (g[c][i] - xh[c][i] * dot);
      if (dres != nullptr) {
        if (!kEarly) load4<TX>(dres + base + idx, t[c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] += t[c][i];
      }
      store4<TX>(dx + base + idx, o);
      if (dx_bf != nullptr) store4<__nv_bfloat16>(dx_bf + base + idx, o);  // bf16 copy for a bf16 residual branch
    }
  }
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) atomicAdd(&sdw[(c * 32 + lane) * 4 + i], acc[c][i]);
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
}

// ---------------------------------------------------------------- gated RMSNorm
__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

template <int NC>
__global__ void __launch_bounds__(32 * kNormWarps)
gated_fwd_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ g,
                 const float* __restrict__ w, __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int rows,
                 float eps, int act) {
  constexpr int H = NC * 128;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int row = blockIdx.x * kNormWarps + warp; row < rows; row += gridDim.x * kNormWarps) {
    const int64_t base = (int64_t)row * H;
    float v[NC][4];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      load4<__nv_bfloat16>(o + base + (c * 32 + lane) * 4, v[c]);
#pragma unroll
      for (int i = 0; i < 4; ++i) ss += v[c][i] * v[c][i];
    }
    const float r = rsqrtf(warp_sum(ss) / H + eps);
    if (lane == 0) rstd[row] = r;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int idx = (c * 32 + lane) * 4;
      float wv[4], gv[4], out[4];
      load4<float>(w + idx, wv);
      if (g != nullptr) load4<__nv_bfloat16>(g + base + idx, gv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float a = 1.f;
        if (g != nullptr) a = act == 0 ? gv[i] * sigm(gv[i]) : sigm(gv[i]);
        out[i] = v[c][i] * r * wv[i] * a;
      }
      store4<__nv_bfloat16>(y + base + idx, out);
    }
  }
}

template <int NC>
__global__ void __launch_bounds__(32 * kNormWarps)
gated_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ o,
                 const __nv_bfloat16* __restrict__ g, const float* __restrict__ w, const float* __restrict__ rstd,
                 __nv_bfloat16* __restrict__ dO, __nv_bfloat16* __restrict__ dg, float* __restrict__ dw, int rows,
                 int act) {
  constexpr int H = NC * 128;
  __shared__ float sdw[H];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < H; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  float acc[NC][4] = {};
  for (int row = blockIdx.x * kNormWarps + warp; row < rows; row += gridDim.x * kNormWarps) {
    const int64_t base = (int64_t)row * H;
    const float r = rstd[row];
    float xh[NC][4], gg[NC][4];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int idx = (c * 32 + lane) * 4;
      float ov[4], dv[4], gv[4] = {0.f, 0.f, 0.f, 0.f}, wv[4];
      load4<__nv_bfloat16>(o + base + idx, ov);
      load4<__nv_bfloat16>(dy + base + idx, dv);
      load4<float>(w + idx, wv);
      if (g != nullptr) load4<__nv_bfloat16>(g + base + idx, gv);
      float dgo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        xh[c][i] = ov[i] * r;
        float a = 1.f, da = 0.f;
        if (g != nullptr) {
          const float s = sigm(gv[i]);
          if (act == 0) {
            a = gv[i] * s;
            da = s * (1.f + gv[i] * (1.f - s));
          } else {
            a = s;
            da = s * (1.f - s);
          }
        }
        const float nw = xh[c][i] * wv[i];
        dgo[i] = dv[i] * nw * da;  // d gate
        const float dn = dv[i] * a;  // d (normed * w)
        acc[c][i] += dn * xh[c][i];
        gg[c][i] = dn * wv[i];
        dot += gg[c][i] * xh[c][i];
      }
      if (g != nullptr) store4<__nv_bfloat16>(dg + base + idx, dgo);
    }
    dot = warp_sum(dot) / H;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float out[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) out[i] = r * (gg[c][i] - xh[c][i] * dot);
      store4<__nv_bfloat16>(dO + base + (c * 32 + lane) * 4, out);
    }
  }
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) atomicAdd(&sdw[(c * 32 + lane) * 4 + i], acc[c][i]);
  __syncthreads();
  for (int i = threadIdx.x; i < H; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
}

// -------------------------------------------------------------------------------------
// host
// -------------------------------------------------------------------------------------
static int norm_grid(int rows) {
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int blocks = (rows + kNormWarps - 1) / kNormWarps;
  return std::max(1, std::min(blocks, sms * 8));
}

#define MYKB_NC_SWITCH(H, ...)                                    \
  switch (H) {                                                    \
    case 64: { /* two rows of 32 lanes would be wasteful; use NC=... */ \
      TORCH_CHECK(false, "rmsnorm: hidden 64 handled by the packed path"); } \
    case 128: { constexpr int NC = 1; __VA_ARGS__; break; }       \
    case 256: { constexpr int NC = 2; __VA_ARGS__; break; }       \
    case 512: { constexpr int NC = 4; __VA_ARGS__; break; }       \
    case 768: { constexpr int NC = 6; __VA_ARGS__; break; }       \
    case 1024: { constexpr int NC = 8; __VA_ARGS__; break; }      \
    case 1536: { constexpr int NC = 12; __VA_ARGS__; break; }     \
    case 2048: { constexpr int NC = 16; __VA_ARGS__; break; }     \
    default: TORCH_CHECK(false, "rmsnorm: unsupported hidden size ", H); \
  }

template <typename TX, typename TU, typename TY>
static void rms_fwd_launch(int H, const TX* x, const TU* u, TX* s, const float* w, TY* y, float* rstd, int rows,
                           float eps, cudaStream_t st) {
  const int grid = norm_grid(rows);
  MYKB_NC_SWITCH(H, rmsnorm_fwd_kernel<NC, TX, TU, TY><<<grid, 32 * kNormWarps, 0, st>>>(x, u, s, w, y, rstd, rows, eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Rows whose width is 64 (per-head q/k norms of head_dim 64) are processed as pairs folded
// into width 128 would mix statistics, so they get their own simple kernel.
__global__ void rmsnorm64_fwd_kernel(const __nv_bfloat16* x, const float* w, __nv_bfloat16* y, float* rstd, int rows,
                                     float eps) {
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  float2 v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(x + (int64_t)row * 64)[lane]);
  float ss = warp_sum(v.x * v.x + v.y * v.y);
  float r = rsqrtf(ss / 64 + eps);
  if (lane == 0) rstd[row] = r;
  reinterpret_cast<__nv_bfloat162*>(y + (int64_t)row * 64)[lane] =
      __floats2bfloat162_rn(v.x * r * w[2 * lane], v.y * r * w[2 * lane + 1]);
}

__global__ void rmsnorm64_bwd_kernel(const __nv_bfloat16* dy, const __nv_bfloat16* x, const float* w,
                                     const float* rstd, __nv_bfloat16* dx, float* dw, int rows) {
  __shared__ float sdw[64];
  if (threadIdx.x < 64) sdw[threadIdx.x] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row < rows) {
    float2 xv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(x + (int64_t)row * 64)[lane]);
    float2 dv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(dy + (int64_t)row * 64)[lane]);
    const float r = rstd[row];
    float h0 = xv.x * r, h1 = xv.y * r;
    float g0 = dv.x * w[2 * lane], g1 = dv.y * w[2 * lane + 1];
    float dot = warp_sum(g0 * h0 + g1 * h1) / 64;
    reinterpret_cast<__nv_bfloat162*>(dx + (int64_t)row * 64)[lane] =
        __floats2bfloat162_rn(r * (g0 - h0 * dot), r * (g1 - h1 * dot));
    atomicAdd(&sdw[2 * lane], dv.x * h0);
    atomicAdd(&sdw[2 * lane + 1], dv.y * h1);
  }
  __syncthreads();
  if (threadIdx.x < 64) atomicAdd(&dw[threadIdx.x], sdw[threadIdx.x]);
}

// Gated RMSNorm over width-64 rows (per-head DeltaNet outputs of head_v_dim 64): one warp
// per row, two elements per lane.
__device__ __forceinline__ void gate_act(float g, int act, float& a, float& da) {
  const float s = sigm(g);
  if (act == 0) {
    a = g * s;
    da = s * (1.f + g * (1.f - s));
  } else {
    a = s;
    da = s * (1.f - s);
  }
}

__global__ void gated64_fwd_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ g,
                                   const float* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                   float* __restrict__ rstd, int rows, float eps, int act) {
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const int64_t base = (int64_t)row * 64;
  const float2 v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(o + base)[lane]);
  const float r = rsqrtf(warp_sum(v.x * v.x + v.y * v.y) / 64 + eps);
  if (lane == 0) rstd[row] = r;
  float a0 = 1.f, a1 = 1.f, unused;
  if (g != nullptr) {
    const float2 gv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(g + base)[lane]);
    gate_act(gv.x, act, a0, unused);
    gate_act(gv.y, act, a1, unused);
  }
  reinterpret_cast<__nv_bfloat162*>(y + base)[lane] =
      __floats2bfloat162_rn(v.x * r * w[2 * lane] * a0, v.y * r * w[2 * lane + 1] * a1);
}

__global__ void gated64_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ o,
                                   const __nv_bfloat16* __restrict__ g, const float* __restrict__ w,
                                   const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dO,
                                   __nv_bfloat16* __restrict__ dg, float* __restrict__ dw, int rows, int act) {
  __shared__ float sdw[64];
  if (threadIdx.x < 64) sdw[threadIdx.x] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row < rows) {
    const int64_t base = (int64_t)row * 64;
    const float2 ov = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(o + base)[lane]);
    const float2 dv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(dy + base)[lane]);
    const float r = rstd[row];
    const float w0 = w[2 * lane], w1 = w[2 * lane + 1];
    const float h0 = ov.x * r, h1 = ov.y * r;
    float a0 = 1.f, a1 = 1.f, da0 = 0.f, da1 = 0.f;
    if (g != nullptr) {
      const float2 gv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(g + base)[lane]);
      gate_act(gv.x, act, a0, da0);
      gate_act(gv.y, act, a1, da1);
      reinterpret_cast<__nv_bfloat162*>(dg + base)[lane] =
          __floats2bfloat162_rn(dv.x * h0 * w0 * da0, dv.y * h1 * w1 * da1);
    }
    const float dn0 = dv.x * a0, dn1 = dv.y * a1;  // d (normed * w)
    const float g0 = dn0 * w0, g1 = dn1 * w1;
    const float dot = warp_sum(g0 * h0 + g1 * h1) / 64;
    reinterpret_cast<__nv_bfloat162*>(dO + base)[lane] = __floats2bfloat162_rn(r * (g0 - h0 * dot), r * (g1 - h1 * dot));
    atomicAdd(&sdw[2 * lane], dn0 * h0);
    atomicAdd(&sdw[2 * lane + 1], dn1 * h1);
  }
  __syncthreads();
  if (threadIdx.x < 64) atomicAdd(&dw[threadIdx.x], sdw[threadIdx.x]);
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, c10::optional<std::vector<torch::Tensor>> add,
                                       double eps, c10::ScalarType out_dtype) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() == 2, "rmsnorm_fwd: contiguous 2-D CUDA x");
  c10::cuda::CUDAGuard guard(x.device());
  const int rows = x.size(0), H = x.size(1);
  auto wf = w.to(at::kFloat).contiguous();
  auto y = torch::empty({rows, H}, x.options().dtype(out_dtype));
  auto rstd = torch::empty({rows}, x.options().dtype(at::kFloat));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (rows == 0) return {y, rstd};
  if (H == 64) {
    TORCH_CHECK(!add.has_value() && x.scalar_type() == at::kBFloat16 && out_dtype == at::kBFloat16,
                "rmsnorm_fwd: width 64 supports bf16 in/out without residual add");
    rmsnorm64_fwd_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(
        (const __nv_bfloat16*)x.data_ptr(), wf.data_ptr<float>(), (__nv_bfloat16*)y.data_ptr(), rstd.data_ptr<float>(),
        rows, (float)eps);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {y, rstd};
  }
  const void* u = nullptr;
  void* s = nullptr;
  bool u_f32 = false;
  if (add.has_value()) {
    auto& v = *add;
    TORCH_CHECK(v.size() == 2 && v[0].is_contiguous() && v[1].is_contiguous(), "rmsnorm_fwd: bad add operands");
    u = v[0].data_ptr();
    s = v[1].data_ptr();
    u_f32 = v[0].scalar_type() == at::kFloat;
    TORCH_CHECK(v[1].scalar_type() == x.scalar_type(), "rmsnorm_fwd: sum must have x's dtype");
  }
  const bool x_f32 = x.scalar_type() == at::kFloat;
  const bool y_f32 = out_dtype == at::kFloat;
  using bf = __nv_bfloat16;
#define MYKB_RMS(TX, TU, TY) \
  rms_fwd_launch<TX, TU, TY>(H, (const TX*)x.data_ptr(), (const TU*)u, (TX*)s, wf.data_ptr<float>(), (TY*)y.data_ptr(), \
                             rstd.data_ptr<float>(), rows, (float)eps, st)
  if (x_f32 && u_f32 && y_f32) MYKB_RMS(float, float, float);
  else if (x_f32 && u_f32 && !y_f32) MYKB_RMS(float, float, bf);
  else if (x_f32 && !u_f32 && y_f32) MYKB_RMS(float, bf, float);
  else if (x_f32 && !u_f32 && !y_f32) MYKB_RMS(float, bf, bf);
  else if (!x_f32 && u_f32 && y_f32) MYKB_RMS(bf, float, float);
  else if (!x_f32 && u_f32 && !y_f32) MYKB_RMS(bf, float, bf);
  else if (!x_f32 && !u_f32 && y_f32) MYKB_RMS(bf, bf, float);
  else MYKB_RMS(bf, bf, bf);
#undef MYKB_RMS
  return {y, rstd};
}

// dres: gradient arriving at the (un-normed) sum directly, added to dx.  bf16_copy: also
// return dx rounded to bf16 (third output), written by the same kernel.
std::vector<torch::Tensor> rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd,
                                       c10::optional<torch::Tensor> dres, bool bf16_copy) {
  c10::cuda::CUDAGuard guard(x.device());
  const int rows = x.size(0), H = x.size(1);
  auto wf = w.to(at::kFloat).contiguous();
  auto dx = torch::empty_like(x);
  auto dw = torch::zeros({H}, x.options().dtype(at::kFloat));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (rows == 0) return {dx, dw.to(w.scalar_type())};
  if (H == 64) {
    TORCH_CHECK(!dres.has_value() && dy.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16,
                "rmsnorm_bwd: width 64 supports bf16 only");
    rmsnorm64_bwd_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(
        (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), wf.data_ptr<float>(),
        rstd.data_ptr<float>(), (__nv_bfloat16*)dx.data_ptr(), dw.data_ptr<float>(), rows);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {dx, dw.to(w.scalar_type())};
  }
  const void* dr = nullptr;
  if (dres.has_value()) {
    TORCH_CHECK(dres->scalar_type() == x.scalar_type(), "rmsnorm_bwd: residual grad dtype must match x");
    dr = dres->data_ptr();
  }
  const int grid = norm_grid(rows);
  using bf = __nv_bfloat16;
  const bool x_f32 = x.scalar_type() == at::kFloat, y_f32 = dy.scalar_type() == at::kFloat;
  torch::Tensor dx_bf;
  if (bf16_copy && x_f32) dx_bf = torch::empty(x.sizes(), x.options().dtype(at::kBFloat16));
  bf* dxb = dx_bf.defined() ? (bf*)dx_bf.data_ptr() : nullptr;
#define MYKB_RMSB(TX, TY)                                                                                       \
  MYKB_NC_SWITCH(H, rmsnorm_bwd_kernel<NC, TX, TY><<<grid, 32 * kNormWarps, 0, st>>>(                          \
                        (const TY*)dy.data_ptr(), (const TX*)x.data_ptr(), wf.data_ptr<float>(),               \
                        rstd.data_ptr<float>(), (const TX*)dr, (TX*)dx.data_ptr(), dw.data_ptr<float>(), rows, \
                        dxb))
  if (x_f32 && y_f32) { MYKB_RMSB(float, float); }
  else if (x_f32) { MYKB_RMSB(float, bf); }
  else if (y_f32) { MYKB_RMSB(bf, float); }
  else { MYKB_RMSB(bf, bf); }
#undef MYKB_RMSB
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (bf16_copy) return {dx, dw.to(w.scalar_type()), dx_bf.defined() ? dx_bf : dx};
  return {dx, dw.to(w.scalar_type())};
}

std::vector<torch::Tensor> gated_rmsnorm_fwd(torch::Tensor o, c10::optional<torch::Tensor> g, torch::Tensor w,
                                             double eps, int64_t act) {
  c10::cuda::CUDAGuard guard(o.device());
  TORCH_CHECK(o.scalar_type() == at::kBFloat16, "gated_rmsnorm: bf16 input");
  const int rows = o.size(0), H = o.size(1);
  auto wf = w.to(at::kFloat).contiguous();
  auto y = torch::empty_like(o);
  auto rstd = torch::empty({rows}, o.options().dtype(at::kFloat));
  if (rows == 0) return {y, rstd};
  const __nv_bfloat16* gp = g.has_value() ? (const __nv_bfloat16*)g->data_ptr() : nullptr;
  const int grid = norm_grid(rows);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (H == 64) {
    gated64_fwd_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>((const __nv_bfloat16*)o.data_ptr(), gp,
                                                               wf.data_ptr<float>(), (__nv_bfloat16*)y.data_ptr(),
                                                               rstd.data_ptr<float>(), rows, (float)eps, (int)act);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {y, rstd};
  }
  MYKB_NC_SWITCH(H, gated_fwd_kernel<NC><<<grid, 32 * kNormWarps, 0, st>>>(
                        (const __nv_bfloat16*)o.data_ptr(), gp, wf.data_ptr<float>(), (__nv_bfloat16*)y.data_ptr(),
                        rstd.data_ptr<float>(), rows, (float)eps, (int)act));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, rstd};
}

std::vector<torch::Tensor> gated_rmsnorm_bwd(torch::Tensor dy, torch::Tensor o, c10::optional<torch::Tensor> g,
                                             torch::Tensor w, torch::Tensor rstd, int64_t act) {
  c10::cuda::CUDAGuard guard(o.device());
  const int rows = o.size(0), H = o.size(1);
  auto wf = w.to(at::kFloat).contiguous();
  auto dO = torch::empty_like(o);
  auto dg = g.has_value() ? torch::empty_like(*g) : torch::empty({0}, o.options());
  auto dw = torch::zeros({H}, o.options().dtype(at::kFloat));
  if (rows == 0) return {dO, dg, dw.to(w.scalar_type())};
  const __nv_bfloat16* gp = g.has_value() ? (const __nv_bfloat16*)g->data_ptr() : nullptr;
  const int grid = norm_grid(rows);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (H == 64) {
    gated64_bwd_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(
        (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)o.data_ptr(), gp, wf.data_ptr<float>(),
        rstd.data_ptr<float>(), (__nv_bfloat16*)dO.data_ptr(), g.has_value() ? (__nv_bfloat16*)dg.data_ptr() : nullptr,
        dw.data_ptr<float>(), rows, (int)act);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {dO, dg, dw.to(w.scalar_type())};
  }
  MYKB_NC_SWITCH(H, gated_bwd_kernel<NC><<<grid, 32 * kNormWarps, 0, st>>>(
                        (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)o.data_ptr(), gp,
                        wf.data_ptr<float>(), rstd.data_ptr<float>(), (__nv_bfloat16*)dO.data_ptr(),
                        g.has_value() ? (__nv_bfloat16*)dg.data_ptr() : nullptr, dw.data_ptr<float>(), rows,
                        (int)act));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dO, dg, dw.to(w.scalar_type())};
}

}  // namespace mykb
