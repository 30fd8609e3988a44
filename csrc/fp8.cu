// Float8 quantisers (sm_100a) for the per-tensor / per-row float8 linears.
//
// Statement (the same as the PyTorch form in myk_llm_b200/ops/float8.py, which the tests
// compare against):  amax = max(|x|) over the scaling group, clamped below by 1e-12;
// inv = (1 / amax) * fp8_max, each step IEEE-rounded (PyTorch evaluates `scalar / tensor`
// as a reciprocal and a product, and so does this kernel), for power-of-two scaling the exponent bits
// of inv alone (rounding inv down to a power of two); q = saturate_to_fp8(x * inv) with
// round-to-nearest-even; the dequantisation scale written out is 1 / inv.
//
//  * fp8_quant_rows      one scale per row: a CTA per row, amax and cast in one kernel
//                        (the row is re-read from L1/L2 for the cast).
//  * fp8_quant_tensor    one scale for the whole tensor: an amax kernel (float bits of
//                        |x| combined with integer atomicMax, valid for non-negative floats)
//                        and a cast kernel that reads the amax from device memory.
//  * fp8_quant_cols_t    one scale per column, written transposed: a column-amax kernel,
//                        then 64 x 64 tiles staged through shared memory and stored as rows
//                        of the transposed output (the operand layout of the weight-
//                        gradient GEMM, whose reduction runs over tokens).
//
// Inputs are bf16 (rows, cols) with cols % 8 == 0 and 16-byte aligned rows; every global
// access is 8 or 16 bytes wide.  The reference has no such kernels: it calls torchao.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp8.h>

#include "common.cuh"

namespace mykb {
namespace {

constexpr int kQThreads = 256;
constexpr float kAmaxEps = 1e-12f;

struct alignas(16) Bf16x8 {
  __nv_bfloat162 v[4];
};

__device__ __forceinline__ float inv_scale(float amax, float fmax, bool pow2) {
  const float inv = __fmul_rn(__frcp_rn(fmaxf(amax, kAmaxEps)), fmax);
  return pow2 ? __int_as_float(__float_as_int(inv) & 0x7f800000) : inv;
}

__device__ __forceinline__ float absmax8(const Bf16x8& v, float m) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(v.v[j]);
    m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  return m;
}

template <bool E5>
__device__ __forceinline__ uint32_t cvt2(float a, float b) {
  return (uint32_t)(uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, E5 ? __NV_E5M2 : __NV_E4M3);
}

template <bool E5>
__device__ __forceinline__ uint2 cast8(const Bf16x8& v, float inv) {
  uint32_t w[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float2 a = __bfloat1622float2(v.v[2 * h]);
    const float2 b = __bfloat1622float2(v.v[2 * h + 1]);
    w[h] = cvt2<E5>(__fmul_rn(a.x, inv), __fmul_rn(a.y, inv)) |
           (cvt2<E5>(__fmul_rn(b.x, inv), __fmul_rn(b.y, inv)) << 16);
  }
  return make_uint2(w[0], w[1]);
}

__device__ __forceinline__ float block_max(float m, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[0] = m;
  }
  __syncthreads();
  return red[0];
}

template <bool E5>
__global__ void __launch_bounds__(kQThreads) fp8_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t C,
                                                             float fmax, bool pow2, uint8_t* __restrict__ q,
                                                             float* __restrict__ scale) {
  __shared__ float red[kQThreads / 32];
  const int64_t r = blockIdx.x;
  const __nv_bfloat16* row = x + r * C;
  float m = 0.f;
  for (int64_t c = threadIdx.x * 8; c < C; c += kQThreads * 8)
    m = absmax8(*reinterpret_cast<const Bf16x8*>(row + c), m);
  const float inv = inv_scale(block_max(m, red), fmax, pow2);
  if (threadIdx.x == 0) scale[r] = __frcp_rn(inv);
  for (int64_t c = threadIdx.x * 8; c < C; c += kQThreads * 8)
    *reinterpret_cast<uint2*>(q + r * C + c) = cast8<E5>(*reinterpret_cast<const Bf16x8*>(row + c), inv);
}

// Column (per_col) or whole-tensor amax.  Block: 32 column groups of 8 x 8 row lanes; the
// grid covers 256 columns by kAmaxRows rows per block.  `out` starts at zero.
constexpr int kAmaxRows = 128;

__global__ void __launch_bounds__(kQThreads) fp8_amax_kernel(const __nv_bfloat16* __restrict__ x, int64_t R,
                                                             int64_t C, bool per_col, unsigned* __restrict__ out) {
  __shared__ float part[8][256];
  __shared__ float red[kQThreads / 32];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 256 + tx * 8;
  const int64_t r0 = (int64_t)blockIdx.y * kAmaxRows;
  const int64_t r1 = min(R, r0 + kAmaxRows);
  float m[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) m[j] = 0.f;
  if (c < C) {
    for (int64_t r = r0 + ty; r < r1; r += 8) {
      const Bf16x8 v = *reinterpret_cast<const Bf16x8*>(x + r * C + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(v.v[j]);
        m[2 * j] = fmaxf(m[2 * j], fabsf(f.x));
        m[2 * j + 1] = fmaxf(m[2 * j + 1], fabsf(f.y));
      }
    }
  }
  if (!per_col) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t = fmaxf(t, m[j]);
    t = block_max(t, red);
    if (threadIdx.x == 0) atomicMax(out, __float_as_uint(t));
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) part[ty][tx * 8 + j] = m[j];
  __syncthreads();
  const int col = threadIdx.x;   // 256 threads, one per column of the block
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) t = fmaxf(t, part[k][col]);
  const int64_t cc = (int64_t)blockIdx.x * 256 + col;
  if (cc < C) atomicMax(out + cc, __float_as_uint(t));
}

template <bool E5>
__global__ void __launch_bounds__(kQThreads) fp8_cast_kernel(const __nv_bfloat16* __restrict__ x, int64_t n8,
                                                             const unsigned* __restrict__ amax, float fmax,
                                                             uint8_t* __restrict__ q, float* __restrict__ scale) {
  const float inv = inv_scale(__uint_as_float(*amax), fmax, false);
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale = __frcp_rn(inv);
  for (int64_t i = blockIdx.x * (int64_t)kQThreads + threadIdx.x; i < n8; i += (int64_t)gridDim.x * kQThreads)
    *reinterpret_cast<uint2*>(q + i * 8) = cast8<E5>(reinterpret_cast<const Bf16x8*>(x)[i], inv);
}

// x (R, C) -> qT (C, R) with one scale per column of x (per row of qT).  64 x 64 tiles; R % 16 == 0.
template <bool E5>
__global__ void __launch_bounds__(kQThreads) fp8_cast_t_kernel(const __nv_bfloat16* __restrict__ x, int64_t R,
                                                               int64_t C, const unsigned* __restrict__ amax,
                                                               float fmax, bool pow2, uint8_t* __restrict__ qt,
                                                               float* __restrict__ scale) {
  __shared__ float tile[64][65];
  const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
  {
    const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;   // 8 column groups x 32 rows
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int rr = ty + 32 * it;
      const int64_t r = r0 + rr, c = c0 + tx * 8;
      Bf16x8 v;
      if (r < R && c < C) {
        v = *reinterpret_cast<const Bf16x8*>(x + r * C + c);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) v.v[j] = __floats2bfloat162_rn(0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(v.v[j]);
        tile[rr][tx * 8 + 2 * j] = f.x;
        tile[rr][tx * 8 + 2 * j + 1] = f.y;
      }
    }
  }
  __syncthreads();
  const int oc = threadIdx.x >> 2, part = threadIdx.x & 3;   // 64 output rows x 4 chunks of 16
  const int64_t c = c0 + oc, r = r0 + part * 16;
  if (c >= C || r >= R) return;
  const float inv = inv_scale(__uint_as_float(amax[c]), fmax, pow2);
  if (blockIdx.y == 0 && part == 0) scale[c] = __frcp_rn(inv);
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = part * 16 + 4 * k;
    w[k] = cvt2<E5>(__fmul_rn(tile[i][oc], inv), __fmul_rn(tile[i + 1][oc], inv)) |
           (cvt2<E5>(__fmul_rn(tile[i + 2][oc], inv), __fmul_rn(tile[i + 3][oc], inv)) << 16);
  }
  *reinterpret_cast<uint4*>(qt + c * R + r) = make_uint4(w[0], w[1], w[2], w[3]);
}

void check_input(const torch::Tensor& x, const char* who) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous() &&
                  x.size(1) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              who, ": contiguous bf16 (rows, cols) with cols % 8 == 0");
}

float fp8_max(bool e5m2) { return e5m2 ? 57344.f : 448.f; }

at::ScalarType fp8_type(bool e5m2) { return e5m2 ? at::ScalarType::Float8_e5m2 : at::ScalarType::Float8_e4m3fn; }

}  // namespace

std::vector<torch::Tensor> fp8_quant_rows(torch::Tensor x, bool e5m2, bool pow2) {
  check_input(x, "fp8_quant_rows");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t R = x.size(0), C = x.size(1);
  auto q = torch::empty({R, C}, x.options().dtype(fp8_type(e5m2)));
  auto s = torch::empty({R, 1}, x.options().dtype(at::kFloat));
  if (R > 0) {
    TORCH_CHECK(R < (int64_t)INT32_MAX, "fp8_quant_rows: too many rows");
    auto stream = at::cuda::getCurrentCUDAStream();
    auto* qp = reinterpret_cast<uint8_t*>(q.data_ptr());
    auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    if (e5m2)
      fp8_rows_kernel<true><<<(unsigned)R, kQThreads, 0, stream>>>(xp, C, fp8_max(e5m2), pow2, qp, s.data_ptr<float>());
    else
      fp8_rows_kernel<false><<<(unsigned)R, kQThreads, 0, stream>>>(xp, C, fp8_max(e5m2), pow2, qp, s.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {q, s};
}

std::vector<torch::Tensor> fp8_quant_tensor(torch::Tensor x, bool e5m2) {
  check_input(x, "fp8_quant_tensor");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t R = x.size(0), C = x.size(1);
  auto q = torch::empty({R, C}, x.options().dtype(fp8_type(e5m2)));
  auto s = torch::empty({}, x.options().dtype(at::kFloat));
  auto amax = torch::zeros({1}, x.options().dtype(at::kInt));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* ap = reinterpret_cast<unsigned*>(amax.data_ptr());
  if (R > 0 && C > 0) {
    TORCH_CHECK((R + kAmaxRows - 1) / kAmaxRows < 65536, "fp8_quant_tensor: too many rows");
    dim3 grid((unsigned)((C + 255) / 256), (unsigned)((R + kAmaxRows - 1) / kAmaxRows));
    fp8_amax_kernel<<<grid, kQThreads, 0, stream>>>(xp, R, C, false, ap);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  const int64_t n8 = R * C / 8;
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n8 + kQThreads - 1) / kQThreads, 148 * 16));
  auto* qp = reinterpret_cast<uint8_t*>(q.data_ptr());
  if (e5m2)
    fp8_cast_kernel<true><<<blocks, kQThreads, 0, stream>>>(xp, n8, ap, fp8_max(e5m2), qp, s.data_ptr<float>());
  else
    fp8_cast_kernel<false><<<blocks, kQThreads, 0, stream>>>(xp, n8, ap, fp8_max(e5m2), qp, s.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {q, s};
}

std::vector<torch::Tensor> fp8_quant_cols_t(torch::Tensor x, bool e5m2, bool pow2) {
  check_input(x, "fp8_quant_cols_t");
  const int64_t R = x.size(0), C = x.size(1);
  TORCH_CHECK(R % 16 == 0, "fp8_quant_cols_t: rows must be a multiple of 16");
  c10::cuda::CUDAGuard guard(x.device());
  auto qt = torch::empty({C, R}, x.options().dtype(fp8_type(e5m2)));
  auto s = torch::empty({C, 1}, x.options().dtype(at::kFloat));
  if (R == 0 || C == 0) return {qt, s};
  TORCH_CHECK((R + 63) / 64 < 65536 && (R + kAmaxRows - 1) / kAmaxRows < 65536, "fp8_quant_cols_t: too many rows");
  auto amax = torch::zeros({C}, x.options().dtype(at::kInt));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* ap = reinterpret_cast<unsigned*>(amax.data_ptr());
  dim3 g1((unsigned)((C + 255) / 256), (unsigned)((R + kAmaxRows - 1) / kAmaxRows));
  fp8_amax_kernel<<<g1, kQThreads, 0, stream>>>(xp, R, C, true, ap);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  dim3 g2((unsigned)((C + 63) / 64), (unsigned)((R + 63) / 64));
  auto* qp = reinterpret_cast<uint8_t*>(qt.data_ptr());
  if (e5m2)
    fp8_cast_t_kernel<true><<<g2, kQThreads, 0, stream>>>(xp, R, C, ap, fp8_max(e5m2), pow2, qp, s.data_ptr<float>());
  else
    fp8_cast_t_kernel<false><<<g2, kQThreads, 0, stream>>>(xp, R, C, ap, fp8_max(e5m2), pow2, qp, s.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {qt, s};
}

}  // namespace mykb
