// Gated DeltaNet kernels (sm_100a): the chunked gated delta rule forward / backward
// (chunk 64, head dims 128), the token recurrence for decoding, and the short causal
// convolution + SiLU with its backward.
//
// Per chunk of 64 tokens (myk_llm_b200/ops/gdn_chunk.py states the same algebra and is
// the oracle), with k^ / q^ the L2-normalised key / query (q^ also scaled by dk^-1/2),
// gamma the cumulative log decay inside the chunk, E_ts = exp(gamma_t - gamma_s):
//
//   A  = strictly_lower(diag(beta) (E * K^ K^T)),   T = (I + A)^-1
//   W  = T diag(beta e^gamma) K^,                   U~ = T diag(beta) V
//   U  = U~ - W S0                                  (S0: state entering the chunk)
//   O  = diag(e^gamma) Q^ S0 + lower_incl(E * Q^ K^T) U
//   S1 = e^{gamma_C} S0 + (F * K^)^T U,             F_s = exp(gamma_C - gamma_s)
//
// Everything except the S0 -> S1 recurrence is independent per chunk; all five kernels
// are tcgen05 kernels in gdn_tc.cu:
//
//   forward:  gdn_prep_tc   (K^K^T, blocked triangular inverse, W, U~, T), one CTA per (chunk, head)
//             gdn_state_tc  (U = U~ - W S0, S1 = ...; saves S0 per chunk, U), one CTA per
//                           (sequence, head, 64 value columns), state in TMEM
//             gdn_out_tc    (P = lower(E * Q^K^T), O)
//   backward: gdn_dstate_tc (dS at every chunk end, reverse recurrence, dS in TMEM)
//             gdn_grad_tc   (dq, dk, dv, dg, dbeta of every chunk, l2-norm backward)
//
// This file holds the host entry points, the token recurrence for decoding and the
// speculative-decoding window, and the short causal convolution.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gdn_geo.cuh"

namespace mykb {
namespace gdnk {

typedef __nv_bfloat16 bf16;
constexpr int C = 64;      // chunk length
constexpr int DK = 128;    // head_k_dim
constexpr int DV = 128;    // head_v_dim
constexpr int NT = 256;    // threads of the recurrent decoding kernels

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void st2(bf16* p, float a, float b) { *reinterpret_cast<uint32_t*>(p) = pack2(a, b); }
__device__ __forceinline__ float2 ld2(const bf16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

// ---------------------------------------------------------------------- recurrence
// Token-by-token decoding: one CTA per (batch row, head); state (dk x dv) fp32 in shared
// memory; q/k normalised in-kernel.

struct RecSmem {
  float* S;    // [dk][dv]
  float* kv;   // [dk] normalised k
  float* qv;   // [dk] normalised, scaled q
  float* red;  // [32]
  float* u;    // [dv]
  __device__ RecSmem(float* sm, int dk, int dv)
      : S(sm), kv(sm + dk * dv), qv(sm + dk * dv + dk), red(sm + dk * dv + 2 * dk), u(sm + dk * dv + 2 * dk + 32) {}
};

// One token of the gated delta rule on the CTA's state:
//   S <- exp(g) S;  u = beta (v - S^T k);  S <- S + k u^T;  o = S^T q  (when o != nullptr).
// q/k/v point at this (token, head)'s vectors, g at its decay (one value, or dk values when
// per_channel).  Ends with a barrier, so S may be read or written right after.
__device__ __forceinline__ void rec_step(const RecSmem& s, const bf16* __restrict__ q, const bf16* __restrict__ k,
                                         const bf16* __restrict__ v, const float* __restrict__ g, float beta, int dk,
                                         int dv, float qscale, bool per_channel, bf16* __restrict__ o) {
  const int tid = threadIdx.x;
  __syncthreads();
  if (tid < 32) {
    float sk = 0.f, sq = 0.f;
    for (int i = tid; i < dk; i += 32) {
      const float a_ = __bfloat162float(k[i]);
      const float c_ = __bfloat162float(q[i]);
      s.kv[i] = a_;
      s.qv[i] = c_;
      sk += a_ * a_;
      sq += c_ * c_;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      sk += __shfl_xor_sync(0xffffffff, sk, off);
      sq += __shfl_xor_sync(0xffffffff, sq, off);
    }
    if (tid == 0) {
      s.red[0] = 1.f / fmaxf(sqrtf(sk), 1e-6f);
      s.red[1] = qscale / fmaxf(sqrtf(sq), 1e-6f);
    }
  }
  __syncthreads();
  for (int i = tid; i < dk; i += blockDim.x) {
    s.kv[i] *= s.red[0];
    s.qv[i] *= s.red[1];
  }
  __syncthreads();
  for (int i = tid; i < dk * dv; i += blockDim.x) {
    const float dec = per_channel ? __expf(g[i / dv]) : __expf(g[0]);
    s.S[i] *= dec;
  }
  __syncthreads();
  for (int c = tid; c < dv; c += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < dk; ++r) acc = fmaf(s.S[r * dv + c], s.kv[r], acc);
    s.u[c] = beta * (__bfloat162float(v[c]) - acc);
  }
  __syncthreads();
  for (int i = tid; i < dk * dv; i += blockDim.x) s.S[i] = fmaf(s.kv[i / dv], s.u[i % dv], s.S[i]);
  __syncthreads();
  if (o != nullptr) {
    for (int c = tid; c < dv; c += blockDim.x) {
      float acc = 0.f;
      for (int r = 0; r < dk; ++r) acc = fmaf(s.S[r * dv + c], s.qv[r], acc);
      o[c] = __float2bfloat16(acc);
    }
  }
  __syncthreads();
}

// Inputs of token t of row b, head h in a (B, T, H, d) layout.
struct RecInputs {
  const bf16 *q, *k, *v;
  const float *g, *beta;
  int T, H, dk, dv;
  bool per_channel;
  __device__ __forceinline__ int64_t row(int b, int t) const { return ((int64_t)b * T + t) * H; }
};

__device__ __forceinline__ void rec_token(const RecSmem& s, const RecInputs& in, int b, int t, int h, float qscale,
                                          bf16* out) {
  const int64_t r = in.row(b, t) + h;
  rec_step(s, in.q + r * in.dk, in.k + r * in.dk, in.v + r * in.dv, in.g + (in.per_channel ? r * in.dk : r),
           in.beta[r], in.dk, in.dv, qscale, in.per_channel, out != nullptr ? out + r * in.dv : nullptr);
}

// Decode T tokens from `init` (or zeros); outputs and the final state.
__global__ void __launch_bounds__(NT)
gdn_recurrent_kernel(RecInputs in, const float* __restrict__ init, bf16* __restrict__ out, float* __restrict__ fin,
                     float qscale) {
  extern __shared__ float sm[];
  const RecSmem s(sm, in.dk, in.dv);
  const int b = blockIdx.x / in.H, h = blockIdx.x % in.H;
  const int64_t sz = (int64_t)in.dk * in.dv, base = ((int64_t)b * in.H + h) * sz;
  for (int i = threadIdx.x; i < sz; i += blockDim.x) s.S[i] = init != nullptr ? init[base + i] : 0.f;
  for (int t = 0; t < in.T; ++t) rec_token(s, in, b, t, h, qscale, out);
  for (int i = threadIdx.x; i < sz; i += blockDim.x) fin[base + i] = s.S[i];
}

// One speculative-decoding window.  `state` holds the committed state of every (row,
// head); the previous window's inputs wait in `pend` and the first pending[b] of them were
// accepted.  The CTA folds those into the state and stores it (the new committed state),
// runs the W tokens of this window from there producing their outputs, and leaves this
// window's inputs in `pend` for the next call.  State traffic per call: one read and one
// write, whatever the acceptance.
__global__ void __launch_bounds__(NT)
gdn_spec_window_kernel(RecInputs in, RecInputs pend, float* __restrict__ state, const int* __restrict__ pending,
                       bf16* __restrict__ out, float qscale) {
  extern __shared__ float sm[];
  const RecSmem s(sm, in.dk, in.dv);
  const int b = blockIdx.x / in.H, h = blockIdx.x % in.H;
  const int64_t sz = (int64_t)in.dk * in.dv, base = ((int64_t)b * in.H + h) * sz;
  for (int i = threadIdx.x; i < sz; i += blockDim.x) s.S[i] = state[base + i];
  const int n = min(max(pending[b], 0), pend.T);
  for (int t = 0; t < n; ++t) rec_token(s, pend, b, t, h, qscale, nullptr);
  for (int i = threadIdx.x; i < sz; i += blockDim.x) state[base + i] = s.S[i];
  for (int t = 0; t < in.T; ++t) rec_token(s, in, b, t, h, qscale, out);
  // this window's inputs become the pending ones (only this CTA reads its (b, h) slice)
  const int gdim = in.per_channel ? in.dk : 1;
  for (int t = 0; t < in.T; ++t) {
    const int64_t r = in.row(b, t) + h;
    for (int i = threadIdx.x; i < in.dk; i += blockDim.x) {
      const_cast<bf16*>(pend.q)[r * in.dk + i] = in.q[r * in.dk + i];
      const_cast<bf16*>(pend.k)[r * in.dk + i] = in.k[r * in.dk + i];
    }
    for (int i = threadIdx.x; i < in.dv; i += blockDim.x) const_cast<bf16*>(pend.v)[r * in.dv + i] = in.v[r * in.dv + i];
    for (int i = threadIdx.x; i < gdim; i += blockDim.x) const_cast<float*>(pend.g)[r * gdim + i] = in.g[r * gdim + i];
    if (threadIdx.x == 0) const_cast<float*>(pend.beta)[r] = in.beta[r];
  }
}

// ---------------------------------------------------------------------- short conv
// y[t, c] = silu(sum_i w[c, i] x[t - K + 1 + i, c]), inputs before a document start read
// as 0 (batch layout: the initial state).  One thread owns 2 channels of a 64-token tile
// and slides a register window over time.
constexpr int kConvTile = 64;

struct ConvDocs {
  const int* cu;
  int nseq;
  __device__ __forceinline__ void find(int t, int T, int& start, int& end, int& d) const {
    if (cu == nullptr) {
      start = 0, end = T, d = 0;
      return;
    }
    int lo = 0, hi = nseq - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cu[mid] <= t) lo = mid; else hi = mid - 1;
    }
    d = lo, start = cu[lo], end = cu[lo + 1];
  }
};

template <int K>
__device__ __forceinline__ void conv_prime(float2 (&win)[K], const bf16* xb, const float* init, int b, int c, int D,
                                           int t0, int start, bool batch) {
#pragma unroll
  for (int i = 0; i < K - 1; ++i) {
    const int p = t0 - (K - 1) + i;
    if (p >= start) win[i] = ld2(xb + (int64_t)p * D);
    else if (init != nullptr && batch)
      win[i] = make_float2(init[((int64_t)b * D + c) * (K - 1) + (p + K - 1)],
                           init[((int64_t)b * D + c + 1) * (K - 1) + (p + K - 1)]);
    else win[i] = make_float2(0.f, 0.f);
  }
}

template <int K>
__global__ void conv1d_fwd_kernel(const bf16* __restrict__ x, const float* __restrict__ w, ConvDocs docs,
                                  const float* __restrict__ init, bf16* __restrict__ y, int T, int D) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (c >= D) return;
  const int b = blockIdx.z, t0 = blockIdx.y * kConvTile;
  if (t0 >= T) return;
  float w0[K], w1[K];
#pragma unroll
  for (int i = 0; i < K; ++i) {
    w0[i] = w[c * K + i];
    w1[i] = w[(c + 1) * K + i];
  }
  const bf16* xb = x + (int64_t)b * T * D + c;
  int start, end, d;
  docs.find(t0, T, start, end, d);
  float2 win[K];
  conv_prime<K>(win, xb, init, b, c, D, t0, start, docs.cu == nullptr);
  const int t1 = min(T, t0 + kConvTile);
  constexpr int kPre = 8;  // time steps loaded ahead: 8 independent loads in flight per thread
  for (int tb = t0; tb < t1; tb += kPre) {
    float2 xin[kPre];
#pragma unroll
    for (int u = 0; u < kPre; ++u) xin[u] = tb + u < t1 ? ld2(xb + (int64_t)(tb + u) * D) : make_float2(0.f, 0.f);
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
      const int t = tb + u;
      if (t >= t1) break;
      if (t >= end) {
        docs.find(t, T, start, end, d);
#pragma unroll
        for (int i = 0; i < K - 1; ++i) win[i] = make_float2(0.f, 0.f);
      }
      win[K - 1] = xin[u];
      float z0 = 0.f, z1 = 0.f;
#pragma unroll
      for (int i = 0; i < K; ++i) {
        z0 = fmaf(w0[i], win[i].x, z0);
        z1 = fmaf(w1[i], win[i].y, z1);
      }
      st2(y + ((int64_t)b * T + t) * D + c, z0 / (1.f + __expf(-z0)), z1 / (1.f + __expf(-z1)));
#pragma unroll
      for (int i = 0; i < K - 1; ++i) win[i] = win[i + 1];
    }
  }
}

// Backward in one pass over t in [t0, t0 + 64 + K - 1): recompute z, dz = dy silu'(z);
// dw[c][i] += dz_t x_{t-K+1+i} for the tile's own t; dx_{t'} = sum_i w_i dz_{t'+K-1-i}
// over t' + K - 1 - i inside the document of t'.  One atomic per (channel, tap) per tile.
template <int K>
__global__ void conv1d_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x, const float* __restrict__ w,
                                  ConvDocs docs, const float* __restrict__ init, bf16* __restrict__ dx,
                                  float* __restrict__ dw, int T, int D) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (c >= D) return;
  const int b = blockIdx.z, t0 = blockIdx.y * kConvTile;
  if (t0 >= T) return;
  float w0[K], w1[K], g0[K], g1[K];
#pragma unroll
  for (int i = 0; i < K; ++i) {
    w0[i] = w[c * K + i];
    w1[i] = w[(c + 1) * K + i];
    g0[i] = g1[i] = 0.f;
  }
  const bf16* xb = x + (int64_t)b * T * D + c;
  const bf16* dyb = dy + (int64_t)b * T * D + c;
  int start, end, d;
  docs.find(t0, T, start, end, d);
  float2 win[K];
  conv_prime<K>(win, xb, init, b, c, D, t0, start, docs.cu == nullptr);
  float2 dz[K];  // dz of positions t-K+1 .. t
  int dd[K];     // their document (-1: none)
#pragma unroll
  for (int i = 0; i < K; ++i) {
    dz[i] = make_float2(0.f, 0.f);
    dd[i] = -1;
  }
  const int tend = t0 + kConvTile + K - 1;
  constexpr int kPre = 8;  // time steps of x and dy loaded ahead
  for (int tb = t0; tb < tend; tb += kPre) {
    float2 xin[kPre], gin[kPre];
#pragma unroll
    for (int v = 0; v < kPre; ++v) {
      const bool in = tb + v < T && tb + v < tend;
      xin[v] = in ? ld2(xb + (int64_t)(tb + v) * D) : make_float2(0.f, 0.f);
      gin[v] = in ? ld2(dyb + (int64_t)(tb + v) * D) : make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
      const int t = tb + u;
      if (t >= tend) break;
#pragma unroll
      for (int i = 0; i < K - 1; ++i) {
        dz[i] = dz[i + 1];
        dd[i] = dd[i + 1];
      }
      if (t < T) {
        if (t >= end) {
          docs.find(t, T, start, end, d);
#pragma unroll
          for (int i = 0; i < K - 1; ++i) win[i] = make_float2(0.f, 0.f);
        }
        win[K - 1] = xin[u];
        float z0 = 0.f, z1 = 0.f;
#pragma unroll
        for (int i = 0; i < K; ++i) {
          z0 = fmaf(w0[i], win[i].x, z0);
          z1 = fmaf(w1[i], win[i].y, z1);
        }
        const float2 gy = gin[u];
        const float s0 = 1.f / (1.f + __expf(-z0)), s1 = 1.f / (1.f + __expf(-z1));
        dz[K - 1] = make_float2(gy.x * s0 * (1.f + z0 * (1.f - s0)), gy.y * s1 * (1.f + z1 * (1.f - s1)));
        dd[K - 1] = d;
        if (t < t0 + kConvTile) {
#pragma unroll
          for (int i = 0; i < K; ++i) {
            g0[i] = fmaf(dz[K - 1].x, win[i].x, g0[i]);
            g1[i] = fmaf(dz[K - 1].y, win[i].y, g1[i]);
          }
        }
#pragma unroll
        for (int i = 0; i < K - 1; ++i) win[i] = win[i + 1];
      } else {
        dz[K - 1] = make_float2(0.f, 0.f);
        dd[K - 1] = -1;
      }
      const int tp = t - (K - 1);  // the dx position completed at this step: dz[m] is tp + m
      if (tp >= t0 && tp < T && tp < t0 + kConvTile) {
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int m = 0; m < K; ++m) {
          if (dd[m] == dd[0]) {
            a0 = fmaf(w0[K - 1 - m], dz[m].x, a0);
            a1 = fmaf(w1[K - 1 - m], dz[m].y, a1);
          }
        }
        st2(dx + ((int64_t)b * T + tp) * D + c, a0, a1);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < K; ++i) {
    atomicAdd(&dw[c * K + i], g0[i]);
    atomicAdd(&dw[(c + 1) * K + i], g1[i]);
  }
}

}  // namespace gdnk

// ------------------------------------------------------------------------------ host
using gdnk::bf16;

template <int K>
static void conv_launch(bool fwd, const torch::Tensor& x, const float* w, gdnk::ConvDocs docs, const float* init,
                        const torch::Tensor& y_or_dy, torch::Tensor* dx, float* dw) {
  const int B = x.size(0), T = x.size(1), D = x.size(2);
  dim3 grid((D / 2 + 127) / 128, (T + gdnk::kConvTile - 1) / gdnk::kConvTile, B);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (fwd)
    gdnk::conv1d_fwd_kernel<K><<<grid, 128, 0, st>>>((const bf16*)x.data_ptr(), w, docs, init,
                                                     (bf16*)y_or_dy.data_ptr(), T, D);
  else
    gdnk::conv1d_bwd_kernel<K><<<grid, 128, 0, st>>>((const bf16*)y_or_dy.data_ptr(), (const bf16*)x.data_ptr(), w,
                                                     docs, init, (bf16*)dx->data_ptr(), dw, T, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static void conv_dispatch(int K, bool fwd, const torch::Tensor& x, const float* w, gdnk::ConvDocs docs,
                          const float* init, const torch::Tensor& y_or_dy, torch::Tensor* dx, float* dw) {
  switch (K) {
    case 2: conv_launch<2>(fwd, x, w, docs, init, y_or_dy, dx, dw); break;
    case 3: conv_launch<3>(fwd, x, w, docs, init, y_or_dy, dx, dw); break;
    case 4: conv_launch<4>(fwd, x, w, docs, init, y_or_dy, dx, dw); break;
    case 5: conv_launch<5>(fwd, x, w, docs, init, y_or_dy, dx, dw); break;
    case 6: conv_launch<6>(fwd, x, w, docs, init, y_or_dy, dx, dw); break;
    case 8: conv_launch<8>(fwd, x, w, docs, init, y_or_dy, dx, dw); break;
    default: TORCH_CHECK(false, "causal_conv1d: kernel width ", K, " not instantiated (2-6, 8)");
  }
}

static void conv_check(const torch::Tensor& x, const c10::optional<torch::Tensor>& cu) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 3, "causal_conv1d: bf16 (B, T, D)");
  TORCH_CHECK(x.size(2) % 2 == 0, "causal_conv1d: even channel count");
  TORCH_CHECK(!cu.has_value() || (x.size(0) == 1 && cu->scalar_type() == at::kInt),
              "causal_conv1d: packed layout needs batch 1 and int32 cu_seqlens");
}

std::vector<torch::Tensor> conv1d_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> cu,
                                      c10::optional<torch::Tensor> init) {
  c10::cuda::CUDAGuard guard(x.device());
  conv_check(x, cu);
  const int B = x.size(0), T = x.size(1), D = x.size(2), K = w.size(-1);
  auto wf = w.reshape({D, K}).to(at::kFloat).contiguous();
  auto y = torch::empty_like(x);
  const int nseq = cu.has_value() ? cu->numel() - 1 : B;
  torch::Tensor init_f;
  if (init.has_value()) init_f = init->to(at::kFloat).contiguous();
  if (x.numel() > 0)
    conv_dispatch(K, true, x, wf.data_ptr<float>(),
                  gdnk::ConvDocs{cu.has_value() ? cu->data_ptr<int>() : nullptr, nseq},
                  init.has_value() ? init_f.data_ptr<float>() : nullptr, y, nullptr, nullptr);
  // final states (the last K-1 inputs of every sequence), assembled on the device
  auto fin = torch::zeros({nseq, D, K - 1}, x.options().dtype(at::kFloat));
  if (K > 1) {
    if (cu.has_value()) {
      auto cuc = cu->to(at::kLong);
      auto ends = cuc.slice(0, 1);
      auto starts = cuc.slice(0, 0, nseq);
      for (int j = 0; j < K - 1; ++j) {
        auto idx = ends - (K - 1) + j;
        auto valid = idx.ge(starts);
        auto rows = x[0].index_select(0, idx.clamp_min(0)).to(at::kFloat) * valid.unsqueeze(1).to(at::kFloat);
        fin.select(2, j).copy_(rows);
      }
    } else {
      for (int j = 0; j < K - 1; ++j) {
        const int tt = T - (K - 1) + j;
        if (tt >= 0) fin.select(2, j).copy_(x.select(1, tt).to(at::kFloat));
        else if (init.has_value()) fin.select(2, j).copy_(init_f.select(2, tt + K - 1));
      }
    }
  }
  return {y, fin.to(x.scalar_type())};
}

std::vector<torch::Tensor> conv1d_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w,
                                      c10::optional<torch::Tensor> cu, c10::optional<torch::Tensor> init) {
  c10::cuda::CUDAGuard guard(x.device());
  conv_check(x, cu);
  const int B = x.size(0), D = x.size(2), K = w.size(-1);
  auto wf = w.reshape({D, K}).to(at::kFloat).contiguous();
  auto dx = torch::empty_like(x);
  auto dw = torch::zeros({D, K}, x.options().dtype(at::kFloat));
  const int nseq = cu.has_value() ? cu->numel() - 1 : B;
  torch::Tensor init_f;
  if (init.has_value()) init_f = init->to(at::kFloat).contiguous();
  auto dyc = dy.to(at::kBFloat16).contiguous();
  if (x.numel() > 0)
    conv_dispatch(K, false, x, wf.data_ptr<float>(),
                  gdnk::ConvDocs{cu.has_value() ? cu->data_ptr<int>() : nullptr, nseq},
                  init.has_value() ? init_f.data_ptr<float>() : nullptr, dyc, &dx, dw.data_ptr<float>());
  return {dx, dw.reshape(w.sizes())};
}

// Chunk offsets are computed on the device (no host synchronisation); `bound` is the
// host-side upper bound T_total / 64 + num_seqs on the number of chunks, which sizes the
// per-chunk buffers and the chunk-parallel grids (CTAs past the real count exit).
static gdnk::Geo make_geo(const torch::Tensor& q, const torch::Tensor& v, const c10::optional<torch::Tensor>& cu,
                          torch::Tensor& chunk_off, torch::Tensor& order, int& bound) {
  gdnk::Geo g{};
  const int B = q.size(0), T = q.size(1), H = q.size(2);
  g.heads = H;
  g.rows = (int64_t)B * T;
  g.row_q = (int64_t)H * q.size(3);
  g.row_v = (int64_t)H * v.size(3);
  if (cu.has_value()) {
    TORCH_CHECK(B == 1 && cu->scalar_type() == at::kInt, "gdn: packed layout needs batch 1 and int32 cu_seqlens");
    const int n = cu->numel() - 1;
    g.num_seqs = n;
    g.cu = cu->data_ptr<int>();
    auto lens = cu->slice(0, 1) - cu->slice(0, 0, n);
    auto nch = torch::floor_divide(lens + (gdnk::C - 1), gdnk::C);
    chunk_off = torch::cat({torch::zeros({1}, cu->options()), torch::cumsum(nch, 0, at::kInt)}).contiguous();
    order = torch::argsort(lens, /*stable=*/true, /*dim=*/0, /*descending=*/true).to(at::kInt).contiguous();
    bound = (int)(((int64_t)T + gdnk::C - 1) / gdnk::C + n);
  } else {
    g.num_seqs = B;
    g.seq_len = T;
    const int per = (T + gdnk::C - 1) / gdnk::C;
    chunk_off = (torch::arange(B + 1, q.options().dtype(at::kInt)) * per).contiguous();
    order = torch::arange(B, q.options().dtype(at::kInt));
    bound = B * per;
  }
  g.chunk_off = chunk_off.data_ptr<int>();
  g.order = order.data_ptr<int>();
  return g;
}

static void gdn_check(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, const char* who) {
  TORCH_CHECK(q.dim() == 4 && q.size(3) == gdnk::DK && k.sizes() == q.sizes() && v.size(3) == gdnk::DV &&
                  v.size(2) == q.size(2) && v.size(1) == q.size(1),
              who, ": head_k_dim 128, head_v_dim 128, as many value heads as key heads");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              who, ": bf16 q/k/v");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), who, ": contiguous q/k/v");
}

void gdn_grad_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& q, const torch::Tensor& k,
                        const torch::Tensor& v, const torch::Tensor& beta_f, const torch::Tensor& gcum,
                        const torch::Tensor& kinv, const torch::Tensor& qinv, const torch::Tensor& u,
                        const torch::Tensor& states, const torch::Tensor& dstates, const torch::Tensor& tmat,
                        const torch::Tensor& dout, torch::Tensor& dq, torch::Tensor& dk, torch::Tensor& dv,
                        torch::Tensor& dg, torch::Tensor& db, float qscale, int* status, cudaStream_t stream);

void gdn_prep_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& q, const torch::Tensor& k,
                        const torch::Tensor& v, const torch::Tensor& gg_f, const torch::Tensor& beta_f,
                        torch::Tensor& gcum, torch::Tensor& kinv, torch::Tensor& qinv, torch::Tensor& w,
                        torch::Tensor& u, torch::Tensor& tmat, float qscale, int* status, cudaStream_t stream);
void gdn_state_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& k, const torch::Tensor& gcum,
                         const torch::Tensor& kinv, const torch::Tensor& w, torch::Tensor& u, const float* init,
                         torch::Tensor& states, torch::Tensor& fin, int* status, cudaStream_t stream);
void gdn_dstate_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& q, const torch::Tensor& k,
                          const torch::Tensor& gcum, const torch::Tensor& kinv, const torch::Tensor& qinv,
                          const torch::Tensor& w, const torch::Tensor& p, const torch::Tensor& dout,
                          const float* dfinal, torch::Tensor& dstates, torch::Tensor& dinit, int* status,
                          cudaStream_t stream);
void gdn_out_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& q, const torch::Tensor& k,
                       const torch::Tensor& gcum, const torch::Tensor& kinv, const torch::Tensor& qinv,
                       const torch::Tensor& u, const torch::Tensor& states, torch::Tensor& p, torch::Tensor& out,
                       int* status, cudaStream_t stream);

// Returns (o, final state, saved...) with saved = [states, u, p, w, gcum, kinv, qinv, t].
std::vector<torch::Tensor> gdn_chunk_fwd_entry(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor gg,
                                               torch::Tensor beta, c10::optional<torch::Tensor> init,
                                               c10::optional<torch::Tensor> cu, bool per_channel) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(!per_channel, "gdn_chunk_fwd: per-channel (KDA) decay is not handled by the chunk kernels");
  gdn_check(q, k, v, "gdn_chunk_fwd");
  torch::Tensor chunk_off, order;
  int bound = 0;
  gdnk::Geo g = make_geo(q, v, cu, chunk_off, order, bound);
  const int H = g.heads;
  const int64_t rows = (int64_t)q.size(0) * q.size(1);
  auto f32 = q.options().dtype(at::kFloat);
  auto out = torch::empty_like(v);
  const int nb = std::max(bound, 1);
  auto states = torch::empty({nb, H, gdnk::DK, gdnk::DV}, q.options());
  auto w = torch::empty({nb, H, gdnk::C, gdnk::DK}, q.options());
  auto u = torch::empty({nb, H, gdnk::C, gdnk::DV}, q.options());
  auto p = torch::empty({nb, H, gdnk::C, gdnk::C}, q.options());
  auto tmat = torch::empty({nb, H, gdnk::C, gdnk::C}, q.options());  // T = (I + A)^-1 per chunk and head
  auto gcum = torch::empty({H, rows}, f32);  // head-major per-token scalars
  auto kinv = torch::empty({H, rows}, f32);
  auto qinv = torch::empty({H, rows}, f32);
  auto fin = torch::empty({g.num_seqs, H, gdnk::DK, gdnk::DV}, f32);
  auto gf = gg.to(at::kFloat).contiguous();
  auto bf = beta.to(at::kFloat).contiguous();
  torch::Tensor init_f;
  if (init.has_value()) init_f = init->to(at::kFloat).contiguous();
  const float qscale = 1.f / std::sqrt((float)gdnk::DK);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (rows > 0 && g.num_seqs > 0) {
    gdn_prep_tc_launch(g, bound, q, k, v, gf, bf, gcum, kinv, qinv, w, u, tmat, qscale, device_status(), st);
    gdn_state_tc_launch(g, bound, k, gcum, kinv, w, u, init.has_value() ? init_f.data_ptr<float>() : nullptr, states,
                        fin, device_status(), st);
    gdn_out_tc_launch(g, bound, q, k, gcum, kinv, qinv, u, states, p, out, device_status(), st);
  } else {
    fin.zero_();
  }
  return {out, fin, states, u, p, w, gcum, kinv, qinv, tmat};
}

// Returns (dq, dk, dv, dg, dbeta, dinit).
std::vector<torch::Tensor> gdn_chunk_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                         torch::Tensor gg, torch::Tensor beta, c10::optional<torch::Tensor> init,
                                         c10::optional<torch::Tensor> cu, std::vector<torch::Tensor> saved,
                                         c10::optional<torch::Tensor> dfinal, bool per_channel) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(!per_channel, "gdn_chunk_bwd: per-channel decay is not handled by the chunk kernels");
  TORCH_CHECK(saved.size() == 8, "gdn_chunk_bwd: expects the 8 saved tensors of gdn_chunk_fwd");
  gdn_check(q, k, v, "gdn_chunk_bwd");
  torch::Tensor chunk_off, order;
  int bound = 0;
  gdnk::Geo g = make_geo(q, v, cu, chunk_off, order, bound);
  const int H = g.heads;
  auto &states = saved[0], &u = saved[1], &p = saved[2], &w = saved[3], &gcum = saved[4], &kinv = saved[5],
       &qinv = saved[6], &tmat = saved[7];
  auto bf = beta.to(at::kFloat).contiguous();
  auto doc = dout.to(at::kBFloat16).contiguous();
  auto f32 = q.options().dtype(at::kFloat);
  auto dstates = torch::empty_like(states);
  auto dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  auto dg = torch::empty(gg.sizes(), f32);
  auto db = torch::empty(beta.sizes(), f32);
  auto dinit = torch::empty({g.num_seqs, H, gdnk::DK, gdnk::DV}, f32);
  torch::Tensor dfin_f;
  if (dfinal.has_value()) dfin_f = dfinal->to(at::kFloat).contiguous();
  const float qscale = 1.f / std::sqrt((float)gdnk::DK);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t rows = (int64_t)q.size(0) * q.size(1);
  if (rows > 0 && g.num_seqs > 0) {
    gdn_dstate_tc_launch(g, bound, q, k, gcum, kinv, qinv, w, p, doc,
                         dfinal.has_value() ? dfin_f.data_ptr<float>() : nullptr, dstates, dinit, device_status(), st);
    gdn_grad_tc_launch(g, bound, q, k, v, bf, gcum, kinv, qinv, u, states, dstates, tmat, doc, dq, dk, dv, dg, db,
                       qscale, device_status(), st);
  } else {
    dinit.zero_();
  }
  return {dq, dk, dv, dg, db, dinit};
}

static gdnk::RecInputs rec_inputs(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                                  const torch::Tensor& g, const torch::Tensor& beta, bool per_channel) {
  gdnk::RecInputs in;
  in.q = (const bf16*)q.data_ptr();
  in.k = (const bf16*)k.data_ptr();
  in.v = (const bf16*)v.data_ptr();
  in.g = g.data_ptr<float>();
  in.beta = beta.data_ptr<float>();
  in.T = q.size(1);
  in.H = q.size(2);
  in.dk = q.size(3);
  in.dv = v.size(3);
  in.per_channel = per_channel;
  return in;
}

static int rec_smem(int dk, int dv) {
  const int smem = (dk * dv + 2 * dk + 32 + dv) * 4;
  TORCH_CHECK(smem <= 227 * 1024, "gated delta rule decode: state too large");
  return smem;
}

std::vector<torch::Tensor> gdn_recurrent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor gg,
                                         torch::Tensor beta, c10::optional<torch::Tensor> init, bool per_channel) {
  c10::cuda::CUDAGuard guard(q.device());
  const int B = q.size(0), H = q.size(2), dk = q.size(3), dv = v.size(3);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && v.size(2) == H, "gdn_recurrent: bf16, as many value heads as key heads");
  auto qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
  auto out = torch::empty_like(vc);
  auto fin = torch::empty({B, H, dk, dv}, q.options().dtype(at::kFloat));
  auto gf = gg.to(at::kFloat).contiguous();
  auto bf = beta.to(at::kFloat).contiguous();
  torch::Tensor init_f;
  if (init.has_value()) init_f = init->to(at::kFloat).contiguous();
  const int smem = rec_smem(dk, dv);
  static SmemOptIn a_rec;
  C10_CUDA_CHECK(a_rec.ensure(gdnk::gdn_recurrent_kernel, 227 * 1024));
  gdnk::gdn_recurrent_kernel<<<B * H, gdnk::NT, smem, at::cuda::getCurrentCUDAStream()>>>(
      rec_inputs(qc, kc, vc, gf, bf, per_channel), init.has_value() ? init_f.data_ptr<float>() : nullptr,
      (bf16*)out.data_ptr(), fin.data_ptr<float>(), 1.f / std::sqrt((float)dk));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {out, fin};
}

torch::Tensor gdn_spec_window(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
                              torch::Tensor state, torch::Tensor pq, torch::Tensor pk, torch::Tensor pv,
                              torch::Tensor pg, torch::Tensor pbeta, torch::Tensor pending, bool per_channel) {
  c10::cuda::CUDAGuard guard(q.device());
  const int B = q.size(0), W = q.size(1), H = q.size(2), dk = q.size(3), dv = v.size(3);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "gdn_spec_window: bf16 q/k/v");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && g.is_contiguous() && beta.is_contiguous(),
              "gdn_spec_window: contiguous inputs");
  TORCH_CHECK(g.scalar_type() == at::kFloat && beta.scalar_type() == at::kFloat, "gdn_spec_window: fp32 g / beta");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.size(0) == B && state.size(1) == H &&
                  state.size(2) == dk && state.size(3) == dv,
              "gdn_spec_window: state (B, H, dk, dv) fp32");
  TORCH_CHECK(pq.sizes() == q.sizes() && pk.sizes() == k.sizes() && pv.sizes() == v.sizes() &&
                  pg.sizes() == g.sizes() && pbeta.sizes() == beta.sizes(),
              "gdn_spec_window: pending buffers shaped like the window");
  TORCH_CHECK(pq.is_contiguous() && pk.is_contiguous() && pv.is_contiguous() && pg.is_contiguous() &&
                  pbeta.is_contiguous() && pq.scalar_type() == at::kBFloat16 && pg.scalar_type() == at::kFloat,
              "gdn_spec_window: pending buffers contiguous, bf16 q/k/v, fp32 g / beta");
  TORCH_CHECK(pending.scalar_type() == at::kInt && pending.numel() == B, "gdn_spec_window: pending (B,) int32");
  TORCH_CHECK(v.size(2) == H && beta.size(1) == W, "gdn_spec_window: shapes");
  auto out = torch::empty_like(v);
  const int smem = rec_smem(dk, dv);
  static SmemOptIn a_spec;
  C10_CUDA_CHECK(a_spec.ensure(gdnk::gdn_spec_window_kernel, 227 * 1024));
  gdnk::gdn_spec_window_kernel<<<B * H, gdnk::NT, smem, at::cuda::getCurrentCUDAStream()>>>(
      rec_inputs(q, k, v, g, beta, per_channel), rec_inputs(pq, pk, pv, pg, pbeta, per_channel),
      state.data_ptr<float>(), pending.data_ptr<int>(), (bf16*)out.data_ptr(), 1.f / std::sqrt((float)dk));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

}  // namespace mykb
