// Collectives fused with compute over NVLink peer memory (sm_100a).
//
// The data-parallel runtime (myk_llm_b200/parallel/sharded.py) keeps, per rank, one flat
// fp32 parameter buffer and one flat fp32 gradient buffer in symmetric memory (every rank
// can load/store every other rank's buffers through peer pointers).  Each rank owns a set
// of element ranges of the flat buffers (whole matrices for Muon, even slices for AdamW).
// One optimizer step is:
//
//   peer_barrier                    all ranks finished backward (grads complete)
//   dp_reduce_sumsq                 owner reads its ranges from every peer's gradient
//                                   buffer (16-byte peer loads), writes the sum into its
//                                   own buffer and accumulates the squared norm
//   peer_barrier                    all partial norms written
//   dp_adamw_allgather              clip factor from all ranks' partial norms, AdamW on the
//                                   owned AdamW ranges, updated fp32 values stored into
//                                   every rank's parameter buffer (16-byte peer stores)
//   muon_prepare_owned / NS GEMMs / dp_muon_apply_allgather   same for owned matrices
//   peer_barrier                    all parameter writes visible before the next forward
//
// so the reduce-scatter is fused with the norm, and the all-gather with the optimizer
// update; no NCCL call is on this path.  Cross-GPU waits spin on flags with an acquire
// load and give up after kWaitNs, recording the call site in the status word.  Plain
// peer loads/stores only, no TMA.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace mykb {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// flags[r] points at rank r's flag array (world uint32 per barrier slot).  Rank `rank`
// writes `epoch` into slot [rank] of every peer, then waits until its own slots of all
// peers reach `epoch`.
__global__ void peer_barrier_kernel(const int64_t* __restrict__ flag_ptrs, int rank, int world, uint32_t epoch,
                                    int* status) {
  const int t = threadIdx.x;
  __threadfence_system();
  if (t < world) {
    uint32_t* peer = reinterpret_cast<uint32_t*>(flag_ptrs[t]);
    st_release_sys(peer + rank, epoch);
  }
  __syncwarp();
  if (t < world) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(flag_ptrs[rank]) + t;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      const uint32_t v = ld_acquire_sys(mine);
      if ((int32_t)(v - epoch) >= 0) break;
      if (globaltimer_ns() - t0 > kWaitNs) {
        set_status(status, kTimeoutPeer);
        break;
      }
    }
  }
  __syncwarp();
  __threadfence_system();
}

struct RangeTable {
  const int64_t* offset;  // [n] element offset in the flat buffers (multiple of 4)
  const int64_t* prefix;  // [n+1] prefix of lengths (each a multiple of 4)
  int n;
};

__device__ __forceinline__ int find_range(const int64_t* prefix, int n, int64_t i) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= i) lo = mid; else hi = mid - 1;
  }
  return lo;
}

constexpr int kMaxWorld = 8;

// grads[r] = rank r's flat gradient buffer.  For every owned element: own = sum_r grads[r],
// sumsq += own^2.  Vectorised by 4 (all offsets/lengths are multiples of 4).
__global__ void __launch_bounds__(256)
dp_reduce_sumsq_kernel(const int64_t* __restrict__ grad_ptrs, int rank, int world, RangeTable tab,
                       float* __restrict__ partial) {
  const int64_t total4 = tab.prefix[tab.n] / 4;
  const float4* src[kMaxWorld];
#pragma unroll
  for (int r = 0; r < kMaxWorld; ++r) src[r] = r < world ? reinterpret_cast<const float4*>(grad_ptrs[r]) : nullptr;
  float4* own = reinterpret_cast<float4*>(grad_ptrs[rank]);
  float ss = 0.f;
  for (int64_t i4 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i4 < total4; i4 += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = i4 * 4;
    const int k = find_range(tab.prefix, tab.n, i);
    const int64_t e = (tab.offset[k] + (i - tab.prefix[k])) / 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r) {
      if (r < world) {
        const float4 v = src[r][e];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
    }
    own[e] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(partial, t);
  }
}

// The same reduce-scatter through NVSwitch multicast (NVLS): one `multimem.ld_reduce`
// per 16 bytes reads the element from every rank's gradient buffer and returns the sum,
// reduced inside the switch, so each owned element crosses NVLink once instead of once
// per rank.  `mc` is the multicast address of the gradient buffer (same offsets as the
// per-rank buffers).
__device__ __forceinline__ float4 multimem_sum_f32x4(const float4* addr) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(addr)
               : "memory");
  return v;
}

__global__ void __launch_bounds__(256)
dp_reduce_sumsq_multimem_kernel(const float4* __restrict__ mc, float4* __restrict__ own, RangeTable tab,
                                float* __restrict__ partial) {
  const int64_t total4 = tab.prefix[tab.n] / 4;
  float ss = 0.f;
  for (int64_t i4 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i4 < total4; i4 += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = i4 * 4;
    const int k = find_range(tab.prefix, tab.n, i);
    const int64_t e = (tab.offset[k] + (i - tab.prefix[k])) / 4;
    const float4 acc = multimem_sum_f32x4(mc + e);
    own[e] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(partial, t);
  }
}

// Clip coefficient from every rank's partial squared norm (partials[r] points at rank r's
// float) plus the replicated-parameter part `extra_sq` (already global).
__device__ __forceinline__ float clip_coef(const int64_t* partial_ptrs, int world, float extra_sq, float max_norm,
                                           float* norm_out) {
  float s = extra_sq;
  for (int r = 0; r < world; ++r) s += *reinterpret_cast<const volatile float*>(partial_ptrs[r]);
  const float n = sqrtf(s);
  if (norm_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *norm_out = n;
  return max_norm > 0.f ? fminf(1.f, max_norm / (n + 1e-6f)) : 1.f;
}

// AdamW over the owned AdamW ranges; state m/v are rank-local arrays indexed by the
// position within the owned ranges.  The updated parameter is stored into every rank's
// parameter buffer.
__global__ void __launch_bounds__(256)
dp_adamw_allgather_kernel(const int64_t* __restrict__ param_ptrs, const int64_t* __restrict__ grad_ptrs, int rank,
                          int world, RangeTable tab, const float* __restrict__ wd_per_range,
                          const float* __restrict__ lr_per_range, float* __restrict__ m, float* __restrict__ v,
                          float b1, float b2, float eps, float bc1, float bc2_sqrt, const int64_t* partial_ptrs,
                          float extra_sq, float max_norm, float* norm_out) {
  const float coef = clip_coef(partial_ptrs, world, extra_sq, max_norm, norm_out);
  const int64_t total4 = tab.prefix[tab.n] / 4;
  float4* dst[kMaxWorld];
#pragma unroll
  for (int r = 0; r < kMaxWorld; ++r) dst[r] = r < world ? reinterpret_cast<float4*>(param_ptrs[r]) : nullptr;
  const float4* g4 = reinterpret_cast<const float4*>(grad_ptrs[rank]);
  float4* m4 = reinterpret_cast<float4*>(m);
  float4* v4 = reinterpret_cast<float4*>(v);
  for (int64_t i4 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i4 < total4; i4 += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = i4 * 4;
    const int k = find_range(tab.prefix, tab.n, i);
    const int64_t e = (tab.offset[k] + (i - tab.prefix[k])) / 4;
    const float lr = lr_per_range[k], wd = wd_per_range[k];
    float4 p = dst[rank][e];
    float4 g = g4[e];
    float4 mm = m4[i4], vv = v4[i4];
    float* pp = reinterpret_cast<float*>(&p);
    float* gg = reinterpret_cast<float*>(&g);
    float* mp = reinterpret_cast<float*>(&mm);
    float* vp = reinterpret_cast<float*>(&vv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gj = gg[j] * coef;
      mp[j] = mp[j] + (1.f - b1) * (gj - mp[j]);
      vp[j] = b2 * vp[j] + (1.f - b2) * gj * gj;
      const float denom = sqrtf(vp[j]) / bc2_sqrt + eps;
      pp[j] = pp[j] * (1.f - lr * wd) - (lr / bc1) * mp[j] / denom;
    }
    m4[i4] = mm;
    v4[i4] = vv;
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < world) dst[r][e] = p;
  }
}

// Muon, owned matrices: momentum / Nesterov / bf16 pack of (reduced grad * clip coef).
__global__ void __launch_bounds__(256)
dp_muon_prepare_kernel(const int64_t* __restrict__ grad_ptrs, int rank, int world, const int64_t* __restrict__ offs,
                       int n, int64_t numel, float* __restrict__ mom, float mu, bool nesterov,
                       __nv_bfloat16* __restrict__ out, const int64_t* partial_ptrs, float extra_sq, float max_norm) {
  const float coef = clip_coef(partial_ptrs, world, extra_sq, max_norm, nullptr);
  const float* g = reinterpret_cast<const float*>(grad_ptrs[rank]);
  const int64_t total = (int64_t)n * numel;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / numel);
    const int64_t j = i - (int64_t)t * numel;
    const float gv = g[offs[t] + j] * coef;
    const float mv = mom[i] + (1.f - mu) * (gv - mom[i]);
    mom[i] = mv;
    out[i] = __float2bfloat16(nesterov ? gv + mu * (mv - gv) : mv);
  }
}

// Muon, owned matrices: p <- p (1 - lr wd) + step_scale * orth, stored into every rank.
__global__ void __launch_bounds__(256)
dp_muon_apply_allgather_kernel(const int64_t* __restrict__ param_ptrs, int rank, int world,
                               const int64_t* __restrict__ offs, int n, int64_t numel, float decay, float step_scale,
                               const __nv_bfloat16* __restrict__ orth) {
  const int64_t total = (int64_t)n * numel;
  float* mine = reinterpret_cast<float*>(param_ptrs[rank]);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / numel);
    const int64_t e = offs[t] + (i - (int64_t)t * numel);
    const float p = mine[e] * (1.f - decay) + step_scale * __bfloat162float(orth[i]);
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < world) reinterpret_cast<float*>(param_ptrs[r])[e] = p;
  }
}

// Muon, owned row-sharded matrices (parameter-sharded mode): orth[t] is the full update of
// matrix t; row `row` of it lives on rank row / rows_per_rank.  The owner reads that rank's
// fp32 master row (peer load), applies p <- p (1 - lr wd) + step_scale * orth, and stores the
// fp32 master and its bf16 compute copy back into that rank's shard buffers (peer stores).
// Vectorised by 4 (cols is a multiple of 8).
__global__ void __launch_bounds__(256)
dp_muon_apply_shards_kernel(const int64_t* __restrict__ param_ptrs, const int64_t* __restrict__ bf16_ptrs,
                            const int64_t* __restrict__ poffs, const int64_t* __restrict__ boffs, int n, int rows,
                            int cols, int rows_per_rank, float decay, float step_scale,
                            const __nv_bfloat16* __restrict__ orth) {
  const int64_t numel = (int64_t)rows * cols;
  const int64_t total4 = (int64_t)n * numel / 4;
  for (int64_t i4 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i4 < total4; i4 += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = i4 * 4;
    const int t = (int)(i / numel);
    const int64_t j = i - (int64_t)t * numel;
    const int row = (int)(j / cols), col = (int)(j - (int64_t)row * cols);
    const int r = row / rows_per_rank;
    const int64_t local = (int64_t)(row - r * rows_per_rank) * cols + col;
    float4* pm = reinterpret_cast<float4*>(reinterpret_cast<float*>(param_ptrs[r]) + poffs[t] + local);
    uint2* pb = reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(bf16_ptrs[r]) + boffs[t] + local);
    const uint2 ov = *reinterpret_cast<const uint2*>(orth + i);
    const float2 o01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ov.x));
    const float2 o23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ov.y));
    float4 p = *pm;
    p.x = p.x * (1.f - decay) + step_scale * o01.x;
    p.y = p.y * (1.f - decay) + step_scale * o01.y;
    p.z = p.z * (1.f - decay) + step_scale * o23.x;
    p.w = p.w * (1.f - decay) + step_scale * o23.y;
    *pm = p;
    *pb = make_uint2(pack_bf16x2(p.x, p.y), pack_bf16x2(p.z, p.w));
  }
}

// Parameter-sharded mode, set-up and checkpoint load: bf16 compute copy of this rank's
// fp32 master shards (ranges of the flat buffers, multiples of 4 elements).
__global__ void __launch_bounds__(256)
cast_ranges_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, RangeTable src_tab,
                        const int64_t* __restrict__ dst_offs) {
  const int64_t total4 = src_tab.prefix[src_tab.n] / 4;
  for (int64_t i4 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i4 < total4; i4 += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = i4 * 4;
    const int k = find_range(src_tab.prefix, src_tab.n, i);
    const int64_t within = i - src_tab.prefix[k];
    const float4 v = *reinterpret_cast<const float4*>(src + src_tab.offset[k] + within);
    *reinterpret_cast<uint2*>(dst + dst_offs[k] + within) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

// -------------------------------------------------------------------------------------
// host wrappers
// -------------------------------------------------------------------------------------
static int comm_grid(int64_t work) {
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)sms * 4));
}

// fp8 all-gather of one MXFP8 weight whose rows are sharded over the ranks.  Every rank
// holds, in symmetric memory, the MXFP8 copies of its R rows of W (N x K): q0 (R x K) with
// its row-blocked scale atoms s0, and q1 = (W rows)^T (K x R) blocked along R with atoms
// s1.  The full operands are assembled locally from every rank's copies with 16-byte peer
// loads: q0 / s0 are one contiguous run per rank, q1 a column slab (one run of rows_r bytes
// per K row) and s1 one run of atoms per 128-row block of K.  grid.y = rank, grid.z =
// part (q0, s0, q1, s1).
struct MxGatherArgs {
  int64_t base[kMaxWorld];  // each rank's copies: q0 at +0, s0 at +R K, q1 at +R K (1 + 1/32), s1 after it
  uint8_t* q0;              // full (N x K)
  uint8_t* s0;
  uint8_t* q1;              // full (K x N)
  uint8_t* s1;
  int64_t R, K, N;
};

__global__ void __launch_bounds__(256) mx_shard_gather_kernel(MxGatherArgs a) {
  const int r = blockIdx.y, part = blockIdx.z;
  const int64_t row0 = (int64_t)r * a.R;
  const int64_t rows = max((int64_t)0, min(a.R, a.N - row0));  // this rank's valid rows (multiple of 128)
  if (rows == 0) return;
  const uint8_t* src = reinterpret_cast<const uint8_t*>(a.base[r]);
  const int64_t rk = a.R * a.K;
  int64_t units;
  if (part == 0 || part == 2) units = rows * a.K / 16;
  else units = rows * a.K / 32 / 16;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
    const uint4* from;
    uint4* to;
    if (part == 0) {
      from = reinterpret_cast<const uint4*>(src) + u;
      to = reinterpret_cast<uint4*>(a.q0 + row0 * a.K) + u;
    } else if (part == 1) {
      from = reinterpret_cast<const uint4*>(src + rk) + u;
      to = reinterpret_cast<uint4*>(a.s0 + row0 * a.K / 32) + u;
    } else if (part == 2) {
      const int64_t per = rows / 16, k = u / per, c = u - k * per;
      from = reinterpret_cast<const uint4*>(src + rk + rk / 32 + k * a.R) + c;
      to = reinterpret_cast<uint4*>(a.q1 + k * a.N + row0) + c;
    } else {
      const int64_t per = rows / 4, kb = u / per, c = u - kb * per;  // rows / 128 atoms of 512 bytes per K block
      from = reinterpret_cast<const uint4*>(src + 2 * rk + rk / 32 + kb * (a.R / 128) * 512) + c;
      to = reinterpret_cast<uint4*>(a.s1 + kb * (a.N / 128) * 512 + (row0 / 128) * 512) + c;
    }
    *to = *from;
  }
}

void peer_barrier(torch::Tensor flag_ptrs, int64_t rank, int64_t world, int64_t epoch) {
  TORCH_CHECK(world <= kMaxWorld, "peer_barrier: world > 8");
  peer_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(flag_ptrs.data_ptr<int64_t>(), (int)rank,
                                                                      (int)world, (uint32_t)epoch, device_status());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_reduce_sumsq(torch::Tensor grad_ptrs, int64_t rank, int64_t world, torch::Tensor offsets,
                     torch::Tensor prefix, torch::Tensor partial, int64_t total) {
  TORCH_CHECK(world <= kMaxWorld, "dp_reduce: world > 8");
  RangeTable tab{offsets.data_ptr<int64_t>(), prefix.data_ptr<int64_t>(), (int)offsets.numel()};
  if (total == 0 || tab.n == 0) return;
  dp_reduce_sumsq_kernel<<<comm_grid(total / 4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      grad_ptrs.data_ptr<int64_t>(), (int)rank, (int)world, tab, partial.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_reduce_sumsq_multimem(int64_t grad_mc, torch::Tensor own_grad, torch::Tensor offsets, torch::Tensor prefix,
                              torch::Tensor partial, int64_t total) {
  RangeTable tab{offsets.data_ptr<int64_t>(), prefix.data_ptr<int64_t>(), (int)offsets.numel()};
  if (total == 0 || tab.n == 0) return;
  TORCH_CHECK(grad_mc != 0 && grad_mc % 16 == 0, "dp_reduce_multimem: a 16-byte aligned multicast address");
  dp_reduce_sumsq_multimem_kernel<<<comm_grid(total / 4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(grad_mc), reinterpret_cast<float4*>(own_grad.data_ptr<float>()), tab,
      partial.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_adamw_allgather(torch::Tensor param_ptrs, torch::Tensor grad_ptrs, int64_t rank, int64_t world,
                        torch::Tensor offsets, torch::Tensor prefix, torch::Tensor wd, torch::Tensor lr,
                        torch::Tensor m, torch::Tensor v, double b1, double b2, double eps, int64_t step,
                        torch::Tensor partial_ptrs, double extra_sq, double max_norm, torch::Tensor norm_out,
                        int64_t total) {
  RangeTable tab{offsets.data_ptr<int64_t>(), prefix.data_ptr<int64_t>(), (int)offsets.numel()};
  if (total == 0 || tab.n == 0) return;
  const float bc1 = 1.f - (float)std::pow(b1, (double)step);
  const float bc2s = (float)std::sqrt(1.0 - std::pow(b2, (double)step));
  dp_adamw_allgather_kernel<<<comm_grid(total / 4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      param_ptrs.data_ptr<int64_t>(), grad_ptrs.data_ptr<int64_t>(), (int)rank, (int)world, tab,
      wd.data_ptr<float>(), lr.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), (float)b1, (float)b2,
      (float)eps, bc1, bc2s, partial_ptrs.data_ptr<int64_t>(), (float)extra_sq, (float)max_norm,
      norm_out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_muon_prepare(torch::Tensor grad_ptrs, int64_t rank, int64_t world, torch::Tensor offs, int64_t numel,
                     torch::Tensor mom, double mu, bool nesterov, torch::Tensor out, torch::Tensor partial_ptrs,
                     double extra_sq, double max_norm) {
  const int n = offs.numel();
  if (n == 0) return;
  dp_muon_prepare_kernel<<<comm_grid((int64_t)n * numel), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      grad_ptrs.data_ptr<int64_t>(), (int)rank, (int)world, offs.data_ptr<int64_t>(), n, numel,
      mom.data_ptr<float>(), (float)mu, nesterov, (__nv_bfloat16*)out.data_ptr(), partial_ptrs.data_ptr<int64_t>(),
      (float)extra_sq, (float)max_norm);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_muon_apply_allgather(torch::Tensor param_ptrs, int64_t rank, int64_t world, torch::Tensor offs,
                             int64_t numel, double decay, double step_scale, torch::Tensor orth) {
  const int n = offs.numel();
  if (n == 0) return;
  dp_muon_apply_allgather_kernel<<<comm_grid((int64_t)n * numel), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      param_ptrs.data_ptr<int64_t>(), (int)rank, (int)world, offs.data_ptr<int64_t>(), n, numel, (float)decay,
      (float)step_scale, (const __nv_bfloat16*)orth.data_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void dp_muon_apply_shards(torch::Tensor param_ptrs, torch::Tensor bf16_ptrs, torch::Tensor poffs,
                          torch::Tensor boffs, int64_t rows, int64_t cols, int64_t rows_per_rank, double decay,
                          double step_scale, torch::Tensor orth) {
  const int n = poffs.numel();
  if (n == 0) return;
  TORCH_CHECK(cols % 8 == 0 && rows_per_rank > 0, "dp_muon_apply_shards: cols must be a multiple of 8");
  TORCH_CHECK(orth.is_contiguous() && orth.numel() == (int64_t)n * rows * cols, "dp_muon_apply_shards: orth shape");
  dp_muon_apply_shards_kernel<<<comm_grid((int64_t)n * rows * cols / 4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      param_ptrs.data_ptr<int64_t>(), bf16_ptrs.data_ptr<int64_t>(), poffs.data_ptr<int64_t>(),
      boffs.data_ptr<int64_t>(), n, (int)rows, (int)cols, (int)rows_per_rank, (float)decay, (float)step_scale,
      (const __nv_bfloat16*)orth.data_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void cast_ranges_bf16(torch::Tensor src, torch::Tensor dst, torch::Tensor src_offsets, torch::Tensor prefix,
                      torch::Tensor dst_offsets, int64_t total) {
  RangeTable tab{src_offsets.data_ptr<int64_t>(), prefix.data_ptr<int64_t>(), (int)src_offsets.numel()};
  if (total == 0 || tab.n == 0) return;
  TORCH_CHECK(src.scalar_type() == at::kFloat && dst.scalar_type() == at::kBFloat16, "cast_ranges_bf16: dtypes");
  cast_ranges_bf16_kernel<<<comm_grid(total / 4), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      src.data_ptr<float>(), (__nv_bfloat16*)dst.data_ptr(), tab, dst_offsets.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mx_shard_gather(torch::Tensor bases, int64_t R, int64_t K, int64_t N, torch::Tensor q0, torch::Tensor s0,
                     torch::Tensor q1, torch::Tensor s1) {
  auto b = bases.to(at::kCPU);
  const int world = (int)b.numel();
  TORCH_CHECK(b.scalar_type() == at::kLong && world >= 1 && world <= kMaxWorld, "mx_shard_gather: rank bases");
  TORCH_CHECK(R % 128 == 0 && K % 128 == 0 && N % 128 == 0 && R * world >= N, "mx_shard_gather: 128-multiples");
  TORCH_CHECK(q0.numel() == N * K && q1.numel() == N * K && s0.numel() == N * K / 32 && s1.numel() == N * K / 32,
              "mx_shard_gather: output sizes");
  MxGatherArgs a{};
  for (int r = 0; r < world; ++r) {
    a.base[r] = b.data_ptr<int64_t>()[r];
    TORCH_CHECK(a.base[r] % 16 == 0, "mx_shard_gather: 16-byte aligned copies");
  }
  a.q0 = q0.data_ptr<uint8_t>();
  a.s0 = s0.data_ptr<uint8_t>();
  a.q1 = q1.data_ptr<uint8_t>();
  a.s1 = s1.data_ptr<uint8_t>();
  a.R = R;
  a.K = K;
  a.N = N;
  const int64_t units = R * K / 16;
  dim3 grid((unsigned)std::min<int64_t>((units + 255) / 256, 148 * 2), world, 4);
  mx_shard_gather_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
