// Gated DeltaNet chunk gradient on the tcgen05 tensor cores (sm_100a).
//
// One CTA per (64-token chunk, head).  Inputs arrive by TMA in 128-byte-swizzled tiles
// (K^, Q^ rows of the chunk, dO, U, the state S0 entering the chunk, dS at its end, and
// T = (I + A)^-1 stored by the forward), every chunk product is a 64-row tcgen05 MMA
// issued by one thread with its fp32 accumulator in TMEM, and eight warps run the
// element-wise steps between the products on accumulator rows read with tcgen05.ld.
// The algebra is the one of the mma.sync kernel in gdn.cu (gdn_grad_kernel) and of the
// PyTorch statement in myk_llm_b200/ops/gdn_chunk.py:
//
//   P   = lower_incl(E * Q^K^T)                      dP  = dO U^T
//   dU  = P^T dO + F (K^ dS)                         dY  = T^T dU,  dV = beta dY
//   dA  = -(dY U^T) (strictly lower, times E)        dKK = beta dA,  dPE = dP * E
//   dQ^ = dPE K^ + e^gamma (dO S0^T)
//   dK^ = -e^gamma beta (dY S0^T) + dKK K^ + dKK^T K^ + dPE^T Q^ + F (U dS^T)
//
// followed by the l2-norm backward of q and k and the reverse cumulative sum of dgamma.
// Reference: the chunked gated delta rule of flash-linear-attention, which the reference
// framework calls from src/myk_llm/model/mixers.py (GatedDeltaNet).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gdn_geo.cuh"
#include "gdn_tc.cuh"
#include "tma_host.h"

namespace mykb {
namespace gtc {

constexpr int C = 64;
constexpr int NT = 256;

// Shared memory (bytes from a 1024-aligned base).
struct GradTcSm {
  static constexpr int kKH = 0;          // K^   64 x 128
  static constexpr int kQH = 16384;      // Q^   64 x 128
  static constexpr int kDO = 32768;      // dO   64 x 128
  static constexpr int kU = 49152;       // U    64 x 128
  static constexpr int kS0 = 65536;      // S0  128 x 128 (rows dk, columns dv)
  static constexpr int kDS = 98304;      // dS  128 x 128
  static constexpr int kT = 131072;      // T    64 x 64, then dKK
  static constexpr int kP = 139264;      // P    64 x 64, then dPE
  static constexpr int kDU = 147456;     // dU   64 x 128
  static constexpr int kDY = 163840;     // dY   64 x 128
  static constexpr int kScal = 180224;   // 10 x 64 floats
  static constexpr int kBars = kScal + 2560;
  static constexpr int kTotal = kBars + 128;
  static constexpr uint32_t kLoadBytes = 4 * 16384 + 2 * 32768 + 8192;  // KH QH DO U, S0 DS, T
};

// TMEM columns of the accumulators (64-row products, halves of NH columns at lane
// offsets 0 / 16).  Regions are reused once their readers have finished.
struct GradTcCols {
  static constexpr uint32_t kKK = 0;      // K^K^T        NH 32
  static constexpr uint32_t kQK = 32;     // Q^K^T        NH 32
  static constexpr uint32_t kKS = 64;     // K^ S0        NH 64, later dQ accumulator
  static constexpr uint32_t kKdS = 128;   // K^ dS        NH 64, later dY, later dK accumulator
  static constexpr uint32_t kDP = 192;    // dO U^T       NH 32
  static constexpr uint32_t kQS = 224;    // Q^ S0        NH 64
  static constexpr uint32_t kDOS = 288;   // dO S0^T      NH 64
  static constexpr uint32_t kUdS = 352;   // U dS^T       NH 64
  static constexpr uint32_t kPdO = 416;   // P^T dO       NH 64, later dA (NH 32)
  static constexpr uint32_t kDYS = 448;   // dY S0^T      NH 64 (issued after dA)
  static constexpr uint32_t kDY = kKdS;
  static constexpr uint32_t kDA = kPdO;
  static constexpr uint32_t kDQ = kKS;
  static constexpr uint32_t kDK = kKdS;
};

struct GradTcArgs {
  gdnk::Geo g;
  const bf16* q;
  const bf16* k;
  const bf16* v;
  const float* beta;   // (rows, heads)
  const float* gcum;   // head-major (heads, rows)
  const float* kinv;
  const float* qinv;
  bf16* dq;
  bf16* dk;
  bf16* dv;
  float* dg;
  float* db;
  float qscale;
  int* status;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int N>
__device__ __forceinline__ void to_f(const uint32_t (&r)[N], float (&f)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) f[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(NT, 1)
gdn_grad_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmDO, const __grid_constant__ CUtensorMap tmU,
                   const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmDS,
                   const __grid_constant__ CUtensorMap tmT, const GradTcArgs a) {
  using S = GradTcSm;
  using TC = GradTcCols;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const gdnk::Geo& g = a.g;
  const int chunk = blockIdx.x / g.heads, h = blockIdx.x % g.heads;
  int row0, n;
  if (!gdnk::locate(g, chunk, row0, n)) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* gam = reinterpret_cast<float*>(sm + S::kScal);
  float* eg = gam + 64;
  float* bet = gam + 128;
  float* ki = gam + 192;
  float* qi = gam + 256;
  float* fF = gam + 320;
  float* dgam = gam + 384;
  float* dbet = gam + 448;
  float* dotq = gam + 512;
  float* dotk = gam + 576;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kBars);  // load, A1, A2, B, C, D, E
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kBars + 8 * 8);
  const int64_t cbase = (int64_t)chunk * g.heads + h;
  const int64_t hb = (int64_t)h * g.rows + row0;

  if (tid == 0) {
    for (int i = 0; i < 7; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  if (tid < C) {
    gam[tid] = tid < n ? a.gcum[hb + tid] : 0.f;
    ki[tid] = tid < n ? a.kinv[hb + tid] : 0.f;
    qi[tid] = tid < n ? a.qinv[hb + tid] : 0.f;
    bet[tid] = tid < n ? a.beta[(int64_t)(row0 + tid) * g.heads + h] : 0.f;
    dgam[tid] = 0.f;
    dbet[tid] = 0.f;
    dotq[tid] = 0.f;
    dotk[tid] = 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sb = smem_u32(sm);
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], S::kLoadBytes);
    for (int cb = 0; cb < 2; ++cb) {
      tma_load_3d(sm + S::kKH + cb * 8192, &tmK, &bars[0], h * 128 + cb * 64, row0, 0);
      tma_load_3d(sm + S::kQH + cb * 8192, &tmQ, &bars[0], h * 128 + cb * 64, row0, 0);
      tma_load_3d(sm + S::kDO + cb * 8192, &tmDO, &bars[0], h * 128 + cb * 64, row0, 0);
      tma_load_3d(sm + S::kU + cb * 8192, &tmU, &bars[0], cb * 64, (int)(cbase * 64), 0);
      tma_load_3d(sm + S::kS0 + cb * 16384, &tmS, &bars[0], cb * 64, (int)(cbase * 128), 0);
      tma_load_3d(sm + S::kDS + cb * 16384, &tmDS, &bars[0], cb * 64, (int)(cbase * 128), 0);
    }
    tma_load_3d(sm + S::kT, &tmT, &bars[0], 0, (int)(cbase * 64), 0);
  }
  bool ok = mbar_wait_warp(&bars[0], 0, a.status, __LINE__);
  ok = __syncthreads_and(ok);
  if (ok) {
    // gamma past the chunk's end repeats gamma_{n-1}; e^gamma; F_t = e^{gamma_C - gamma_t}
    const float glast = gam[n - 1];
    if (tid < C) {
      const float gv = tid < n ? gam[tid] : glast;
      eg[tid] = __expf(gv);
      fF[tid] = tid < n ? __expf(glast - gv) : 0.f;
    }
    __syncthreads();
    if (tid < C && tid >= n) gam[tid] = glast;
    // K^ = k / |k|, Q^ = c q / |q| (rows past n zero); dO rows past n zero
    for (int i = tid; i < 3 * 2 * 64 * 8; i += NT) {
      const int t = i / (2 * 64 * 8), rem = i % (2 * 64 * 8);
      const int r = (rem >> 3) & 63;
      uint4* p = reinterpret_cast<uint4*>(sm + (t == 0 ? S::kKH : t == 1 ? S::kQH : S::kDO) + rem * 16);
      if (r >= n) {
        *p = make_uint4(0, 0, 0, 0);
      } else if (t < 2) {
        const float sc = t == 0 ? ki[r] : qi[r];
        uint4 w = *p;
        uint32_t* u = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u[e]));
          u[e] = pack_bf16x2(f.x * sc, f.y * sc);
        }
        *p = w;
      }
    }
    {  // dgamma_C += e^{gamma_C} <S0, dS>  (same swizzle in both tiles: compare bytes in place)
      float dot = 0.f;
      for (int i = tid; i < 32768 / 16; i += NT) {
        const uint4 x = reinterpret_cast<const uint4*>(sm + S::kS0)[i];
        const uint4 y = reinterpret_cast<const uint4*>(sm + S::kDS)[i];
        const uint32_t xa[4] = {x.x, x.y, x.z, x.w}, ya[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 xf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xa[e]));
          const float2 yf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ya[e]));
          dot += xf.x * yf.x + xf.y * yf.y;
        }
      }
      dot = warp_sum(dot);
      if (lane == 0) atomicAdd(&dgam[C - 1], __expf(glast) * dot);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();

  const uint32_t aKH = sb + S::kKH, aQH = sb + S::kQH, aDO = sb + S::kDO, aU = sb + S::kU, aS0 = sb + S::kS0,
                 aDS = sb + S::kDS, aT = sb + S::kT, aP = sb + S::kP, aDU = sb + S::kDU, aDY = sb + S::kDY;
  if (ok && tid == 0) {
    tc_fence_after();
    // A1: K^K^T, Q^K^T, K^ dS
    mma64<32, 8, false, false>(tmem, TC::kKK, [&](int kk) { return desc_k(aKH, 64, 0, kk); },
                               [&](int hf, int kk) { return desc_k(aKH, 64, 32 * hf, kk); }, false);
    mma64<32, 8, false, false>(tmem, TC::kQK, [&](int kk) { return desc_k(aQH, 64, 0, kk); },
                               [&](int hf, int kk) { return desc_k(aKH, 64, 32 * hf, kk); }, false);
    mma64<64, 8, false, true>(tmem, TC::kKdS, [&](int kk) { return desc_k(aKH, 64, 0, kk); },
                              [&](int hf, int kk) { return desc_mn(aDS, 128, 64 * hf, kk); }, false);
    umma_commit(&bars[1]);
    // A2: K^ S0, dO U^T, Q^ S0, dO S0^T, U dS^T
    mma64<64, 8, false, true>(tmem, TC::kKS, [&](int kk) { return desc_k(aKH, 64, 0, kk); },
                              [&](int hf, int kk) { return desc_mn(aS0, 128, 64 * hf, kk); }, false);
    mma64<32, 8, false, false>(tmem, TC::kDP, [&](int kk) { return desc_k(aDO, 64, 0, kk); },
                               [&](int hf, int kk) { return desc_k(aU, 64, 32 * hf, kk); }, false);
    mma64<64, 8, false, true>(tmem, TC::kQS, [&](int kk) { return desc_k(aQH, 64, 0, kk); },
                              [&](int hf, int kk) { return desc_mn(aS0, 128, 64 * hf, kk); }, false);
    mma64<64, 8, false, false>(tmem, TC::kDOS, [&](int kk) { return desc_k(aDO, 64, 0, kk); },
                               [&](int hf, int kk) { return desc_k(aS0, 128, 64 * hf, kk); }, false);
    mma64<64, 8, false, false>(tmem, TC::kUdS, [&](int kk) { return desc_k(aU, 64, 0, kk); },
                               [&](int hf, int kk) { return desc_k(aDS, 128, 64 * hf, kk); }, false);
    umma_commit(&bars[2]);
  }

  const int r = acc_row();
  // ---- epilogue A: P = lower_incl(E * Q^K^T)
  if (ok) {
    ok = mbar_wait_warp(&bars[1], 0, a.status, __LINE__);
    if (ok) {
      tc_fence_after();
      const int c0 = acc_col0(32);
      uint32_t raw[16];
      tmem_ld16_raw(acc_addr(tmem, TC::kQK, 32), raw);
      tmem_wait_ld();
      float p[16];
      const float gr = gam[r];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = c0 + j;
        p[j] = c <= r ? __expf(gr - gam[c]) * __uint_as_float(raw[j]) : 0.f;
      }
      st8(sm + S::kP, 64, r, c0, p);
      st8(sm + S::kP, 64, r, c0 + 8, p + 8);
      fence_proxy_async_smem();
    }
  }
  tc_fence_before();
  ok = __syncthreads_and(ok);
  if (ok && tid == 0) {
    tc_fence_after();
    // B: P^T dO
    mma64<64, 4, true, true>(tmem, TC::kPdO, [&](int kk) { return desc_mn(aP, 64, 0, kk); },
                             [&](int hf, int kk) { return desc_mn(aDO, 64, 64 * hf, kk); }, false);
    umma_commit(&bars[3]);
  }
  // ---- epilogue B: dU = P^T dO + F (K^ dS); dF
  if (ok) {
    ok = mbar_wait_warp(&bars[3], 0, a.status, __LINE__);
    if (ok) {
      tc_fence_after();
      const int c0 = acc_col0(64);
      uint32_t r1[32], r2[32];
      tmem_ld32_raw(acc_addr(tmem, TC::kPdO, 64), r1);
      tmem_ld32_raw(acc_addr(tmem, TC::kKdS, 64), r2);
      tmem_wait_ld();
      float u[32], du[32];
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) ld8(sm + S::kU, 64, r, c0 + 8 * q8, u + 8 * q8);
      const float fr = fF[r];
      float d = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float kd = __uint_as_float(r2[j]);
        du[j] = __uint_as_float(r1[j]) + fr * kd;
        d += kd * u[j];
      }
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) st8(sm + S::kDU, 64, r, c0 + 8 * q8, du + 8 * q8);
      d *= fr;
      atomicAdd(&dgam[r], -d);
      d = warp_sum(d);
      if (lane == 0) atomicAdd(&dgam[C - 1], d);
      fence_proxy_async_smem();
    }
  }
  tc_fence_before();
  ok = __syncthreads_and(ok);
  if (ok && tid == 0) {
    tc_fence_after();
    // C: dY = T^T dU
    mma64<64, 4, true, true>(tmem, TC::kDY, [&](int kk) { return desc_mn(aT, 64, 0, kk); },
                             [&](int hf, int kk) { return desc_mn(aDU, 64, 64 * hf, kk); }, false);
    umma_commit(&bars[4]);
  }
  // ---- epilogue C: dY, dV = beta dY, dbeta, dgamma
  if (ok) {
    ok = mbar_wait_warp(&bars[4], 0, a.status, __LINE__) && mbar_wait_warp(&bars[2], 0, a.status, __LINE__);
    if (ok) {
      tc_fence_after();
      const int c0 = acc_col0(64);
      uint32_t r1[32], r2[32];
      tmem_ld32_raw(acc_addr(tmem, TC::kDY, 64), r1);
      tmem_ld32_raw(acc_addr(tmem, TC::kKS, 64), r2);
      tmem_wait_ld();
      float dy[32], vv[32];
      to_f(r1, dy);
      const bool valid = r < n;
      const bf16* vrow = a.v + (int64_t)(row0 + r) * g.row_v + (int64_t)h * 128 + c0;
      bf16* dvrow = a.dv + (int64_t)(row0 + r) * g.row_v + (int64_t)h * 128 + c0;
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        uint4 w = valid ? *reinterpret_cast<const uint4*>(vrow + 8 * q8) : make_uint4(0, 0, 0, 0);
        const uint32_t wa[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wa[e]));
          vv[8 * q8 + 2 * e] = f.x;
          vv[8 * q8 + 2 * e + 1] = f.y;
        }
      }
      const float br = bet[r], er = eg[r];
      float dbp = 0.f, dkp = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float ks = __uint_as_float(r2[j]);
        dbp += dy[j] * (vv[j] - er * ks);
        dkp += ks * dy[j];
      }
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        st8(sm + S::kDY, 64, r, c0 + 8 * q8, dy + 8 * q8);
        if (valid) {
          uint4 w;
          w.x = pack_bf16x2(br * dy[8 * q8 + 0], br * dy[8 * q8 + 1]);
          w.y = pack_bf16x2(br * dy[8 * q8 + 2], br * dy[8 * q8 + 3]);
          w.z = pack_bf16x2(br * dy[8 * q8 + 4], br * dy[8 * q8 + 5]);
          w.w = pack_bf16x2(br * dy[8 * q8 + 6], br * dy[8 * q8 + 7]);
          *reinterpret_cast<uint4*>(dvrow + 8 * q8) = w;
        }
      }
      atomicAdd(&dbet[r], dbp);
      atomicAdd(&dgam[r], -er * br * dkp);
      fence_proxy_async_smem();
    }
  }
  tc_fence_before();
  ok = __syncthreads_and(ok);
  if (ok && tid == 0) {
    tc_fence_after();
    // D: dA = dY U^T; then dY S0^T (read in epilogue E)
    mma64<32, 8, false, false>(tmem, TC::kDA, [&](int kk) { return desc_k(aDY, 64, 0, kk); },
                               [&](int hf, int kk) { return desc_k(aU, 64, 32 * hf, kk); }, false);
    umma_commit(&bars[5]);
    mma64<64, 8, false, false>(tmem, TC::kDYS, [&](int kk) { return desc_k(aDY, 64, 0, kk); },
                               [&](int hf, int kk) { return desc_k(aS0, 128, 64 * hf, kk); }, false);
  }
  // ---- epilogue D: dKK (into T's tile), dPE (into P's tile), dbeta, dgamma rows and columns
  if (ok) {
    ok = mbar_wait_warp(&bars[5], 0, a.status, __LINE__);
    if (ok) {
      tc_fence_after();
      const int c0 = acc_col0(32);
      uint32_t rA[16], rP[16], rK[16], rQ[16];
      tmem_ld16_raw(acc_addr(tmem, TC::kDA, 32), rA);
      tmem_ld16_raw(acc_addr(tmem, TC::kDP, 32), rP);
      tmem_ld16_raw(acc_addr(tmem, TC::kKK, 32), rK);
      tmem_ld16_raw(acc_addr(tmem, TC::kQK, 32), rQ);
      tmem_wait_ld();
      const int t = r;
      const float gt = gam[t], bt = bet[t];
      float dkk[16], dpe[16], colg[16];
      float rowb = 0.f, rowg = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = c0 + j;
        const float ex = c <= t ? __expf(gt - gam[c]) : 0.f;
        const float kk = __uint_as_float(rK[j]);
        float gs = 0.f;
        dkk[j] = 0.f;
        if (c < t) {
          const float dae = -__uint_as_float(rA[j]) * ex;
          rowb += dae * kk;
          dkk[j] = dae * bt;
          gs += dkk[j] * kk;
        }
        dpe[j] = __uint_as_float(rP[j]) * ex;
        gs += dpe[j] * __uint_as_float(rQ[j]);
        rowg += gs;
        colg[j] = -gs;
      }
      st8(sm + S::kT, 64, t, c0, dkk);
      st8(sm + S::kT, 64, t, c0 + 8, dkk + 8);
      st8(sm + S::kP, 64, t, c0, dpe);
      st8(sm + S::kP, 64, t, c0 + 8, dpe + 8);
      atomicAdd(&dbet[t], rowb);
      atomicAdd(&dgam[t], rowg);
      // column sums over the 16 rows of this lane's half (lanes sharing lane / 16)
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float v = colg[j];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        colg[j] = v;
      }
      if ((lane & 15) == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) atomicAdd(&dgam[c0 + j], colg[j]);
      }
      fence_proxy_async_smem();
    }
  }
  tc_fence_before();
  ok = __syncthreads_and(ok);
  if (ok && tid == 0) {
    tc_fence_after();
    // E: dQ acc = dPE K^;  dK acc = dKK K^ + dKK^T K^ + dPE^T Q^
    mma64<64, 4, false, true>(tmem, TC::kDQ, [&](int kk) { return desc_k(aP, 64, 0, kk); },
                              [&](int hf, int kk) { return desc_mn(aKH, 64, 64 * hf, kk); }, false);
    mma64<64, 4, false, true>(tmem, TC::kDK, [&](int kk) { return desc_k(aT, 64, 0, kk); },
                              [&](int hf, int kk) { return desc_mn(aKH, 64, 64 * hf, kk); }, false);
    mma64<64, 4, true, true>(tmem, TC::kDK, [&](int kk) { return desc_mn(aT, 64, 0, kk); },
                             [&](int hf, int kk) { return desc_mn(aKH, 64, 64 * hf, kk); }, true);
    mma64<64, 4, true, true>(tmem, TC::kDK, [&](int kk) { return desc_mn(aP, 64, 0, kk); },
                             [&](int hf, int kk) { return desc_mn(aQH, 64, 64 * hf, kk); }, true);
    umma_commit(&bars[6]);
  }
  // ---- epilogue E: dQ^, dK^, their l2-norm backward, dgamma of the inter-chunk term
  if (ok) {
    ok = mbar_wait_warp(&bars[6], 0, a.status, __LINE__);
  }
  float dqv[32], dkv[32];
  const int c0 = acc_col0(64);
  if (ok) {
    tc_fence_after();
    const float er = eg[r], br = bet[r], fr = fF[r];
    uint32_t r1[32], r2[32];
    float x[32];
    tmem_ld32_raw(acc_addr(tmem, TC::kDQ, 64), r1);
    tmem_ld32_raw(acc_addr(tmem, TC::kDOS, 64), r2);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) dqv[j] = __uint_as_float(r1[j]) + er * __uint_as_float(r2[j]);
    tmem_ld32_raw(acc_addr(tmem, TC::kQS, 64), r1);
    tmem_wait_ld();
    float gq = 0.f, qd = 0.f;
#pragma unroll
    for (int q8 = 0; q8 < 4; ++q8) ld8(sm + S::kDO, 64, r, c0 + 8 * q8, x + 8 * q8);
#pragma unroll
    for (int j = 0; j < 32; ++j) gq += __uint_as_float(r1[j]) * x[j];
#pragma unroll
    for (int q8 = 0; q8 < 4; ++q8) ld8(sm + S::kQH, 64, r, c0 + 8 * q8, x + 8 * q8);
#pragma unroll
    for (int j = 0; j < 32; ++j) qd += x[j] * dqv[j];
    atomicAdd(&dgam[r], er * gq);
    atomicAdd(&dotq[r], qd);
    tmem_ld32_raw(acc_addr(tmem, TC::kDK, 64), r1);
    tmem_ld32_raw(acc_addr(tmem, TC::kDYS, 64), r2);
    tmem_wait_ld();
    const float sy = -er * br;
#pragma unroll
    for (int j = 0; j < 32; ++j) dkv[j] = __uint_as_float(r1[j]) + sy * __uint_as_float(r2[j]);
    tmem_ld32_raw(acc_addr(tmem, TC::kUdS, 64), r1);
    tmem_wait_ld();
    float kd = 0.f;
#pragma unroll
    for (int q8 = 0; q8 < 4; ++q8) ld8(sm + S::kKH, 64, r, c0 + 8 * q8, x + 8 * q8);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      dkv[j] += fr * __uint_as_float(r1[j]);
      kd += x[j] * dkv[j];
    }
    atomicAdd(&dotk[r], kd);
  }
  tc_fence_before();
  ok = __syncthreads_and(ok);
  if (ok) {
    // l2-norm backward: q^ = c q / |q| (qi = c / |q|): dq = qi (dq^ - q^ (q^.dq^) / c^2);
    // k^ = k / |k| (ki = 1 / |k|): dk = ki (dk^ - k^ (k^.dk^))
    if (r < n) {
      const float qr = qi[r], kr = ki[r], tq = dotq[r] / (a.qscale * a.qscale), tk = dotk[r];
      const int64_t ob = (int64_t)(row0 + r) * g.row_q + (int64_t)h * 128 + c0;
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        const uint4 qw = *reinterpret_cast<const uint4*>(a.q + ob + 8 * q8);
        const uint4 kw = *reinterpret_cast<const uint4*>(a.k + ob + 8 * q8);
        const uint32_t qa[4] = {qw.x, qw.y, qw.z, qw.w}, ka[4] = {kw.x, kw.y, kw.z, kw.w};
        uint32_t oq[4], ok4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 qf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qa[e]));
          const float2 kf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ka[e]));
          const int j = 8 * q8 + 2 * e;
          oq[e] = pack_bf16x2(qr * (dqv[j] - qf.x * qr * tq), qr * (dqv[j + 1] - qf.y * qr * tq));
          ok4[e] = pack_bf16x2(kr * (dkv[j] - kf.x * kr * tk), kr * (dkv[j + 1] - kf.y * kr * tk));
        }
        *reinterpret_cast<uint4*>(a.dq + ob + 8 * q8) = make_uint4(oq[0], oq[1], oq[2], oq[3]);
        *reinterpret_cast<uint4*>(a.dk + ob + 8 * q8) = make_uint4(ok4[0], ok4[1], ok4[2], ok4[3]);
      }
    }
    if (warp == 0) {  // dg = reverse cumulative sum of dgamma over the chunk; dbeta
      const int i0 = 2 * lane, i1 = 2 * lane + 1;
      const float x0 = dgam[i0], x1 = dgam[i1];
      float c = x0 + x1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(0xffffffffu, c, o);
        if (lane + o < 32) c += y;
      }
      if (i0 < n) {
        a.dg[(int64_t)(row0 + i0) * g.heads + h] = c;
        a.db[(int64_t)(row0 + i0) * g.heads + h] = dbet[i0];
      }
      if (i1 < n) {
        a.dg[(int64_t)(row0 + i1) * g.heads + h] = c - x0;
        a.db[(int64_t)(row0 + i1) * g.heads + h] = dbet[i1];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------ forward
// gdn_prep_tc: per (chunk, head): gamma = cumsum(g), the key / query norms, A =
// strictly_lower(beta E * K^K^T), T = (I + A)^-1 (fp32 blocked forward substitution on
// the CUDA cores), W = T diag(beta e^gamma) K^ and U~ = T diag(beta) V (tcgen05).
struct PrepTcSm {
  static constexpr int kKH = 0;        // K -> K^            64 x 128
  static constexpr int kKB = 16384;    // beta e^gamma K^    64 x 128
  static constexpr int kVB = 32768;    // V -> beta V        64 x 128
  static constexpr int kT = 49152;     // T (bf16)           64 x 64
  static constexpr int kA = 57344;     // A (fp32, row stride 65)
  static constexpr int kTf = kA + 64 * 65 * 4;
  static constexpr int kX = kTf + 64 * 65 * 4;  // 768 floats of inversion scratch
  static constexpr int kScal = kX + 768 * 4;    // gam, eg, bet
  static constexpr int kBars = kScal + 3 * 256;
  static constexpr int kTotal = kBars + 64;
};
constexpr int LDA = 65;

struct PrepTcArgs {
  gdnk::Geo g;
  const bf16* q;
  const float* gg;    // (rows, heads) log decay
  const float* bb;    // (rows, heads) beta
  float* gcum;        // head-major outputs
  float* kinv;
  float* qinv;
  bf16* w_out;        // (chunks, heads, 64, 128)
  bf16* u_out;
  bf16* t_out;        // (chunks, heads, 64, 64)
  float qscale;
  int* status;
};

// T = (I + A)^-1 for the strictly lower A (fp32, row stride LDA) by 16 x 16 blocks:
// diagonal blocks by forward substitution (one thread per block column), then
// T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj level by level.  Ends synchronised.
__device__ void invert_lower_from_a(const float* A, float* Tf, float* X) {
  const int tid = threadIdx.x;
  for (int i = tid; i < C * LDA; i += NT) Tf[i] = 0.f;
  __syncthreads();
  if (tid < C) {
    const int base = (tid >> 4) * 16, j = tid & 15;
    Tf[(base + j) * LDA + base + j] = 1.f;
    for (int i = j + 1; i < 16; ++i) {
      float s = 0.f;
      for (int k = j; k < i; ++k) s = fmaf(A[(base + i) * LDA + base + k], Tf[(base + k) * LDA + base + j], s);
      Tf[(base + i) * LDA + base + j] = -s;
    }
  }
  __syncthreads();
  for (int d = 1; d < 4; ++d) {
    const int nb = 4 - d;
    for (int e = tid; e < nb * 256; e += NT) {
      const int bj = e >> 8, bi = bj + d, i = (e >> 4) & 15, j = e & 15;
      const float* arow = A + (bi * 16 + i) * LDA;
      float s = 0.f;
      for (int k = bj * 16; k < bi * 16; ++k) s = fmaf(arow[k], Tf[k * LDA + bj * 16 + j], s);
      X[e] = s;
    }
    __syncthreads();
    for (int e = tid; e < nb * 256; e += NT) {
      const int bj = e >> 8, bi = bj + d, i = (e >> 4) & 15, j = e & 15;
      float s = 0.f;
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) s = fmaf(Tf[(bi * 16 + i) * LDA + bi * 16 + kk], X[(bj << 8) + kk * 16 + j], s);
      Tf[(bi * 16 + i) * LDA + bj * 16 + j] = -s;
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(NT, 2)
gdn_prep_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const PrepTcArgs a) {
  using S = PrepTcSm;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const gdnk::Geo& g = a.g;
  const int chunk = blockIdx.x / g.heads, h = blockIdx.x % g.heads;
  int row0, n;
  if (!gdnk::locate(g, chunk, row0, n)) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* gam = reinterpret_cast<float*>(sm + S::kScal);
  float* eg = gam + 64;
  float* bet = gam + 128;
  float* Af = reinterpret_cast<float*>(sm + S::kA);
  float* Tf = reinterpret_cast<float*>(sm + S::kTf);
  float* X = reinterpret_cast<float*>(sm + S::kX);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kBars);  // load, KK, W/U
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kBars + 32);
  const int64_t cbase = (int64_t)chunk * g.heads + h;
  const int64_t hb = (int64_t)h * g.rows + row0;
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], 2 * 16384);
    for (int cb = 0; cb < 2; ++cb) {
      tma_load_3d(sm + S::kKH + cb * 8192, &tmK, &bars[0], h * 128 + cb * 64, row0, 0);
      tma_load_3d(sm + S::kVB + cb * 8192, &tmV, &bars[0], h * 128 + cb * 64, row0, 0);
    }
  }
  if (warp == 0) {  // gamma = inclusive cumsum of g over the chunk; beta
    const int i0 = 2 * lane, i1 = 2 * lane + 1;
    const float x0 = i0 < n ? a.gg[(int64_t)(row0 + i0) * g.heads + h] : 0.f;
    const float x1 = i1 < n ? a.gg[(int64_t)(row0 + i1) * g.heads + h] : 0.f;
    float c = x0 + x1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, c, o);
      if (lane >= o) c += y;
    }
    const float c0 = c - x1;
    gam[i0] = c0;
    gam[i1] = c;
    eg[i0] = __expf(c0);
    eg[i1] = __expf(c);
    bet[i0] = i0 < n ? a.bb[(int64_t)(row0 + i0) * g.heads + h] : 0.f;
    bet[i1] = i1 < n ? a.bb[(int64_t)(row0 + i1) * g.heads + h] : 0.f;
    if (i0 < n) a.gcum[hb + i0] = c0;
    if (i1 < n) a.gcum[hb + i1] = c;
  } else {  // query norms (rows over warps 1..7), straight from global memory
    for (int r = warp - 1; r < n; r += NT / 32 - 1) {
      const uint2 w = *reinterpret_cast<const uint2*>(a.q + (int64_t)(row0 + r) * g.row_q + (int64_t)h * 128 + lane * 4);
      const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
      const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
      const float sq = warp_sum(x.x * x.x + x.y * x.y + y.x * y.x + y.y * y.y);
      if (lane == 0) a.qinv[hb + r] = a.qscale / fmaxf(sqrtf(sq), 1e-6f);
    }
  }
  bool ok = mbar_wait_warp(&bars[0], 0, a.status, __LINE__);
  ok = __syncthreads_and(ok);
  if (ok) {  // K^ = k / |k|, beta e^gamma K^, beta V; rows past n zero
    for (int r = warp; r < C; r += NT / 32) {
      const uint32_t off = sw_off(64, r, lane * 4);
      uint2* kp = reinterpret_cast<uint2*>(sm + S::kKH + off);
      uint2* vp = reinterpret_cast<uint2*>(sm + S::kVB + off);
      const uint2 kw = *kp, vw = *vp;
      const float2 k0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kw.x));
      const float2 k1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kw.y));
      const float2 v0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vw.x));
      const float2 v1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vw.y));
      const float sk = warp_sum(k0.x * k0.x + k0.y * k0.y + k1.x * k1.x + k1.y * k1.y);
      const bool valid = r < n;
      const float ik = valid ? 1.f / fmaxf(sqrtf(sk), 1e-6f) : 0.f;
      if (lane == 0 && valid) a.kinv[hb + r] = ik;
      const float kbs = valid ? bet[r] * eg[r] * ik : 0.f, bv = valid ? bet[r] : 0.f;
      *kp = valid ? make_uint2(pack_bf16x2(k0.x * ik, k0.y * ik), pack_bf16x2(k1.x * ik, k1.y * ik)) : make_uint2(0, 0);
      *reinterpret_cast<uint2*>(sm + S::kKB + off) =
          valid ? make_uint2(pack_bf16x2(k0.x * kbs, k0.y * kbs), pack_bf16x2(k1.x * kbs, k1.y * kbs)) : make_uint2(0, 0);
      *vp = valid ? make_uint2(pack_bf16x2(v0.x * bv, v0.y * bv), pack_bf16x2(v1.x * bv, v1.y * bv)) : make_uint2(0, 0);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  const uint32_t sb = smem_u32(sm);
  const uint32_t aKH = sb + S::kKH, aKB = sb + S::kKB, aVB = sb + S::kVB, aT = sb + S::kT;
  if (ok && tid == 0) {
    tc_fence_after();
    mma64<32, 8, false, false>(tmem, 0, [&](int kk) { return desc_k(aKH, 64, 0, kk); },
                               [&](int hf, int kk) { return desc_k(aKH, 64, 32 * hf, kk); }, false);
    umma_commit(&bars[1]);
  }
  const int r = acc_row();
  if (ok) {  // A = strictly_lower(beta_r e^{gamma_r - gamma_c} K^K^T)
    ok = mbar_wait_warp(&bars[1], 0, a.status, __LINE__);
    if (ok) {
      tc_fence_after();
      const int c0 = acc_col0(32);
      uint32_t raw[16];
      tmem_ld16_raw(acc_addr(tmem, 0, 32), raw);
      tmem_wait_ld();
      const float br = bet[r], gr = gam[r];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = c0 + j;
        Af[r * LDA + c] = c < r ? br * __expf(gr - gam[c]) * __uint_as_float(raw[j]) : 0.f;
      }
    }
  }
  tc_fence_before();
  ok = __syncthreads_and(ok);
  if (ok) {
    invert_lower_from_a(Af, Tf, X);
    for (int i = tid; i < C * 8; i += NT) {  // T -> bf16 operand tile and global memory
      const int rr = i >> 3, c = (i & 7) * 8;
      float v8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v8[e] = Tf[rr * LDA + c + e];
      st8(sm + S::kT, 64, rr, c, v8);
      *reinterpret_cast<uint4*>(a.t_out + cbase * C * C + rr * C + c) =
          *reinterpret_cast<const uint4*>(sm + S::kT + sw_off(64, rr, c));
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  if (ok && tid == 0) {
    tc_fence_after();
    mma64<64, 4, false, true>(tmem, 32, [&](int kk) { return desc_k(aT, 64, 0, kk); },
                              [&](int hf, int kk) { return desc_mn(aKB, 64, 64 * hf, kk); }, false);
    mma64<64, 4, false, true>(tmem, 96, [&](int kk) { return desc_k(aT, 64, 0, kk); },
                              [&](int hf, int kk) { return desc_mn(aVB, 64, 64 * hf, kk); }, false);
    umma_commit(&bars[2]);
  }
  if (ok) {  // W, U~ rows to global memory
    ok = mbar_wait_warp(&bars[2], 0, a.status, __LINE__);
    if (ok) {
      tc_fence_after();
      const int c0 = acc_col0(64);
      uint32_t rw[32], ru[32];
      tmem_ld32_raw(acc_addr(tmem, 32, 64), rw);
      tmem_ld32_raw(acc_addr(tmem, 96, 64), ru);
      tmem_wait_ld();
      bf16* wo = a.w_out + cbase * C * 128 + r * 128 + c0;
      bf16* uo = a.u_out + cbase * C * 128 + r * 128 + c0;
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        const int j = 8 * q8;
        *reinterpret_cast<uint4*>(wo + j) =
            make_uint4(pack_bf16x2(__uint_as_float(rw[j]), __uint_as_float(rw[j + 1])),
                       pack_bf16x2(__uint_as_float(rw[j + 2]), __uint_as_float(rw[j + 3])),
                       pack_bf16x2(__uint_as_float(rw[j + 4]), __uint_as_float(rw[j + 5])),
                       pack_bf16x2(__uint_as_float(rw[j + 6]), __uint_as_float(rw[j + 7])));
        *reinterpret_cast<uint4*>(uo + j) =
            make_uint4(pack_bf16x2(__uint_as_float(ru[j]), __uint_as_float(ru[j + 1])),
                       pack_bf16x2(__uint_as_float(ru[j + 2]), __uint_as_float(ru[j + 3])),
                       pack_bf16x2(__uint_as_float(ru[j + 4]), __uint_as_float(ru[j + 5])),
                       pack_bf16x2(__uint_as_float(ru[j + 6]), __uint_as_float(ru[j + 7])));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// gdn_out_tc: P = lower_incl(E * Q^K^T) (also stored for the backward's dS recurrence),
// O = diag(e^gamma) Q^ S0 + P U.
struct OutTcSm {
  static constexpr int kQH = 0;        // Q^   64 x 128
  static constexpr int kKH = 16384;    // K^   64 x 128
  static constexpr int kU = 32768;     // U    64 x 128
  static constexpr int kS0 = 49152;    // S0  128 x 128
  static constexpr int kP = 81920;     // P    64 x 64
  static constexpr int kScal = 90112;  // gam, eg, ki, qi
  static constexpr int kBars = kScal + 4 * 256;
  static constexpr int kTotal = kBars + 64;
};

struct OutTcArgs {
  gdnk::Geo g;
  const float* gcum;
  const float* kinv;
  const float* qinv;
  bf16* p_out;   // (chunks, heads, 64, 64)
  bf16* out;     // (rows, heads, 128)
  int* status;
};

__global__ void __launch_bounds__(NT, 2)
gdn_out_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmU, const __grid_constant__ CUtensorMap tmS,
                  const OutTcArgs a) {
  using S = OutTcSm;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const gdnk::Geo& g = a.g;
  const int chunk = blockIdx.x / g.heads, h = blockIdx.x % g.heads;
  int row0, n;
  if (!gdnk::locate(g, chunk, row0, n)) return;
  const int tid = threadIdx.x, warp = tid >> 5;
  float* gam = reinterpret_cast<float*>(sm + S::kScal);
  float* eg = gam + 64;
  float* ki = gam + 128;
  float* qi = gam + 192;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kBars);  // load, QK/QS, PU
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kBars + 32);
  const int64_t cbase = (int64_t)chunk * g.heads + h;
  const int64_t hb = (int64_t)h * g.rows + row0;
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 256);
  if (tid < C) {
    gam[tid] = tid < n ? a.gcum[hb + tid] : 0.f;
    ki[tid] = tid < n ? a.kinv[hb + tid] : 0.f;
    qi[tid] = tid < n ? a.qinv[hb + tid] : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], 3 * 16384 + 32768);
    for (int cb = 0; cb < 2; ++cb) {
      tma_load_3d(sm + S::kQH + cb * 8192, &tmQ, &bars[0], h * 128 + cb * 64, row0, 0);
      tma_load_3d(sm + S::kKH + cb * 8192, &tmK, &bars[0], h * 128 + cb * 64, row0, 0);
      tma_load_3d(sm + S::kU + cb * 8192, &tmU, &bars[0], cb * 64, (int)(cbase * 64), 0);
      tma_load_3d(sm + S::kS0 + cb * 16384, &tmS, &bars[0], cb * 64, (int)(cbase * 128), 0);
    }
  }
  const float glast = gam[n - 1];
  if (tid < C) eg[tid] = __expf(tid < n ? gam[tid] : glast);
  bool ok = mbar_wait_warp(&bars[0], 0, a.status, __LINE__);
  ok = __syncthreads_and(ok);
  if (tid < C && tid >= n) gam[tid] = glast;
  if (ok) {  // Q^ = qi q, K^ = ki k; rows past n zero
    for (int i = tid; i < 2 * 2 * 64 * 8; i += NT) {
      const int t = i / (2 * 64 * 8), rem = i % (2 * 64 * 8);
      const int rr = (rem >> 3) & 63;
      uint4* p = reinterpret_cast<uint4*>(sm + (t == 0 ? S::kQH : S::kKH) + rem * 16);
      if (rr >= n) {
        *p = make_uint4(0, 0, 0, 0);
      } else {
        const float sc = t == 0 ? qi[rr] : ki[rr];
        uint4 w = *p;
        uint32_t* u = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u[e]));
          u[e] = pack_bf16x2(f.x * sc, f.y * sc);
        }
        *p = w;
      }
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  const uint32_t sb = smem_u32(sm);
  const uint32_t aQH = sb + S::kQH, aKH = sb + S::kKH, aU = sb + S::kU, aS0 = sb + S::kS0, aP = sb + S::kP;
  if (ok && tid == 0) {
    tc_fence_after();
    mma64<32, 8, false, false>(tmem, 0, [&](int kk) { return desc_k(aQH, 64, 0, kk); },
                               [&](int hf, int kk) { return desc_k(aKH, 64, 32 * hf, kk); }, false);
    umma_commit(&bars[1]);
    mma64<64, 8, false, true>(tmem, 32, [&](int kk) { return desc_k(aQH, 64, 0, kk); },
                              [&](int hf, int kk) { return desc_mn(aS0, 128, 64 * hf, kk); }, false);
  }
  const int r = acc_row();
  if (ok) {
    ok = mbar_wait_warp(&bars[1], 0, a.status, __LINE__);
    if (ok) {
      tc_fence_after();
      const int c0 = acc_col0(32);
      uint32_t raw[16];
      tmem_ld16_raw(acc_addr(tmem, 0, 32), raw);
      tmem_wait_ld();
      float p[16];
      const float gr = gam[r];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = c0 + j;
        p[j] = c <= r ? __expf(gr - gam[c]) * __uint_as_float(raw[j]) : 0.f;
      }
      st8(sm + S::kP, 64, r, c0, p);
      st8(sm + S::kP, 64, r, c0 + 8, p + 8);
      bf16* pg = a.p_out + cbase * C * C + r * C + c0;
      *reinterpret_cast<uint4*>(pg) = *reinterpret_cast<const uint4*>(sm + S::kP + sw_off(64, r, c0));
      *reinterpret_cast<uint4*>(pg + 8) = *reinterpret_cast<const uint4*>(sm + S::kP + sw_off(64, r, c0 + 8));
      fence_proxy_async_smem();
    }
  }
  tc_fence_before();
  ok = __syncthreads_and(ok);
  if (ok && tid == 0) {
    tc_fence_after();
    mma64<64, 4, false, true>(tmem, 96, [&](int kk) { return desc_k(aP, 64, 0, kk); },
                              [&](int hf, int kk) { return desc_mn(aU, 64, 64 * hf, kk); }, false);
    umma_commit(&bars[2]);
  }
  if (ok) {  // O = e^gamma (Q^ S0) + P U
    ok = mbar_wait_warp(&bars[2], 0, a.status, __LINE__);
    if (ok) {
      tc_fence_after();
      const int c0 = acc_col0(64);
      uint32_t rs[32], ru[32];
      tmem_ld32_raw(acc_addr(tmem, 32, 64), rs);
      tmem_ld32_raw(acc_addr(tmem, 96, 64), ru);
      tmem_wait_ld();
      if (r < n) {
        const float er = eg[r];
        bf16* o = a.out + (int64_t)(row0 + r) * g.row_v + (int64_t)h * 128 + c0;
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float v8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v8[e] = er * __uint_as_float(rs[8 * q8 + e]) + __uint_as_float(ru[8 * q8 + e]);
          *reinterpret_cast<uint4*>(o + 8 * q8) = make_uint4(pack_bf16x2(v8[0], v8[1]), pack_bf16x2(v8[2], v8[3]),
                                                             pack_bf16x2(v8[4], v8[5]), pack_bf16x2(v8[6], v8[7]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// gdn_state_tc: the forward state recurrence.  One CTA (four warps) per (sequence, head,
// 64 value columns); the state slice S (128 x 64, fp32) stays in TMEM as the accumulator
// of its own update.  Per chunk: S0 -> bf16 operand tile and the saved states; S <-
// e^{gamma_C} S (tcgen05.ld / st); U = U~ - W S0 (64-row MMA, written back over U~); then
// S += K^T diag(F kinv) U (128-row MMA on the raw keys).  The next chunk's W, K, U~ and
// per-token scalars are loaded (TMA and cp.async on one mbarrier) while this one runs.
struct StateTcSm {
  static constexpr int kW = 0;          // W        2 x (64 x 128)
  static constexpr int kK = 32768;      // raw K    2 x (64 x 128)
  static constexpr int kU = 65536;      // U~ slice 2 x (64 x 64)
  static constexpr int kS0 = 81920;     // S0 (bf16) 128 x 64
  static constexpr int kFU = 98304;     // diag(F kinv) U  64 x 64
  static constexpr int kScal = 106496;  // 2 x {gamma[64], kinv[64]}
  static constexpr int kBars = kScal + 1024;
  static constexpr int kTotal = kBars + 64;
};

struct StateTcArgs {
  gdnk::Geo g;
  const float* gcum;
  const float* kinv;
  bf16* u_io;          // (chunks, heads, 64, 128): U~ in, U out
  const float* init;   // (seqs, heads, 128, 128) or nullptr
  bf16* states;        // (chunks, heads, 128, 128): S at every chunk start
  float* fin;          // (seqs, heads, 128, 128) or nullptr
  int* status;
};

__global__ void __launch_bounds__(128, 2)
gdn_state_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmU, const StateTcArgs a) {
  using S = StateTcSm;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const gdnk::Geo& g = a.g;
  const int part = blockIdx.x & 1;
  const int h = (blockIdx.x >> 1) % g.heads;
  const int seq = g.order[(blockIdx.x >> 1) / g.heads];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int col0 = part * 64;
  int t0, len;
  gdnk::seq_span(g, seq, t0, len);
  const int nch = (len + C - 1) / C;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kBars);  // load[2], U, S
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kBars + 32);
  if (tid == 0) {
    mbar_init(&bars[0], 1 + C);  // TMA arrival + one cp.async arrival per scalar lane
    mbar_init(&bars[1], 1 + C);
    mbar_init(&bars[2], 1);
    mbar_init(&bars[3], 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tU = tmem + 64;
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
  const int64_t sh = (int64_t)seq * g.heads + h;
  {  // initial state slice: row d = tid
    uint32_t v[2][32];
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      const float x = a.init != nullptr ? a.init[(sh * 128 + tid) * 128 + col0 + c] : 0.f;
      v[c >> 5][c & 31] = __float_as_uint(x);
    }
    tmem_st32(tS + lane_base, v[0]);
    tmem_st32(tS + lane_base + 32, v[1]);
  }
  auto prefetch = [&](int ci) {
    const int b = ci & 1;
    const int chunk = g.chunk_off[seq] + ci;
    const int row0 = t0 + ci * C, n = min(C, len - ci * C);
    const int64_t cbase = (int64_t)chunk * g.heads + h;
    float* sc = reinterpret_cast<float*>(sm + S::kScal + b * 512);
    if (tid < C) {
      const int64_t src = (int64_t)h * g.rows + row0 + (tid < n ? tid : 0);
      cp_async_4(smem_u32(sc + tid), a.gcum + src, tid < n);
      cp_async_4(smem_u32(sc + 64 + tid), a.kinv + src, tid < n);
      cp_async_mbar_arrive_noinc(&bars[b]);
    }
    if (tid == 0) {
      mbar_arrive_expect_tx(&bars[b], 2 * 16384 + 8192);
      for (int cb = 0; cb < 2; ++cb) {
        tma_load_3d(sm + S::kW + b * 16384 + cb * 8192, &tmW, &bars[b], cb * 64, (int)(cbase * 64), 0);
        tma_load_3d(sm + S::kK + b * 16384 + cb * 8192, &tmK, &bars[b], h * 128 + cb * 64, row0, 0);
      }
      tma_load_3d(sm + S::kU + b * 8192, &tmU, &bars[b], col0, (int)(cbase * 64), 0);
    }
  };
  const uint32_t sb = smem_u32(sm);
  bool ok = true;
  if (nch > 0) prefetch(0);
  tc_fence_before();
  __syncthreads();
  for (int ci = 0; ci < nch && ok; ++ci) {
    const int b = ci & 1;
    const int chunk = g.chunk_off[seq] + ci;
    const int n = min(C, len - ci * C);
    const int64_t cbase = (int64_t)chunk * g.heads + h;
    if (ci > 0) ok = mbar_wait_warp(&bars[3], (ci - 1) & 1, a.status, __LINE__);  // previous S update done
    ok = __syncthreads_and(ok);
    if (!ok) break;
    if (ci + 1 < nch) prefetch(ci + 1);  // into the buffer the previous chunk released
    ok = mbar_wait_warp(&bars[b], (ci >> 1) & 1, a.status, __LINE__);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    const float* sc = reinterpret_cast<const float*>(sm + S::kScal + b * 512);
    const float gl = sc[n - 1];
    {  // S0 -> operand tile and saved states; S <- e^{gamma_C} S
      uint32_t v[2][32];
      tmem_ld32_raw(tS + lane_base, v[0]);
      tmem_ld32_raw(tS + lane_base + 32, v[1]);
      tmem_wait_ld();
      const int d = tid;
      bf16* dst = a.states + (cbase * 128 + d) * 128 + col0;
      const float eg = __expf(gl);
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[c8 >> 2][(c8 & 3) * 8 + e]);
        st8(sm + S::kS0, 128, d, c8 * 8, f);
        *reinterpret_cast<uint4*>(dst + c8 * 8) = *reinterpret_cast<const uint4*>(sm + S::kS0 + sw_off(128, d, c8 * 8));
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int i = 0; i < 32; ++i) v[hh][i] = __float_as_uint(__uint_as_float(v[hh][i]) * eg);
      tmem_st32(tS + lane_base, v[0]);
      tmem_st32(tS + lane_base + 32, v[1]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // U (accumulator) = W S0
      tc_fence_after();
      constexpr uint32_t idesc = make_idesc_bf16(64, 64, false, true);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16_ss(tU, desc_k(sb + S::kW + b * 16384, 64, 0, kk), desc_mn(sb + S::kS0, 128, 0, kk), idesc,
                     kk > 0 ? 1u : 0u);
      umma_commit(&bars[2]);
    }
    ok = mbar_wait_warp(&bars[2], ci & 1, a.status, __LINE__);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    {  // U = U~ - W S0 (back to global); diag(F kinv) U -> operand tile
      uint32_t v[2][32];
      tmem_ld32_raw(tU + lane_base, v[0]);
      tmem_ld32_raw(tU + lane_base + 32, v[1]);
      tmem_wait_ld();
      if (lane < 16) {
        const int t = 16 * warp + lane;
        const float f = t < n ? __expf(gl - sc[t]) * sc[64 + t] : 0.f;
        bf16* ug = a.u_io + (cbase * C + t) * 128 + col0;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float ut[8], fu[8];
          ld8(sm + S::kU + b * 8192, 64, t, c8 * 8, ut);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            ut[e] -= __uint_as_float(v[c8 >> 2][(c8 & 3) * 8 + e]);
            fu[e] = f * ut[e];
          }
          *reinterpret_cast<uint4*>(ug + c8 * 8) = make_uint4(pack_bf16x2(ut[0], ut[1]), pack_bf16x2(ut[2], ut[3]),
                                                              pack_bf16x2(ut[4], ut[5]), pack_bf16x2(ut[6], ut[7]));
          st8(sm + S::kFU, 64, t, c8 * 8, fu);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // S += K^T (diag(F kinv) U)
      tc_fence_after();
      constexpr uint32_t idesc = make_idesc_bf16(128, 64, true, true);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16_ss(tS, desc_mn(sb + S::kK + b * 16384, 64, 0, kk), desc_mn(sb + S::kFU, 64, 0, kk), idesc, 1u);
      umma_commit(&bars[3]);
    }
  }
  if (ok && nch > 0) ok = mbar_wait_warp(&bars[3], (nch - 1) & 1, a.status, __LINE__);
  ok = __syncthreads_and(ok);
  if (ok && a.fin != nullptr) {
    tc_fence_after();
    uint32_t v[2][32];
    tmem_ld32_raw(tS + lane_base, v[0]);
    tmem_ld32_raw(tS + lane_base + 32, v[1]);
    tmem_wait_ld();
    float* dst = a.fin + (sh * 128 + tid) * 128 + col0;
#pragma unroll
    for (int c4 = 0; c4 < 16; ++c4)
      *reinterpret_cast<float4*>(dst + c4 * 4) =
          make_float4(__uint_as_float(v[c4 >> 3][(c4 & 7) * 4]), __uint_as_float(v[c4 >> 3][(c4 & 7) * 4 + 1]),
                      __uint_as_float(v[c4 >> 3][(c4 & 7) * 4 + 2]), __uint_as_float(v[c4 >> 3][(c4 & 7) * 4 + 3]));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// gdn_dstate_tc: the reverse state-gradient recurrence.  One CTA (four warps) per
// (sequence, head, 64 value columns); dS (128 x 64, fp32) stays in TMEM.  Per chunk, last
// to first: dS_C -> bf16 operand tile and the saved dstates; dS <- e^{gamma_C} dS;
//   dU  = P^T dO + diag(F kinv) (K_raw dS_C)            (two 64-row MMAs)
//   dS += Q_raw^T diag(e^gamma qinv) dO - W^T dU        (two 128-row MMAs)
struct DStateTcSm {
  static constexpr int kQ = 0;          // raw Q     64 x 128
  static constexpr int kW = 16384;      // W         64 x 128
  static constexpr int kK = 32768;      // raw K     64 x 128
  static constexpr int kP = 49152;      // P         64 x 64
  static constexpr int kDO = 57344;     // dO slice  64 x 64, scaled in place to diag(e^gamma qinv) dO
  static constexpr int kDS = 65536;     // dS_C (bf16) 128 x 64
  static constexpr int kDU = 81920;     // -dU       64 x 64
  static constexpr int kScal = 90112;   // gamma, kinv, qinv (64 each)
  static constexpr int kBars = kScal + 768;
  static constexpr int kTotal = kBars + 64;
};

struct DStateTcArgs {
  gdnk::Geo g;
  const float* gcum;
  const float* kinv;
  const float* qinv;
  const float* dfinal;  // (seqs, heads, 128, 128) or nullptr
  bf16* dstates;        // (chunks, heads, 128, 128): dS at every chunk end
  float* dinit;         // (seqs, heads, 128, 128)
  int* status;
};

__global__ void __launch_bounds__(128, 2)
gdn_dstate_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmP,
                     const __grid_constant__ CUtensorMap tmDO, const DStateTcArgs a) {
  using S = DStateTcSm;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const gdnk::Geo& g = a.g;
  const int part = blockIdx.x & 1;
  const int h = (blockIdx.x >> 1) % g.heads;
  const int seq = g.order[(blockIdx.x >> 1) / g.heads];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int col0 = part * 64;
  int t0, len;
  gdnk::seq_span(g, seq, t0, len);
  const int nch = (len + C - 1) / C;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::kBars);  // load, dU products, dS update
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S::kBars + 32);
  float* gam = reinterpret_cast<float*>(sm + S::kScal);
  float* ki = gam + 64;
  float* qi = gam + 128;
  if (tid == 0) {
    mbar_init(&bars[0], 1 + C);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tA = tmem + 64, tB = tmem + 128;  // dS, P^T dO, K_raw dS_C
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
  const int64_t sh = (int64_t)seq * g.heads + h;
  {
    uint32_t v[2][32];
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      const float x = a.dfinal != nullptr ? a.dfinal[(sh * 128 + tid) * 128 + col0 + c] : 0.f;
      v[c >> 5][c & 31] = __float_as_uint(x);
    }
    tmem_st32(tS + lane_base, v[0]);
    tmem_st32(tS + lane_base + 32, v[1]);
  }
  const uint32_t sb = smem_u32(sm);
  bool ok = true;
  tc_fence_before();
  __syncthreads();
  for (int it = 0; it < nch && ok; ++it) {
    const int ci = nch - 1 - it;
    const int chunk = g.chunk_off[seq] + ci;
    const int row0 = t0 + ci * C, n = min(C, len - ci * C);
    const int64_t cbase = (int64_t)chunk * g.heads + h;
    if (it > 0) ok = mbar_wait_warp(&bars[2], (it - 1) & 1, a.status, __LINE__);  // previous dS update done
    ok = __syncthreads_and(ok);
    if (!ok) break;
    if (tid < C) {
      const int64_t src = (int64_t)h * g.rows + row0 + (tid < n ? tid : 0);
      cp_async_4(smem_u32(gam + tid), a.gcum + src, tid < n);
      cp_async_4(smem_u32(ki + tid), a.kinv + src, tid < n);
      cp_async_4(smem_u32(qi + tid), a.qinv + src, tid < n);
      cp_async_mbar_arrive_noinc(&bars[0]);
    }
    if (tid == 0) {
      mbar_arrive_expect_tx(&bars[0], 3 * 16384 + 2 * 8192);
      for (int cb = 0; cb < 2; ++cb) {
        tma_load_3d(sm + S::kQ + cb * 8192, &tmQ, &bars[0], h * 128 + cb * 64, row0, 0);
        tma_load_3d(sm + S::kW + cb * 8192, &tmW, &bars[0], cb * 64, (int)(cbase * 64), 0);
        tma_load_3d(sm + S::kK + cb * 8192, &tmK, &bars[0], h * 128 + cb * 64, row0, 0);
      }
      tma_load_3d(sm + S::kP, &tmP, &bars[0], 0, (int)(cbase * 64), 0);
      tma_load_3d(sm + S::kDO, &tmDO, &bars[0], h * 128 + col0, row0, 0);
    }
    tc_fence_after();
    {  // dS_C -> operand tile and saved dstates; dS <- e^{gamma_C} dS (after the scalars land)
      uint32_t v[2][32];
      tmem_ld32_raw(tS + lane_base, v[0]);
      tmem_ld32_raw(tS + lane_base + 32, v[1]);
      tmem_wait_ld();
      const int d = tid;
      bf16* dst = a.dstates + (cbase * 128 + d) * 128 + col0;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[c8 >> 2][(c8 & 3) * 8 + e]);
        st8(sm + S::kDS, 128, d, c8 * 8, f);
        *reinterpret_cast<uint4*>(dst + c8 * 8) = *reinterpret_cast<const uint4*>(sm + S::kDS + sw_off(128, d, c8 * 8));
      }
      ok = mbar_wait_warp(&bars[0], it & 1, a.status, __LINE__);
      ok = __syncthreads_and(ok);
      if (!ok) break;
      const float eg = __expf(gam[n - 1]);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int i = 0; i < 32; ++i) v[hh][i] = __float_as_uint(__uint_as_float(v[hh][i]) * eg);
      tmem_st32(tS + lane_base, v[0]);
      tmem_st32(tS + lane_base + 32, v[1]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // P^T dO and K_raw dS_C
      tc_fence_after();
      constexpr uint32_t id64 = make_idesc_bf16(64, 64, true, true);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16_ss(tA, desc_mn(sb + S::kP, 64, 0, kk), desc_mn(sb + S::kDO, 64, 0, kk), id64, kk > 0 ? 1u : 0u);
      constexpr uint32_t idk = make_idesc_bf16(64, 64, false, true);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16_ss(tB, desc_k(sb + S::kK, 64, 0, kk), desc_mn(sb + S::kDS, 128, 0, kk), idk, kk > 0 ? 1u : 0u);
      umma_commit(&bars[1]);
    }
    ok = mbar_wait_warp(&bars[1], it & 1, a.status, __LINE__);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc_fence_after();
    {  // -dU -> operand tile; dO rows scaled by e^gamma qinv in place (P^T dO has read them)
      uint32_t va[2][32], vb[2][32];
      tmem_ld32_raw(tA + lane_base, va[0]);
      tmem_ld32_raw(tA + lane_base + 32, va[1]);
      tmem_ld32_raw(tB + lane_base, vb[0]);
      tmem_ld32_raw(tB + lane_base + 32, vb[1]);
      tmem_wait_ld();
      const float gl = gam[n - 1];
      if (lane < 16) {
        const int t = 16 * warp + lane;
        const float f = t < n ? __expf(gl - gam[t]) * ki[t] : 0.f;
        const float sq = t < n ? __expf(gam[t]) * qi[t] : 0.f;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float du[8], dq[8];
          ld8(sm + S::kDO, 64, t, c8 * 8, dq);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = (c8 & 3) * 8 + e;
            du[e] = -(__uint_as_float(va[c8 >> 2][j]) + f * __uint_as_float(vb[c8 >> 2][j]));
            dq[e] *= sq;
          }
          st8(sm + S::kDU, 64, t, c8 * 8, du);
          st8(sm + S::kDO, 64, t, c8 * 8, dq);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {  // dS += Q_raw^T (diag(e^gamma qinv) dO) + W^T (-dU)
      tc_fence_after();
      constexpr uint32_t id128 = make_idesc_bf16(128, 64, true, true);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16_ss(tS, desc_mn(sb + S::kQ, 64, 0, kk), desc_mn(sb + S::kDO, 64, 0, kk), id128, 1u);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16_ss(tS, desc_mn(sb + S::kW, 64, 0, kk), desc_mn(sb + S::kDU, 64, 0, kk), id128, 1u);
      umma_commit(&bars[2]);
    }
  }
  if (ok && nch > 0) ok = mbar_wait_warp(&bars[2], (nch - 1) & 1, a.status, __LINE__);
  ok = __syncthreads_and(ok);
  if (ok) {
    tc_fence_after();
    uint32_t v[2][32];
    tmem_ld32_raw(tS + lane_base, v[0]);
    tmem_ld32_raw(tS + lane_base + 32, v[1]);
    tmem_wait_ld();
    float* dst = a.dinit + (sh * 128 + tid) * 128 + col0;
#pragma unroll
    for (int c4 = 0; c4 < 16; ++c4)
      *reinterpret_cast<float4*>(dst + c4 * 4) =
          make_float4(__uint_as_float(v[c4 >> 3][(c4 & 7) * 4]), __uint_as_float(v[c4 >> 3][(c4 & 7) * 4 + 1]),
                      __uint_as_float(v[c4 >> 3][(c4 & 7) * 4 + 2]), __uint_as_float(v[c4 >> 3][(c4 & 7) * 4 + 3]));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace gtc

// Host launcher, called by gdn_chunk_bwd (gdn.cu) after the dS recurrence: one CTA per
// (chunk, head) over `bound` chunks (CTAs past the real chunk count exit at once).
void gdn_grad_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& q, const torch::Tensor& k,
                        const torch::Tensor& v, const torch::Tensor& beta_f, const torch::Tensor& gcum,
                        const torch::Tensor& kinv, const torch::Tensor& qinv, const torch::Tensor& u,
                        const torch::Tensor& states, const torch::Tensor& dstates, const torch::Tensor& tmat,
                        const torch::Tensor& dout, torch::Tensor& dq, torch::Tensor& dk, torch::Tensor& dv,
                        torch::Tensor& dg, torch::Tensor& db, float qscale, int* status, cudaStream_t stream) {
  using S = gtc::GradTcSm;
  const int H = g.heads;
  const int64_t rows = g.rows;
  const int64_t nbh = (int64_t)std::max(bound, 1) * H;
  TORCH_CHECK(nbh * 128 < (int64_t)INT32_MAX, "gdn_grad_tc: too many chunks for 32-bit TMA coordinates");
  auto bfmap = [&](const torch::Tensor& t, int64_t dim0, int64_t dim1, int64_t stride1, int box1) {
    return make_tmap_3d(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dim0, dim1, 1, stride1, 0, 64, box1);
  };
  const CUtensorMap tmK = bfmap(k, g.row_q, rows, g.row_q, 64);
  const CUtensorMap tmQ = bfmap(q, g.row_q, rows, g.row_q, 64);
  const CUtensorMap tmDO = bfmap(dout, g.row_v, rows, g.row_v, 64);
  const CUtensorMap tmU = bfmap(u, 128, nbh * 64, 128, 64);
  const CUtensorMap tmS = bfmap(states, 128, nbh * 128, 128, 128);
  const CUtensorMap tmDS = bfmap(dstates, 128, nbh * 128, 128, 128);
  const CUtensorMap tmT = bfmap(tmat, 64, nbh * 64, 64, 64);
  gtc::GradTcArgs a;
  a.g = g;
  a.q = (const gtc::bf16*)q.data_ptr();
  a.k = (const gtc::bf16*)k.data_ptr();
  a.v = (const gtc::bf16*)v.data_ptr();
  a.beta = beta_f.data_ptr<float>();
  a.gcum = gcum.data_ptr<float>();
  a.kinv = kinv.data_ptr<float>();
  a.qinv = qinv.data_ptr<float>();
  a.dq = (gtc::bf16*)dq.data_ptr();
  a.dk = (gtc::bf16*)dk.data_ptr();
  a.dv = (gtc::bf16*)dv.data_ptr();
  a.dg = dg.data_ptr<float>();
  a.db = db.data_ptr<float>();
  a.qscale = qscale;
  a.status = status;
  static SmemOptIn opt;
  const int smem = S::kTotal + 1024;
  C10_CUDA_CHECK(opt.ensure(gtc::gdn_grad_tc_kernel, smem));
  gtc::gdn_grad_tc_kernel<<<(unsigned)(bound * H), gtc::NT, smem, stream>>>(tmK, tmQ, tmDO, tmU, tmS, tmDS, tmT, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb

namespace mykb {

void gdn_prep_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& q, const torch::Tensor& k,
                        const torch::Tensor& v, const torch::Tensor& gg_f, const torch::Tensor& beta_f,
                        torch::Tensor& gcum, torch::Tensor& kinv, torch::Tensor& qinv, torch::Tensor& w,
                        torch::Tensor& u, torch::Tensor& tmat, float qscale, int* status, cudaStream_t stream) {
  const int64_t rows = g.rows;
  const CUtensorMap tmK = make_tmap_3d(k.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.row_q, rows, 1, g.row_q, 0, 64, 64);
  const CUtensorMap tmV = make_tmap_3d(v.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.row_v, rows, 1, g.row_v, 0, 64, 64);
  gtc::PrepTcArgs a;
  a.g = g;
  a.q = (const gtc::bf16*)q.data_ptr();
  a.gg = gg_f.data_ptr<float>();
  a.bb = beta_f.data_ptr<float>();
  a.gcum = gcum.data_ptr<float>();
  a.kinv = kinv.data_ptr<float>();
  a.qinv = qinv.data_ptr<float>();
  a.w_out = (gtc::bf16*)w.data_ptr();
  a.u_out = (gtc::bf16*)u.data_ptr();
  a.t_out = (gtc::bf16*)tmat.data_ptr();
  a.qscale = qscale;
  a.status = status;
  static SmemOptIn opt;
  const int smem = gtc::PrepTcSm::kTotal + 1024;
  C10_CUDA_CHECK(opt.ensure(gtc::gdn_prep_tc_kernel, smem));
  gtc::gdn_prep_tc_kernel<<<(unsigned)(bound * g.heads), gtc::NT, smem, stream>>>(tmK, tmV, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gdn_out_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& q, const torch::Tensor& k,
                       const torch::Tensor& gcum, const torch::Tensor& kinv, const torch::Tensor& qinv,
                       const torch::Tensor& u, const torch::Tensor& states, torch::Tensor& p, torch::Tensor& out,
                       int* status, cudaStream_t stream) {
  const int64_t rows = g.rows;
  const int64_t nbh = (int64_t)std::max(bound, 1) * g.heads;
  TORCH_CHECK(nbh * 128 < (int64_t)INT32_MAX, "gdn_out_tc: too many chunks for 32-bit TMA coordinates");
  const CUtensorMap tmQ = make_tmap_3d(q.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.row_q, rows, 1, g.row_q, 0, 64, 64);
  const CUtensorMap tmK = make_tmap_3d(k.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.row_q, rows, 1, g.row_q, 0, 64, 64);
  const CUtensorMap tmU = make_tmap_3d(u.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, nbh * 64, 1, 128, 0, 64, 64);
  const CUtensorMap tmS = make_tmap_3d(states.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, nbh * 128, 1, 128, 0, 64, 128);
  gtc::OutTcArgs a;
  a.g = g;
  a.gcum = gcum.data_ptr<float>();
  a.kinv = kinv.data_ptr<float>();
  a.qinv = qinv.data_ptr<float>();
  a.p_out = (gtc::bf16*)p.data_ptr();
  a.out = (gtc::bf16*)out.data_ptr();
  a.status = status;
  static SmemOptIn opt;
  const int smem = gtc::OutTcSm::kTotal + 1024;
  C10_CUDA_CHECK(opt.ensure(gtc::gdn_out_tc_kernel, smem));
  gtc::gdn_out_tc_kernel<<<(unsigned)(bound * g.heads), gtc::NT, smem, stream>>>(tmQ, tmK, tmU, tmS, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb

namespace mykb {

void gdn_state_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& k, const torch::Tensor& gcum,
                         const torch::Tensor& kinv, const torch::Tensor& w, torch::Tensor& u, const float* init,
                         torch::Tensor& states, torch::Tensor& fin, int* status, cudaStream_t stream) {
  const int64_t nbh = (int64_t)std::max(bound, 1) * g.heads;
  TORCH_CHECK(nbh * 128 < (int64_t)INT32_MAX, "gdn_state_tc: too many chunks for 32-bit TMA coordinates");
  const CUtensorMap tmW = make_tmap_3d(w.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, nbh * 64, 1, 128, 0, 64, 64);
  const CUtensorMap tmK = make_tmap_3d(k.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.row_q, g.rows, 1, g.row_q, 0, 64, 64);
  const CUtensorMap tmU = make_tmap_3d(u.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 128, nbh * 64, 1, 128, 0, 64, 64);
  gtc::StateTcArgs a;
  a.g = g;
  a.gcum = gcum.data_ptr<float>();
  a.kinv = kinv.data_ptr<float>();
  a.u_io = (gtc::bf16*)u.data_ptr();
  a.init = init;
  a.states = (gtc::bf16*)states.data_ptr();
  a.fin = fin.data_ptr<float>();
  a.status = status;
  static SmemOptIn opt;
  const int smem = gtc::StateTcSm::kTotal + 1024;
  C10_CUDA_CHECK(opt.ensure(gtc::gdn_state_tc_kernel, smem));
  gtc::gdn_state_tc_kernel<<<(unsigned)(g.num_seqs * g.heads * 2), 128, smem, stream>>>(tmW, tmK, tmU, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb

namespace mykb {

void gdn_dstate_tc_launch(const gdnk::Geo& g, int bound, const torch::Tensor& q, const torch::Tensor& k,
                          const torch::Tensor& gcum, const torch::Tensor& kinv, const torch::Tensor& qinv,
                          const torch::Tensor& w, const torch::Tensor& p, const torch::Tensor& dout,
                          const float* dfinal, torch::Tensor& dstates, torch::Tensor& dinit, int* status,
                          cudaStream_t stream) {
  const int64_t nbh = (int64_t)std::max(bound, 1) * g.heads;
  TORCH_CHECK(nbh * 128 < (int64_t)INT32_MAX, "gdn_dstate_tc: too many chunks for 32-bit TMA coordinates");
  auto bfmap = [&](const torch::Tensor& t, int64_t dim0, int64_t dim1) {
    return make_tmap_3d(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dim0, dim1, 1, dim0, 0, 64, 64);
  };
  const CUtensorMap tmQ = bfmap(q, g.row_q, g.rows);
  const CUtensorMap tmW = bfmap(w, 128, nbh * 64);
  const CUtensorMap tmK = bfmap(k, g.row_q, g.rows);
  const CUtensorMap tmP = bfmap(p, 64, nbh * 64);
  const CUtensorMap tmDO = bfmap(dout, g.row_v, g.rows);
  gtc::DStateTcArgs a;
  a.g = g;
  a.gcum = gcum.data_ptr<float>();
  a.kinv = kinv.data_ptr<float>();
  a.qinv = qinv.data_ptr<float>();
  a.dfinal = dfinal;
  a.dstates = (gtc::bf16*)dstates.data_ptr();
  a.dinit = dinit.data_ptr<float>();
  a.status = status;
  static SmemOptIn opt;
  const int smem = gtc::DStateTcSm::kTotal + 1024;
  C10_CUDA_CHECK(opt.ensure(gtc::gdn_dstate_tc_kernel, smem));
  gtc::gdn_dstate_tc_kernel<<<(unsigned)(g.num_seqs * g.heads * 2), 128, smem, stream>>>(tmQ, tmW, tmK, tmP, tmDO, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
