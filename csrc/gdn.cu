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
// Everything except the S0 -> S1 recurrence is independent per chunk, so the work is
// split into chunk-parallel kernels (one CTA per (chunk, head), on the tcgen05 tensor
// cores, in gdn_tc.cu) around a thin sequential kernel (one CTA per (sequence, head, 32
// value columns), here) that carries the state:
//
//   forward:  gdn_prep_tc (K^K^T, blocked triangular inverse, W, U~, T)
//             gdn_state   (U = U~ - W S0, S1 = ...; saves S0 per chunk, U)
//             gdn_out_tc  (P = lower(E * Q^K^T), O)
//   backward: gdn_dstate  (dS at every chunk end, reverse recurrence)
//             gdn_grad_tc (dq, dk, dv, dg, dbeta of every chunk, l2-norm backward)
//
// The sequential kernels keep their 128 x 32 state slice in the fragments of warp-level
// bf16 MMAs (fp32 accumulate) between chunks, fed by ldmatrix from padded shared-memory
// tiles, with the next chunk's operands streaming in by cp.async; the state and every
// reduction stay in fp32.
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
constexpr int LD = 136;    // padded row stride (elements) of 128-wide bf16 tiles
constexpr int LDS = 72;    // padded row stride of 64-wide bf16 tiles
constexpr int LDP = 40;    // padded row stride of 32-wide bf16 tiles
constexpr int PARTS = 4;   // value-column slices of the sequential kernels
constexpr int PW = DV / PARTS;  // 32 columns per slice
constexpr int NT = 256;    // threads of every chunk kernel (8 warps)

// ---------------------------------------------------------------- warp MMA helpers
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const bf16* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], const bf16* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// acc[j] (16 x 8 tile j) += A(m0.., 0..K) * B(0..K, n0 + 8j ..)
//   A_T == false: A(m, k) at A[m * lda + k];  true: at A[k * lda + m]
//   B_T == false: B(k, n) at B[n * ldb + k];  true: at B[k * ldb + n]
// Fragment element e of acc[j] sits at row m0 + lane/4 + 8 (e >= 2), column
// n0 + 8j + 2 (lane % 4) + (e & 1).
template <int NT8, bool A_T, bool B_T>
__device__ __forceinline__ void warp_mma(float (&acc)[NT8][4], const bf16* A, int lda, int m0, const bf16* B, int ldb,
                                         int n0, int K) {
  static_assert(NT8 % 2 == 0, "pairs of n8 tiles");
  const int lane = threadIdx.x & 31;
  const int r = lane & 7, mat = lane >> 3;
#pragma unroll 2
  for (int k0 = 0; k0 < K; k0 += 16) {
    uint32_t a[4];
    if (!A_T) ldsm4(a, A + (m0 + (lane & 15)) * lda + k0 + (lane >> 4) * 8);
    else ldsm4t(a, A + (k0 + r + (mat >> 1) * 8) * lda + m0 + (mat & 1) * 8);
#pragma unroll
    for (int j = 0; j < NT8; j += 2) {
      uint32_t b[4];
      if (!B_T) ldsm4(b, B + (n0 + j * 8 + r + (mat >> 1) * 8) * ldb + k0 + (mat & 1) * 8);
      else ldsm4t(b, B + (k0 + (mat & 1) * 8 + r) * ldb + n0 + j * 8 + (mat >> 1) * 8);
      mma(acc[j], a, b[0], b[1]);
      mma(acc[j + 1], a, b[2], b[3]);
    }
  }
}

template <int NT8>
__device__ __forceinline__ void zero(float (&acc)[NT8][4]) {
#pragma unroll
  for (int j = 0; j < NT8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void st2(bf16* p, float a, float b) { *reinterpret_cast<uint32_t*>(p) = pack2(a, b); }
__device__ __forceinline__ float2 ld2(const bf16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

// ---------------------------------------------------------------- async copies
__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
  // zero-fills the 16 bytes when !valid (no bytes are read)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 64 token rows (stride `stride` elements) x 128 columns -> padded tile; rows >= n zero.
__device__ __forceinline__ void rows128_async(bf16* dst, const bf16* src, int64_t stride, int n) {
  for (int i = threadIdx.x; i < C * 16; i += NT) {
    const int r = i >> 4, c = (i & 15) * 8;
    cp16(dst + r * LD + c, src + (r < n ? r : 0) * stride + c, r < n);
  }
}
// 64 token rows x 32 columns (a value slice) -> padded tile; rows >= n zero.
__device__ __forceinline__ void rows32_async(bf16* dst, const bf16* src, int64_t stride, int n) {
  if (threadIdx.x < C * 4) {
    const int r = threadIdx.x >> 2, c = (threadIdx.x & 3) * 8;
    cp16(dst + r * LDP + c, src + (r < n ? r : 0) * stride + c, r < n);
  }
}
// contiguous (rows x 128) bf16 block -> padded tile
__device__ __forceinline__ void tile128_async(bf16* dst, const bf16* src, int rows) {
  for (int i = threadIdx.x; i < rows * 16; i += NT) {
    const int r = i >> 4, c = (i & 15) * 8;
    cp16(dst + r * LD + c, src + r * 128 + c, true);
  }
}
// contiguous (64 x 64) bf16 block -> padded tile
__device__ __forceinline__ void tile64_async(bf16* dst, const bf16* src) {
  for (int i = threadIdx.x; i < C * 8; i += NT) {
    const int r = i >> 3, c = (i & 7) * 8;
    cp16(dst + r * LDS + c, src + r * C + c, true);
  }
}
// 64 per-token floats of head-major scalars (rows >= n zero) -> shared
__device__ __forceinline__ void scal_async(float* dst, const float* src, int n) {
  if (threadIdx.x < C) cp4(dst + threadIdx.x, src + (threadIdx.x < n ? threadIdx.x : 0), threadIdx.x < n);
}
// gdn_state: one CTA per (sequence, head, 32 value columns); the state slice (128 x 32,
// fp32) lives in the MMA accumulators of the 8 warps (warp w: key rows 16w..16w+15).
// The next chunk's operands stream in (cp.async, double buffered) while this one runs;
// S += K^T diag(F kinv) U uses the raw keys with the scaling folded into U's rows.
struct StateBuf {
  bf16 w[C * LD];   // W
  bf16 k[C * LD];   // raw keys
  bf16 u[C * LDP];  // U~ slice
  float gam[C], ki[C];
};
struct StateSm {
  StateBuf buf[2];
  bf16 uf[C * LDP];   // diag(F kinv) U (operand)
  bf16 sb[DK * LDP];  // S0 slice (operand)
};

__global__ void __launch_bounds__(NT) gdn_state_kernel(Geo g, const bf16* __restrict__ k, const float* __restrict__ gcum,
                                                       const float* __restrict__ kinv, const bf16* __restrict__ w_in,
                                                       bf16* __restrict__ u_io, const float* __restrict__ init,
                                                       bf16* __restrict__ states, float* __restrict__ fin) {
  extern __shared__ __align__(16) unsigned char smraw[];
  StateSm& s = *reinterpret_cast<StateSm*>(smraw);
  const int part = blockIdx.x % PARTS;
  const int h = (blockIdx.x / PARTS) % g.heads;
  const int seq = g.order[blockIdx.x / (PARTS * g.heads)];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = (lane & 3) * 2;
  const int col0 = part * PW;
  int t0, len;
  seq_span(g, seq, t0, len);
  float S[4][4];
  {
    const float* src = init != nullptr ? init + ((int64_t)seq * g.heads + h) * DK * DV : nullptr;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = warp * 16 + gq, c = col0 + j * 8 + cq;
      S[j][0] = src ? src[r * DV + c] : 0.f;
      S[j][1] = src ? src[r * DV + c + 1] : 0.f;
      S[j][2] = src ? src[(r + 8) * DV + c] : 0.f;
      S[j][3] = src ? src[(r + 8) * DV + c + 1] : 0.f;
    }
  }
  const int nch = (len + C - 1) / C;
  auto prefetch = [&](int ci) {
    StateBuf& b = s.buf[ci & 1];
    const int chunk = g.chunk_off[seq] + ci;
    const int row0 = t0 + ci * C, n = min(C, len - ci * C);
    const int64_t cbase = (int64_t)chunk * g.heads + h;
    tile128_async(b.w, w_in + cbase * C * DK, C);
    rows128_async(b.k, k + (int64_t)row0 * g.row_q + (int64_t)h * DK, g.row_q, n);
    rows32_async(b.u, u_io + cbase * C * DV + col0, DV, C);
    scal_async(b.gam, gcum + (int64_t)h * g.rows + row0, n);
    scal_async(b.ki, kinv + (int64_t)h * g.rows + row0, n);
    cp_commit();
  };
  if (nch > 0) prefetch(0);
  for (int ci = 0; ci < nch; ++ci) {
    if (ci + 1 < nch) {
      prefetch(ci + 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    StateBuf& b = s.buf[ci & 1];
    const int chunk = g.chunk_off[seq] + ci;
    const int n = min(C, len - ci * C);
    const int64_t cbase = (int64_t)chunk * g.heads + h;
    bf16* st = states + cbase * DK * DV + col0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // S0 of this chunk: to global and to the operand tile
      const int r = warp * 16 + gq, c = j * 8 + cq;
      st2(st + r * DV + c, S[j][0], S[j][1]);
      st2(st + (r + 8) * DV + c, S[j][2], S[j][3]);
      st2(s.sb + r * LDP + c, S[j][0], S[j][1]);
      st2(s.sb + (r + 8) * LDP + c, S[j][2], S[j][3]);
    }
    __syncthreads();
    const float gl = b.gam[n - 1];
    {  // U = U~ - W S0  (64 x 32): warp -> rows 16 (w % 4), columns 16 (w / 4)
      float acc[2][4];
      zero(acc);
      const int mt = warp & 3, nb = (warp >> 2) * 16;
      warp_mma<2, false, true>(acc, b.w, LD, mt * 16, s.sb, LDP, nb, DK);
      bf16* ug = u_io + cbase * C * DV + col0;
      const int r = mt * 16 + gq;
      const float f0 = r < n ? __expf(gl - b.gam[r]) * b.ki[r] : 0.f;
      const float f1 = r + 8 < n ? __expf(gl - b.gam[r + 8]) * b.ki[r + 8] : 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int c = nb + j * 8 + cq;
        const float2 u0 = ld2(b.u + r * LDP + c), u1 = ld2(b.u + (r + 8) * LDP + c);
        const float a0 = u0.x - acc[j][0], a1 = u0.y - acc[j][1], a2 = u1.x - acc[j][2], a3 = u1.y - acc[j][3];
        st2(ug + r * DV + c, a0, a1);
        st2(ug + (r + 8) * DV + c, a2, a3);
        st2(s.uf + r * LDP + c, f0 * a0, f0 * a1);
        st2(s.uf + (r + 8) * LDP + c, f1 * a2, f1 * a3);
      }
    }
    __syncthreads();
    {  // S <- e^{gamma_C} S + K_raw^T (diag(F kinv) U)
      const float egl = __expf(gl);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[j][e] *= egl;
      warp_mma<4, true, true>(S, b.k, LD, warp * 16, s.uf, LDP, 0, C);
    }
    __syncthreads();
  }
  if (fin != nullptr) {
    float* dst = fin + ((int64_t)seq * g.heads + h) * DK * DV;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = warp * 16 + gq, c = col0 + j * 8 + cq;
      *reinterpret_cast<float2*>(dst + r * DV + c) = make_float2(S[j][0], S[j][1]);
      *reinterpret_cast<float2*>(dst + (r + 8) * DV + c) = make_float2(S[j][2], S[j][3]);
    }
  }
}

// ----------------------------------------------------------------------- backward
// gdn_dstate: dS at every chunk end (dS_C), in reverse:
//   dU  = P^T dO + diag(F kinv) (K_raw dS_C)
//   dS0 = e^{gamma_C} dS_C + Q_raw^T diag(e^gamma qinv) dO - W^T dU
// with the next (earlier) chunk's operands streaming in while this one runs.
struct DStateBuf {
  bf16 q[C * LD];     // raw queries
  bf16 w[C * LD];
  bf16 k[C * LD];     // raw keys
  bf16 p[C * LDS];
  bf16 dob[C * LDP];  // dO slice
  float gam[C], ki[C], qi[C];
};
struct DStateSm {
  DStateBuf buf[2];
  bf16 doq[C * LDP];  // diag(e^gamma qinv) dO slice
  bf16 du[C * LDP];   // -dU slice
  bf16 dsb[DK * LDP];
};

__global__ void __launch_bounds__(NT) gdn_dstate_kernel(Geo g, const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                        const float* __restrict__ gcum, const float* __restrict__ kinv,
                                                        const float* __restrict__ qinv, const bf16* __restrict__ w_in,
                                                        const bf16* __restrict__ p_in, const bf16* __restrict__ dout,
                                                        const float* __restrict__ dfinal, bf16* __restrict__ dstates,
                                                        float* __restrict__ dinit) {
  extern __shared__ __align__(16) unsigned char smraw[];
  DStateSm& s = *reinterpret_cast<DStateSm*>(smraw);
  const int part = blockIdx.x % PARTS;
  const int h = (blockIdx.x / PARTS) % g.heads;
  const int seq = g.order[blockIdx.x / (PARTS * g.heads)];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = (lane & 3) * 2;
  const int col0 = part * PW;
  int t0, len;
  seq_span(g, seq, t0, len);
  float dS[4][4];
  {
    const float* src = dfinal != nullptr ? dfinal + ((int64_t)seq * g.heads + h) * DK * DV : nullptr;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = warp * 16 + gq, c = col0 + j * 8 + cq;
      dS[j][0] = src ? src[r * DV + c] : 0.f;
      dS[j][1] = src ? src[r * DV + c + 1] : 0.f;
      dS[j][2] = src ? src[(r + 8) * DV + c] : 0.f;
      dS[j][3] = src ? src[(r + 8) * DV + c + 1] : 0.f;
    }
  }
  const int nch = (len + C - 1) / C;
  auto prefetch = [&](int ci) {
    DStateBuf& b = s.buf[ci & 1];
    const int chunk = g.chunk_off[seq] + ci;
    const int row0 = t0 + ci * C, n = min(C, len - ci * C);
    const int64_t cbase = (int64_t)chunk * g.heads + h;
    const int64_t hb = (int64_t)h * g.rows + row0;
    rows128_async(b.q, q + (int64_t)row0 * g.row_q + (int64_t)h * DK, g.row_q, n);
    tile128_async(b.w, w_in + cbase * C * DK, C);
    rows128_async(b.k, k + (int64_t)row0 * g.row_q + (int64_t)h * DK, g.row_q, n);
    tile64_async(b.p, p_in + cbase * C * C);
    rows32_async(b.dob, dout + (int64_t)row0 * g.row_v + (int64_t)h * DV + col0, g.row_v, n);
    scal_async(b.gam, gcum + hb, n);
    scal_async(b.ki, kinv + hb, n);
    scal_async(b.qi, qinv + hb, n);
    cp_commit();
  };
  if (nch > 0) prefetch(nch - 1);
  for (int ci = nch - 1; ci >= 0; --ci) {
    if (ci > 0) {
      prefetch(ci - 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    DStateBuf& b = s.buf[ci & 1];
    const int chunk = g.chunk_off[seq] + ci;
    const int n = min(C, len - ci * C);
    const int64_t cbase = (int64_t)chunk * g.heads + h;
    bf16* dst = dstates + cbase * DK * DV + col0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = warp * 16 + gq, c = j * 8 + cq;
      st2(dst + r * DV + c, dS[j][0], dS[j][1]);
      st2(dst + (r + 8) * DV + c, dS[j][2], dS[j][3]);
      st2(s.dsb + r * LDP + c, dS[j][0], dS[j][1]);
      st2(s.dsb + (r + 8) * LDP + c, dS[j][2], dS[j][3]);
    }
    __syncthreads();  // this chunk's buffer and dsb are visible
    const float gl = b.gam[n - 1];
    if (tid < C * 4) {  // diag(e^gamma qinv) dO
      const int r = tid >> 2, c = (tid & 3) * 8;
      const float sc = r < n ? __expf(b.gam[r]) * b.qi[r] : 0.f;
      uint4 v = *reinterpret_cast<const uint4*>(b.dob + r * LDP + c);
      uint32_t* wv = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&wv[e]));
        wv[e] = pack2(f.x * sc, f.y * sc);
      }
      *reinterpret_cast<uint4*>(s.doq + r * LDP + c) = v;
    }
    {  // -dU = -(P^T dO + diag(F kinv) (K_raw dS_C))
      float acc[2][4], kd[2][4];
      zero(acc);
      zero(kd);
      const int mt = warp & 3, nb = (warp >> 2) * 16;
      warp_mma<2, true, true>(acc, b.p, LDS, mt * 16, b.dob, LDP, nb, C);
      warp_mma<2, false, true>(kd, b.k, LD, mt * 16, s.dsb, LDP, nb, DK);
      const int r = mt * 16 + gq;
      const float f0 = r < n ? __expf(gl - b.gam[r]) * b.ki[r] : 0.f;
      const float f1 = r + 8 < n ? __expf(gl - b.gam[r + 8]) * b.ki[r + 8] : 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int c = nb + j * 8 + cq;
        st2(s.du + r * LDP + c, -(acc[j][0] + f0 * kd[j][0]), -(acc[j][1] + f0 * kd[j][1]));
        st2(s.du + (r + 8) * LDP + c, -(acc[j][2] + f1 * kd[j][2]), -(acc[j][3] + f1 * kd[j][3]));
      }
    }
    __syncthreads();
    {
      const float egl = __expf(gl);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) dS[j][e] *= egl;
      warp_mma<4, true, true>(dS, b.q, LD, warp * 16, s.doq, LDP, 0, C);
      warp_mma<4, true, true>(dS, b.w, LD, warp * 16, s.du, LDP, 0, C);
    }
    __syncthreads();
  }
  if (dinit != nullptr) {
    float* dst = dinit + ((int64_t)seq * g.heads + h) * DK * DV;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = warp * 16 + gq, c = col0 + j * 8 + cq;
      *reinterpret_cast<float2*>(dst + r * DV + c) = make_float2(dS[j][0], dS[j][1]);
      *reinterpret_cast<float2*>(dst + (r + 8) * DV + c) = make_float2(dS[j][2], dS[j][3]);
    }
  }
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
  static SmemOptIn a_state;
  C10_CUDA_CHECK(a_state.ensure(gdnk::gdn_state_kernel, (int)sizeof(gdnk::StateSm)));
  const float qscale = 1.f / std::sqrt((float)gdnk::DK);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (rows > 0 && g.num_seqs > 0) {
    gdn_prep_tc_launch(g, bound, q, k, v, gf, bf, gcum, kinv, qinv, w, u, tmat, qscale, device_status(), st);
    gdnk::gdn_state_kernel<<<g.num_seqs * H * gdnk::PARTS, gdnk::NT, sizeof(gdnk::StateSm), st>>>(
        g, (const bf16*)k.data_ptr(), gcum.data_ptr<float>(), kinv.data_ptr<float>(), (const bf16*)w.data_ptr(),
        (bf16*)u.data_ptr(), init.has_value() ? init_f.data_ptr<float>() : nullptr, (bf16*)states.data_ptr(),
        fin.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
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
  static SmemOptIn a_dstate;
  C10_CUDA_CHECK(a_dstate.ensure(gdnk::gdn_dstate_kernel, (int)sizeof(gdnk::DStateSm)));
  const float qscale = 1.f / std::sqrt((float)gdnk::DK);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t rows = (int64_t)q.size(0) * q.size(1);
  if (rows > 0 && g.num_seqs > 0) {
    gdnk::gdn_dstate_kernel<<<g.num_seqs * H * gdnk::PARTS, gdnk::NT, sizeof(gdnk::DStateSm), st>>>(
        g, (const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), gcum.data_ptr<float>(), kinv.data_ptr<float>(),
        qinv.data_ptr<float>(), (const bf16*)w.data_ptr(), (const bf16*)p.data_ptr(), (const bf16*)doc.data_ptr(),
        dfinal.has_value() ? dfin_f.data_ptr<float>() : nullptr, (bf16*)dstates.data_ptr(), dinit.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
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
