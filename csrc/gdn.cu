// Gated DeltaNet kernels (sm_100a): short causal convolution + SiLU, the chunked gated
// delta rule forward / backward (chunk 64), the token recurrence for decoding, and the
// q/k L2-norm backward.
//
// The chunk algorithm is the one stated in myk_llm_b200/ops/gdn_chunk.py:
//   E_ts = exp(gamma_t - gamma_s), A = strictly_lower(diag(beta) (E * K K^T)),
//   U = (I + A)^{-1} diag(beta) (V - Gamma K S0)   (forward substitution),
//   O = Gamma Q S0 + lower_incl(E * Q K^T) U,
//   S_C = exp(gamma_C) S0 + K^T diag(exp(gamma_C - gamma)) U,
// and its hand-derived reverse (backward substitution for dY = (I + A)^{-T} dU).
//
// One CTA owns one (sequence, head, half of the value dimension) and walks the sequence's
// chunks in order (forward) or in reverse (backward), keeping its half of the state in
// shared memory.  Splitting the value dimension in halves is exact: U, O, S, dV and dS
// are column-separable, and every quantity that mixes value columns (dq, dk, dbeta,
// dgamma, dA, dP) is a sum of per-half parts, accumulated with fp32 atomics.  The chunk
// products run on fp32 CUDA cores with 4x4 / 8x4 register tiles from shared memory.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace mykb {

constexpr int kC = 64;        // chunk length
constexpr int kDK = 128;      // head_k_dim supported by the chunk kernels
constexpr int kDVH = 64;      // value columns per CTA (half of head_v_dim 128)
constexpr int kGdnThreads = 256;

struct GdnGeom {
  const int* cu;          // packed document offsets or nullptr (batch layout)
  const int* chunk_off;   // first global chunk index of every sequence
  int num_seqs, heads, seq_len;  // seq_len: batch layout length
  int64_t row_q;          // elements between token rows of q/k (heads * dk)
  int64_t row_v;          // heads * dv
  int dv;                 // full head_v_dim
};

__device__ __forceinline__ void seq_span(const GdnGeom& g, int s, int& t0, int& len) {
  if (g.cu != nullptr) {
    t0 = g.cu[s];
    len = g.cu[s + 1] - t0;
  } else {
    t0 = s * g.seq_len;
    len = g.seq_len;
  }
}

// out[4][4] += A(rows r0..r0+3, k) * B(k, cols c0..c0+3) over k in [0, K)
// A element (r, k) at A[r * sar + k * sak]; B element (k, c) at B[k * sbk + c * sbc].
template <int R, int CC>
__device__ __forceinline__ void mm_acc(float (&out)[R][CC], const float* A, int sar, int sak, const float* B, int sbk,
                                       int sbc, int r0, int c0, int K) {
#pragma unroll 4
  for (int k = 0; k < K; ++k) {
    float a[R], b[CC];
#pragma unroll
    for (int i = 0; i < R; ++i) a[i] = A[(r0 + i) * sar + k * sak];
#pragma unroll
    for (int j = 0; j < CC; ++j) b[j] = B[k * sbk + (c0 + j) * sbc];
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int j = 0; j < CC; ++j) out[i][j] = fmaf(a[i], b[j], out[i][j]);
  }
}

template <int R, int CC>
__device__ __forceinline__ void zero(float (&o)[R][CC]) {
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int j = 0; j < CC; ++j) o[i][j] = 0.f;
}

// Shared-memory plan of the forward (floats)
struct FwdSm {
  static constexpr int S = 0;                        // [dk][64]
  static constexpr int K = S + kDK * kDVH;           // [C][dk]
  static constexpr int Q = K + kC * kDK;             // [C][dk]
  static constexpr int V = Q + kC * kDK;             // [C][64]  V -> W -> U
  static constexpr int A = V + kC * kDVH;            // [C][C]   A, then P
  static constexpr int KS = A + kC * kC;             // [C][64]  K S0, then Q S0
  static constexpr int GAM = KS + kC * kDVH;         // [C] gamma, [C] beta, [C] exp(gamma)
  static constexpr int TOTAL = GAM + 3 * kC;
};

// Loads a chunk: L2-normalised k and q (q also scaled), this half of v, gamma (cumulative
// log decay), beta.  One warp normalises 8 rows.
__device__ __forceinline__ void load_chunk(const GdnGeom& g, float* sm_k, float* sm_q, float* sm_v, float* gam,
                                           float* bet, float* eg, const __nv_bfloat16* q, const __nv_bfloat16* k,
                                           const __nv_bfloat16* v, const float* gg, const float* bb, int t0, int a,
                                           int n, int h, int half, float qscale) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int r = warp; r < kC; r += kGdnThreads / 32) {
    float kv[4], qv[4];
    if (r < n) {
      const int64_t row = (int64_t)(t0 + a + r);
      const __nv_bfloat16* kp = k + row * g.row_q + (int64_t)h * kDK + lane * 4;
      const __nv_bfloat16* qp = q + row * g.row_q + (int64_t)h * kDK + lane * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kv[i] = __bfloat162float(kp[i]);
        qv[i] = __bfloat162float(qp[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) kv[i] = qv[i] = 0.f;
    }
    float sk = kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3];
    float sq = qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sk += __shfl_xor_sync(0xffffffff, sk, o);
      sq += __shfl_xor_sync(0xffffffff, sq, o);
    }
    const float ik = 1.f / fmaxf(sqrtf(sk), 1e-6f), iq = qscale / fmaxf(sqrtf(sq), 1e-6f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sm_k[r * kDK + lane * 4 + i] = kv[i] * ik;
      sm_q[r * kDK + lane * 4 + i] = qv[i] * iq;
    }
    // v half: 64 columns, 2 per lane
    for (int c = lane; c < kDVH; c += 32) {
      float val = 0.f;
      if (r < n) val = __bfloat162float(v[(int64_t)(t0 + a + r) * g.row_v + (int64_t)h * g.dv + half * kDVH + c]);
      sm_v[r * kDVH + c] = val;
    }
  }
  if (warp == 0) {
    // gamma = inclusive cumsum of g over the chunk (2 elements per lane), padded with 0
    float x0 = (2 * lane < n) ? gg[(int64_t)(t0 + a + 2 * lane) * g.heads + h] : 0.f;
    float x1 = (2 * lane + 1 < n) ? gg[(int64_t)(t0 + a + 2 * lane + 1) * g.heads + h] : 0.f;
    float s = x0 + x1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      float y = __shfl_up_sync(0xffffffff, s, o);
      if (lane >= o) s += y;
    }
    const float c1 = s, c0 = s - x1;
    gam[2 * lane] = c0;
    gam[2 * lane + 1] = c1;
    eg[2 * lane] = __expf(c0);
    eg[2 * lane + 1] = __expf(c1);
    bet[2 * lane] = (2 * lane < n) ? bb[(int64_t)(t0 + a + 2 * lane) * g.heads + h] : 0.f;
    bet[2 * lane + 1] = (2 * lane + 1 < n) ? bb[(int64_t)(t0 + a + 2 * lane + 1) * g.heads + h] : 0.f;
  }
}

__global__ void __launch_bounds__(kGdnThreads, 1)
gdn_chunk_fwd_kernel(GdnGeom g, const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                     const __nv_bfloat16* __restrict__ v, const float* __restrict__ gg, const float* __restrict__ bb,
                     const float* __restrict__ init, __nv_bfloat16* __restrict__ out, float* __restrict__ states,
                     float* __restrict__ final_state, float qscale) {
  extern __shared__ float sm[];
  float* S = sm + FwdSm::S;
  float* Ks = sm + FwdSm::K;
  float* Qs = sm + FwdSm::Q;
  float* Vs = sm + FwdSm::V;
  float* As = sm + FwdSm::A;
  float* KS = sm + FwdSm::KS;
  float* gam = sm + FwdSm::GAM;
  float* bet = gam + kC;
  float* eg = bet + kC;
  const int seq = blockIdx.x / (g.heads * 2);
  const int h = (blockIdx.x / 2) % g.heads;
  const int half = blockIdx.x % 2;
  const int tid = threadIdx.x;
  int t0, len;
  seq_span(g, seq, t0, len);
  // initial state (this half)
  for (int i = tid; i < kDK * kDVH; i += kGdnThreads) {
    const int r = i / kDVH, c = i % kDVH;
    S[i] = init != nullptr ? init[(((int64_t)seq * g.heads + h) * kDK + r) * g.dv + half * kDVH + c] : 0.f;
  }
  __syncthreads();
  const int ty = tid / 16, tx = tid % 16;
  int chunk = g.chunk_off[seq];
  for (int a = 0; a < len; a += kC, ++chunk) {
    const int n = min(kC, len - a);
    // save the chunk's starting state for the backward
    float* st = states + (((int64_t)chunk * g.heads + h) * kDK) * g.dv + half * kDVH;
    for (int i = tid; i < kDK * kDVH; i += kGdnThreads) st[(int64_t)(i / kDVH) * g.dv + i % kDVH] = S[i];
    load_chunk(g, Ks, Qs, Vs, gam, bet, eg, q, k, v, gg, bb, t0, a, n, h, half, qscale);
    __syncthreads();
    // KS = K S0  (C x 64), W = V - e^gamma * KS  (in place in Vs)
    {
      float o[4][4];
      zero(o);
      mm_acc<4, 4>(o, Ks, kDK, 1, S, kDVH, 1, ty * 4, tx * 4, kDK);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = ty * 4 + i, c = tx * 4 + j;
          Vs[r * kDVH + c] = Vs[r * kDVH + c] - eg[r] * o[i][j];
        }
      // A = strictly_lower(beta_t * E_ts * k_t . k_s)
      float kk[4][4];
      zero(kk);
      mm_acc<4, 4>(kk, Ks, kDK, 1, Ks, 1, kDK, ty * 4, tx * 4, kDK);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int t = ty * 4 + i, s = tx * 4 + j;
          As[t * kC + s] = (s < t) ? bet[t] * __expf(gam[t] - gam[s]) * kk[i][j] : 0.f;
        }
    }
    __syncthreads();
    // U = (I + A)^{-1} diag(beta) W: forward substitution, row by row; thread c of 64
    // owns value column c (4 threads per column split the inner sum).
    {
      const int c = tid % kDVH, part = tid / kDVH;  // 4 parts
      for (int t = 0; t < kC; ++t) {
        float acc = 0.f;
        for (int s = part; s < t; s += 4) acc = fmaf(As[t * kC + s], Vs[s * kDVH + c], acc);
        // combine the 4 parts through shared scratch (KS area row t)
        KS[part * kDVH + c] = acc;
        __syncthreads();
        if (part == 0) {
          const float tot = KS[c] + KS[kDVH + c] + KS[2 * kDVH + c] + KS[3 * kDVH + c];
          Vs[t * kDVH + c] = bet[t] * Vs[t * kDVH + c] - tot;
        }
        __syncthreads();
      }
    }
    // P = lower_incl(E * Q K^T) into As (A is no longer needed)
    {
      float qk[4][4];
      zero(qk);
      mm_acc<4, 4>(qk, Qs, kDK, 1, Ks, 1, kDK, ty * 4, tx * 4, kDK);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int t = ty * 4 + i, s = tx * 4 + j;
          As[t * kC + s] = (s <= t) ? __expf(gam[t] - gam[s]) * qk[i][j] : 0.f;
        }
    }
    __syncthreads();
    // O = e^gamma * (Q S0) + P U
    {
      float o[4][4], pu[4][4];
      zero(o);
      zero(pu);
      mm_acc<4, 4>(o, Qs, kDK, 1, S, kDVH, 1, ty * 4, tx * 4, kDK);
      mm_acc<4, 4>(pu, As, kC, 1, Vs, kDVH, 1, ty * 4, tx * 4, kC);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = ty * 4 + i;
        if (r < n) {
          __nv_bfloat16* op = out + (int64_t)(t0 + a + r) * g.row_v + (int64_t)h * g.dv + half * kDVH + tx * 4;
#pragma unroll
          for (int j = 0; j < 4; ++j) op[j] = __float2bfloat16(eg[r] * o[i][j] + pu[i][j]);
        }
      }
    }
    __syncthreads();
    // S <- e^{gamma_C} S + K^T (F * U),  F_s = exp(gamma_C - gamma_s)  (dk x 64; 8x4 tiles)
    {
      const float gl = gam[n - 1];
      // scale U rows by F in place (U in Vs is no longer needed unscaled)
      for (int i = tid; i < kC * kDVH; i += kGdnThreads) {
        const int s = i / kDVH;
        Vs[i] = (s < n) ? Vs[i] * __expf(gl - gam[s]) : 0.f;
      }
      __syncthreads();
      float o[8][4];
      zero(o);
      mm_acc<8, 4>(o, Ks, 1, kDK, Vs, kDVH, 1, ty * 8, tx * 4, n);
      const float egl = __expf(gl);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = ty * 8 + i, c = tx * 4 + j;
          S[r * kDVH + c] = egl * S[r * kDVH + c] + o[i][j];
        }
    }
    __syncthreads();
  }
  if (final_state != nullptr) {
    for (int i = tid; i < kDK * kDVH; i += kGdnThreads) {
      const int r = i / kDVH, c = i % kDVH;
      final_state[(((int64_t)seq * g.heads + h) * kDK + r) * g.dv + half * kDVH + c] = S[i];
    }
  }
}

// ------------------------------------------------------------------------------ backward
struct BwdSm {
  static constexpr int S0 = 0;                      // [dk][64] chunk start state
  static constexpr int DS = S0 + kDK * kDVH;        // [dk][64] carried dS
  static constexpr int K = DS + kDK * kDVH;         // [C][dk]
  static constexpr int Q = K + kC * kDK;            // [C][dk]
  static constexpr int R = Q + kC * kDK;            // [C][64]  V - Gamma K S0
  static constexpr int U = R + kC * kDVH;           // [C][64]
  static constexpr int DU = U + kC * kDVH;          // [C][64]  dU -> dY
  static constexpr int DO = DU + kC * kDVH;         // [C][64]
  static constexpr int A = DO + kC * kDVH;          // [C][C]
  static constexpr int P = A + kC * kC;             // [C][C]   P, then dP-derived
  static constexpr int GAM = P + kC * kC;           // gamma, beta, e^gamma, dgam, dbeta
  static constexpr int TOTAL = GAM + 5 * kC;
};

__global__ void __launch_bounds__(kGdnThreads, 1)
gdn_chunk_bwd_kernel(GdnGeom g, const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                     const __nv_bfloat16* __restrict__ v, const float* __restrict__ gg, const float* __restrict__ bb,
                     const float* __restrict__ states, const __nv_bfloat16* __restrict__ dout,
                     const float* __restrict__ dfinal, float* __restrict__ dq_acc, float* __restrict__ dk_acc,
                     __nv_bfloat16* __restrict__ dv, float* __restrict__ dgam_acc, float* __restrict__ db_acc,
                     float* __restrict__ dinit, float qscale) {
  extern __shared__ float sm[];
  float* S0 = sm + BwdSm::S0;
  float* dS = sm + BwdSm::DS;
  float* Ks = sm + BwdSm::K;
  float* Qs = sm + BwdSm::Q;
  float* Rs = sm + BwdSm::R;
  float* Us = sm + BwdSm::U;
  float* dUs = sm + BwdSm::DU;
  float* dOs = sm + BwdSm::DO;
  float* As = sm + BwdSm::A;
  float* Ps = sm + BwdSm::P;
  float* gam = sm + BwdSm::GAM;
  float* bet = gam + kC;
  float* eg = bet + kC;
  float* dgam = eg + kC;
  float* dbet = dgam + kC;
  const int seq = blockIdx.x / (g.heads * 2);
  const int h = (blockIdx.x / 2) % g.heads;
  const int half = blockIdx.x % 2;
  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  int t0, len;
  seq_span(g, seq, t0, len);
  for (int i = tid; i < kDK * kDVH; i += kGdnThreads) {
    const int r = i / kDVH, c = i % kDVH;
    dS[i] = dfinal != nullptr ? dfinal[(((int64_t)seq * g.heads + h) * kDK + r) * g.dv + half * kDVH + c] : 0.f;
  }
  const int nchunks = (len + kC - 1) / kC;
  for (int ci = nchunks - 1; ci >= 0; --ci) {
    const int a = ci * kC;
    const int n = min(kC, len - a);
    const int chunk = g.chunk_off[seq] + ci;
    __syncthreads();
    const float* st = states + (((int64_t)chunk * g.heads + h) * kDK) * g.dv + half * kDVH;
    for (int i = tid; i < kDK * kDVH; i += kGdnThreads) S0[i] = st[(int64_t)(i / kDVH) * g.dv + i % kDVH];
    load_chunk(g, Ks, Qs, Rs, gam, bet, eg, q, k, v, gg, bb, t0, a, n, h, half, qscale);
    for (int i = tid; i < kC * kDVH; i += kGdnThreads) {
      const int r = i / kDVH, c = i % kDVH;
      dOs[i] = r < n ? __bfloat162float(dout[(int64_t)(t0 + a + r) * g.row_v + (int64_t)h * g.dv + half * kDVH + c])
                     : 0.f;
    }
    if (tid < kC) {
      dgam[tid] = 0.f;
      dbet[tid] = 0.f;
    }
    __syncthreads();
    const float gl = gam[n - 1];
    const float egl = __expf(gl);
    // KS = K S0 -> R = V - e^gamma KS; dgamma partial needs KS too (kept in registers).
    float ks[4][4];
    zero(ks);
    mm_acc<4, 4>(ks, Ks, kDK, 1, S0, kDVH, 1, ty * 4, tx * 4, kDK);
    // A (strictly lower), and keep KK in registers
    float kk[4][4];
    zero(kk);
    mm_acc<4, 4>(kk, Ks, kDK, 1, Ks, 1, kDK, ty * 4, tx * 4, kDK);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = ty * 4 + i, c = tx * 4 + j;
        Rs[r * kDVH + c] = Rs[r * kDVH + c] - eg[r] * ks[i][j];
        As[r * kC + c] = (c < r) ? bet[r] * __expf(gam[r] - gam[c]) * kk[i][j] : 0.f;
      }
    __syncthreads();
    // U = (I + A)^{-1} diag(beta) R  (forward substitution)
    {
      const int c = tid % kDVH, part = tid / kDVH;
      for (int t = 0; t < kC; ++t) {
        float acc = 0.f;
        for (int s = part; s < t; s += 4) acc = fmaf(As[t * kC + s], Us[s * kDVH + c], acc);
        dUs[part * kDVH + c] = acc;
        __syncthreads();
        if (part == 0)
          Us[t * kDVH + c] = bet[t] * Rs[t * kDVH + c] - (dUs[c] + dUs[kDVH + c] + dUs[2 * kDVH + c] + dUs[3 * kDVH + c]);
        __syncthreads();
      }
    }
    // P = lower_incl(E * QK)
    float qk[4][4];
    zero(qk);
    mm_acc<4, 4>(qk, Qs, kDK, 1, Ks, 1, kDK, ty * 4, tx * 4, kDK);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = ty * 4 + i, s = tx * 4 + j;
        Ps[t * kC + s] = (s <= t) ? __expf(gam[t] - gam[s]) * qk[i][j] : 0.f;
      }
    __syncthreads();
    // dU = P^T dO + F * (K dS); also dFw_s = sum_c (K dS)_{s,c} U_{s,c}
    float kds[4][4];
    zero(kds);
    mm_acc<4, 4>(kds, Ks, kDK, 1, dS, kDVH, 1, ty * 4, tx * 4, kDK);
    float ptdo[4][4];
    zero(ptdo);
    mm_acc<4, 4>(ptdo, Ps, 1, kC, dOs, kDVH, 1, ty * 4, tx * 4, kC);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
      const float fw = (r < n) ? __expf(gl - gam[r]) : 0.f;
      float dfw = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = tx * 4 + j;
        dUs[r * kDVH + c] = ptdo[i][j] + fw * kds[i][j];
        dfw += kds[i][j] * Us[r * kDVH + c];
      }
      // dgamma_s -= dFw_s F_s ; dgamma_C += sum_s dFw_s F_s
      atomicAdd(&dgam[r], -dfw * fw);
      atomicAdd(&dgam[n - 1], dfw * fw);
    }
    __syncthreads();
    // dY = (I + A)^{-T} dU: backward substitution, in place in dUs
    {
      const int c = tid % kDVH, part = tid / kDVH;
      float* scratch = Ps;  // 4 x 64 floats; P is rebuilt from the registers below
      for (int t = kC - 1; t >= 0; --t) {
        __syncthreads();  // row t + 1 of dY is written
        float acc = 0.f;
        for (int s = t + 1 + part; s < kC; s += 4) acc = fmaf(As[s * kC + t], dUs[s * kDVH + c], acc);
        scratch[part * kDVH + c] = acc;
        __syncthreads();
        if (part == 0)
          dUs[t * kDVH + c] = dUs[t * kDVH + c] - (scratch[c] + scratch[kDVH + c] + scratch[2 * kDVH + c] +
                                                   scratch[3 * kDVH + c]);
      }
      __syncthreads();
    }
    // rebuild P (its storage served as scratch)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = ty * 4 + i, s = tx * 4 + j;
        Ps[t * kC + s] = (s <= t) ? __expf(gam[t] - gam[s]) * qk[i][j] : 0.f;
      }
    // dR = beta dY -> dV; dbeta += sum_c dY R; dKS = -e^gamma dR; dgamma -= e^gamma KS . dR
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
      float db = 0.f, dgk = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = tx * 4 + j;
        const float dy = dUs[r * kDVH + c];
        const float dr = bet[r] * dy;
        db += dy * Rs[r * kDVH + c];
        dgk += ks[i][j] * dr;
        if (r < n) dv[(int64_t)(t0 + a + r) * g.row_v + (int64_t)h * g.dv + half * kDVH + c] = __float2bfloat16(dr);
      }
      atomicAdd(&dbet[r], db);
      atomicAdd(&dgam[r], -eg[r] * dgk);
    }
    __syncthreads();
    // dA = -dY U^T (strictly lower) and dP = dO U^T (lower incl.), each over this half.
    // Derived C x C terms: dKK = dA * E * beta; dPE = dP * E; contributions to dbeta, dgamma.
    float da[4][4], dp[4][4];
    zero(da);
    zero(dp);
    mm_acc<4, 4>(da, dUs, kDVH, 1, Us, 1, kDVH, ty * 4, tx * 4, kDVH);
    mm_acc<4, 4>(dp, dOs, kDVH, 1, Us, 1, kDVH, ty * 4, tx * 4, kDVH);
    __syncthreads();
    // store dKK in As and dPE in Ps (both C x C), accumulate dbeta / dgamma parts
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = ty * 4 + i;
      float dbt = 0.f, dgt = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int s = tx * 4 + j;
        const float e = __expf(gam[t] - gam[s]);
        float dkk = 0.f, dpe = 0.f;
        if (s < t) {
          const float dA = -da[i][j];
          const float dAE = dA * e;
          dbt += dAE * kk[i][j];
          dkk = dAE * bet[t];
          const float dEA = dAE * bet[t] * kk[i][j];
          dgt += dEA;
          atomicAdd(&dgam[s], -dEA);
        }
        if (s <= t) {
          const float P = e * qk[i][j];
          dpe = dp[i][j] * e;
          const float dEP = dp[i][j] * P;
          dgt += dEP;
          atomicAdd(&dgam[s], -dEP);
        }
        As[t * kC + s] = dkk;
        Ps[t * kC + s] = dpe;
      }
      atomicAdd(&dbet[t], dbt);
      atomicAdd(&dgam[t], dgt);
    }
    __syncthreads();
    // dQ (C x dk; 4 x 8 tiles: ty -> 4 rows, tx -> 8 cols) = dPE K + e^gamma dO S0^T
    // dK = dKS S0^T + dKK K + dKK^T K + dPE^T Q + F (U dS^T), with dKS = -e^gamma dR
    {
      float dqt[4][8], dkt[4][8];
      zero(dqt);
      zero(dkt);
      mm_acc<4, 8>(dqt, Ps, kC, 1, Ks, kDK, 1, ty * 4, tx * 8, kC);
      float tmp[4][8];
      zero(tmp);
      mm_acc<4, 8>(tmp, dOs, kDVH, 1, S0, 1, kDVH, ty * 4, tx * 8, kDVH);  // dO S0^T
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) dqt[i][j] += eg[ty * 4 + i] * tmp[i][j];
      mm_acc<4, 8>(dkt, As, kC, 1, Ks, kDK, 1, ty * 4, tx * 8, kC);   // dKK K
      mm_acc<4, 8>(dkt, As, 1, kC, Ks, kDK, 1, ty * 4, tx * 8, kC);   // dKK^T K
      mm_acc<4, 8>(dkt, Ps, 1, kC, Qs, kDK, 1, ty * 4, tx * 8, kC);   // dPE^T Q
      zero(tmp);
      mm_acc<4, 8>(tmp, dUs, kDVH, 1, S0, 1, kDVH, ty * 4, tx * 8, kDVH);  // dY S0^T
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) dkt[i][j] += -eg[ty * 4 + i] * bet[ty * 4 + i] * tmp[i][j];
      zero(tmp);
      mm_acc<4, 8>(tmp, Us, kDVH, 1, dS, 1, kDVH, ty * 4, tx * 8, kDVH);  // U dS^T
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = ty * 4 + i;
        const float fw = (r < n) ? __expf(gl - gam[r]) : 0.f;
        if (r < n) {
          float* dqp = dq_acc + ((int64_t)(t0 + a + r) * g.heads + h) * kDK + tx * 8;
          float* dkp = dk_acc + ((int64_t)(t0 + a + r) * g.heads + h) * kDK + tx * 8;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            atomicAdd(dqp + j, dqt[i][j]);
            atomicAdd(dkp + j, dkt[i][j] + fw * tmp[i][j]);
          }
        }
      }
    }
    // dgamma from Gamma Q S0 (Q S0 . dO) and from e^{gamma_C} S0 (<S0, dS>)
    {
      float qs[4][4];
      zero(qs);
      mm_acc<4, 4>(qs, Qs, kDK, 1, S0, kDVH, 1, ty * 4, tx * 4, kDK);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = ty * 4 + i;
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) s += qs[i][j] * dOs[r * kDVH + tx * 4 + j];
        atomicAdd(&dgam[r], eg[r] * s);
      }
      float part = 0.f;
      for (int i = tid; i < kDK * kDVH; i += kGdnThreads) part += S0[i] * dS[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffff, part, o);
      if ((tid & 31) == 0) atomicAdd(&dgam[n - 1], egl * part);
    }
    __syncthreads();
    // dS <- e^{gamma_C} dS + K^T dKS + Q^T (e^gamma dO),  dKS = -e^gamma beta dY  (dk x 64)
    for (int i = tid; i < kC * kDVH; i += kGdnThreads) {
      const int r = i / kDVH;
      Rs[i] = -eg[r] * bet[r] * dUs[i];  // dKS (R no longer needed)
      dOs[i] = eg[r] * dOs[i];
    }
    __syncthreads();
    {
      float o[8][4];
      zero(o);
      mm_acc<8, 4>(o, Ks, 1, kDK, Rs, kDVH, 1, ty * 8, tx * 4, kC);
      mm_acc<8, 4>(o, Qs, 1, kDK, dOs, kDVH, 1, ty * 8, tx * 4, kC);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = ty * 8 + i, c = tx * 4 + j;
          dS[r * kDVH + c] = egl * dS[r * kDVH + c] + o[i][j];
        }
    }
    __syncthreads();
    // flush dbeta / dgamma (per chunk, before the reverse cumsum done on the host side)
    if (tid < n) {
      atomicAdd(&db_acc[(int64_t)(t0 + a + tid) * g.heads + h], dbet[tid]);
      atomicAdd(&dgam_acc[(int64_t)(t0 + a + tid) * g.heads + h], dgam[tid]);
    }
  }
  __syncthreads();
  if (dinit != nullptr) {
    for (int i = tid; i < kDK * kDVH; i += kGdnThreads) {
      const int r = i / kDVH, c = i % kDVH;
      dinit[(((int64_t)seq * g.heads + h) * kDK + r) * g.dv + half * kDVH + c] = dS[i];
    }
  }
}

// dg from dgamma: reverse cumulative sum inside every chunk of every sequence; and the
// L2-norm backward of q (with its scale) and k: dx = (dy - y (y . dy)) / ||x||.
__global__ void gdn_post_bwd_kernel(GdnGeom g, const __nv_bfloat16* __restrict__ q,
                                    const __nv_bfloat16* __restrict__ k, const float* __restrict__ dq_acc,
                                    const float* __restrict__ dk_acc, __nv_bfloat16* __restrict__ dq,
                                    __nv_bfloat16* __restrict__ dk, int64_t rows, float qscale) {
  // one warp per (token, head) row of 128
  const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows * g.heads) return;
  const int64_t tok = w / g.heads;
  const int h = (int)(w % g.heads);
  const int64_t base = tok * g.row_q + (int64_t)h * kDK + lane * 4;
  const int64_t abase = w * kDK + lane * 4;
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const __nv_bfloat16* x = which ? k : q;
    const float* dy = which ? dk_acc : dq_acc;
    float xv[4], dv_[4];
    float ss = 0.f, dot = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xv[i] = __bfloat162float(x[base + i]);
      dv_[i] = dy[abase + i] * (which ? 1.f : qscale);
      ss += xv[i] * xv[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
    const float nrm = fmaxf(sqrtf(ss), 1e-6f);
#pragma unroll
    for (int i = 0; i < 4; ++i) dot += (xv[i] / nrm) * dv_[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffff, dot, o);
    __nv_bfloat16* out = which ? dk : dq;
#pragma unroll
    for (int i = 0; i < 4; ++i) out[base + i] = __float2bfloat16((dv_[i] - (xv[i] / nrm) * dot) / nrm);
  }
}

__global__ void gdn_dg_kernel(GdnGeom g, const float* __restrict__ dgam, float* __restrict__ dg) {
  // one thread per (sequence, head, chunk): reverse cumsum over the chunk
  const int64_t id = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int total_chunks = g.chunk_off[g.num_seqs];
  if (id >= (int64_t)total_chunks * g.heads) return;
  const int chunk = (int)(id / g.heads), h = (int)(id % g.heads);
  int lo = 0, hi = g.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (g.chunk_off[mid] <= chunk) lo = mid; else hi = mid - 1;
  }
  int t0, len;
  seq_span(g, lo, t0, len);
  const int a = (chunk - g.chunk_off[lo]) * kC;
  const int n = min(kC, len - a);
  float acc = 0.f;
  for (int i = n - 1; i >= 0; --i) {
    const int64_t idx = (int64_t)(t0 + a + i) * g.heads + h;
    acc += dgam[idx];
    dg[idx] = acc;
  }
}

// ------------------------------------------------------------------------- recurrent
// Token-by-token decoding: one CTA per (batch row, head); state (dk x dv) fp32 in shared
// memory; q/k normalised in-kernel.  Returns the outputs and the final state.
__global__ void __launch_bounds__(kGdnThreads)
gdn_recurrent_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                     const __nv_bfloat16* __restrict__ v, const float* __restrict__ gg, const float* __restrict__ bb,
                     const float* __restrict__ init, __nv_bfloat16* __restrict__ out, float* __restrict__ fin, int T,
                     int H, int dk, int dv, float qscale, bool per_channel) {
  extern __shared__ float sm[];
  float* S = sm;                  // [dk][dv]
  float* kv = S + dk * dv;        // [dk] normalised k
  float* qv = kv + dk;            // [dk]
  float* red = qv + dk;           // [2]
  float* u = red + 32;            // [dv]
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int tid = threadIdx.x;
  for (int i = tid; i < dk * dv; i += blockDim.x) S[i] = init != nullptr ? init[((int64_t)b * H + h) * dk * dv + i] : 0.f;
  for (int t = 0; t < T; ++t) {
    const int64_t row = (int64_t)b * T + t;
    __syncthreads();
    if (tid < 32) {
      float sk = 0.f, sq = 0.f;
      for (int i = tid; i < dk; i += 32) {
        const float a_ = __bfloat162float(k[(row * H + h) * dk + i]);
        const float c_ = __bfloat162float(q[(row * H + h) * dk + i]);
        kv[i] = a_;
        qv[i] = c_;
        sk += a_ * a_;
        sq += c_ * c_;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sk += __shfl_xor_sync(0xffffffff, sk, o);
        sq += __shfl_xor_sync(0xffffffff, sq, o);
      }
      if (tid == 0) {
        red[0] = 1.f / fmaxf(sqrtf(sk), 1e-6f);
        red[1] = qscale / fmaxf(sqrtf(sq), 1e-6f);
      }
    }
    __syncthreads();
    for (int i = tid; i < dk; i += blockDim.x) {
      kv[i] *= red[0];
      qv[i] *= red[1];
    }
    __syncthreads();
    const float beta = bb[row * H + h];
    // decay, then u = beta (v - S^T k)
    for (int i = tid; i < dk * dv; i += blockDim.x) {
      const int r = i / dv;
      const float dec = per_channel ? __expf(gg[(row * H + h) * dk + r]) : __expf(gg[row * H + h]);
      S[i] *= dec;
    }
    __syncthreads();
    for (int c = tid; c < dv; c += blockDim.x) {
      float acc = 0.f;
      for (int r = 0; r < dk; ++r) acc = fmaf(S[r * dv + c], kv[r], acc);
      u[c] = beta * (__bfloat162float(v[(row * H + h) * dv + c]) - acc);
    }
    __syncthreads();
    for (int i = tid; i < dk * dv; i += blockDim.x) S[i] = fmaf(kv[i / dv], u[i % dv], S[i]);
    __syncthreads();
    for (int c = tid; c < dv; c += blockDim.x) {
      float acc = 0.f;
      for (int r = 0; r < dk; ++r) acc = fmaf(S[r * dv + c], qv[r], acc);
      out[(row * H + h) * dv + c] = __float2bfloat16(acc);
    }
  }
  __syncthreads();
  for (int i = tid; i < dk * dv; i += blockDim.x) fin[((int64_t)b * H + h) * dk * dv + i] = S[i];
}

// ---------------------------------------------------------------------- short conv
// y[t, c] = silu(sum_i w[c, i] x[t - K + 1 + i, c]) with zero padding before each
// sequence start (or the initial state for the batch layout).
__global__ void conv1d_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                  const int* __restrict__ cu, const float* __restrict__ init,
                                  __nv_bfloat16* __restrict__ y, float* __restrict__ fin, int B, int T, int D, int K,
                                  int nseq) {
  const int64_t total = (int64_t)B * T * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % D);
    const int64_t bt = i / D;
    const int b = (int)(bt / T), t = (int)(bt % T);
    int start = 0;
    if (cu != nullptr) {  // packed: B == 1, find the document of t
      int lo = 0, hi = nseq - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cu[mid] <= t) lo = mid; else hi = mid - 1;
      }
      start = cu[lo];
    }
    float acc = 0.f;
    for (int j = 0; j < K; ++j) {
      const int tt = t - K + 1 + j;
      float xv = 0.f;
      if (tt >= start) xv = __bfloat162float(x[((int64_t)b * T + tt) * D + c]);
      else if (init != nullptr && cu == nullptr) xv = init[((int64_t)b * D + c) * (K - 1) + (tt + K - 1)];
      acc = fmaf(w[c * K + j], xv, acc);
    }
    y[i] = __float2bfloat16(acc / (1.f + __expf(-acc)));
  }
}

__global__ void conv1d_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                  const float* __restrict__ w, const int* __restrict__ cu, const float* __restrict__ init,
                                  __nv_bfloat16* __restrict__ dx, float* __restrict__ dw, int B, int T, int D, int K,
                                  int nseq) {
  // thread per (b, t, c): recompute z at t (for dz), and accumulate dx from the K outputs
  // t' = t .. t+K-1 of the same sequence; dw via atomics.
  const int64_t total = (int64_t)B * T * D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % D);
    const int64_t bt = i / D;
    const int b = (int)(bt / T), t = (int)(bt % T);
    int start = 0, end = T;
    if (cu != nullptr) {
      int lo = 0, hi = nseq - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cu[mid] <= t) lo = mid; else hi = mid - 1;
      }
      start = cu[lo];
      end = cu[lo + 1];
    }
    // dz at t
    float z = 0.f;
    for (int j = 0; j < K; ++j) {
      const int tt = t - K + 1 + j;
      float xv = 0.f;
      if (tt >= start) xv = __bfloat162float(x[((int64_t)b * T + tt) * D + c]);
      else if (init != nullptr && cu == nullptr) xv = init[((int64_t)b * D + c) * (K - 1) + (tt + K - 1)];
      z = fmaf(w[c * K + j], xv, z);
    }
    const float s = 1.f / (1.f + __expf(-z));
    const float dz = __bfloat162float(dy[i]) * s * (1.f + z * (1.f - s));
    for (int j = 0; j < K; ++j) {
      const int tt = t - K + 1 + j;
      float xv = 0.f;
      if (tt >= start) xv = __bfloat162float(x[((int64_t)b * T + tt) * D + c]);
      else if (init != nullptr && cu == nullptr) xv = init[((int64_t)b * D + c) * (K - 1) + (tt + K - 1)];
      atomicAdd(&dw[c * K + j], dz * xv);
    }
    // dx[t] = sum_j w[c, j] dz[t + K - 1 - j]  (same sequence): recompute dz there
    float acc = 0.f;
    for (int j = 0; j < K; ++j) {
      const int to = t + K - 1 - j;
      if (to >= end) continue;
      float zo = 0.f;
      for (int jj = 0; jj < K; ++jj) {
        const int tt = to - K + 1 + jj;
        float xv = 0.f;
        if (tt >= start) xv = __bfloat162float(x[((int64_t)b * T + tt) * D + c]);
        else if (init != nullptr && cu == nullptr) xv = init[((int64_t)b * D + c) * (K - 1) + (tt + K - 1)];
        zo = fmaf(w[c * K + jj], xv, zo);
      }
      const float so = 1.f / (1.f + __expf(-zo));
      const float dzo = __bfloat162float(dy[((int64_t)b * T + to) * D + c]) * so * (1.f + zo * (1.f - so));
      acc = fmaf(w[c * K + j], dzo, acc);
    }
    dx[i] = __float2bfloat16(acc);
  }
}

// -------------------------------------------------------------------------------- host
static int gdn_grid(int64_t work) {
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)sms * 16));
}

std::vector<torch::Tensor> conv1d_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> cu,
                                      c10::optional<torch::Tensor> init) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 3, "conv1d: bf16 (B, T, D)");
  const int B = x.size(0), T = x.size(1), D = x.size(2), K = w.size(-1);
  auto wf = w.reshape({D, K}).to(at::kFloat).contiguous();
  auto y = torch::empty_like(x);
  const int nseq = cu.has_value() ? cu->numel() - 1 : B;
  auto fin = torch::zeros({nseq, D, K - 1}, x.options().dtype(at::kFloat));
  const float* ip = nullptr;
  torch::Tensor init_f;
  if (init.has_value()) {
    init_f = init->to(at::kFloat).contiguous();
    ip = init_f.data_ptr<float>();
  }
  if (x.numel() > 0) {
    conv1d_fwd_kernel<<<gdn_grid(x.numel()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        (const __nv_bfloat16*)x.data_ptr(), wf.data_ptr<float>(), cu.has_value() ? cu->data_ptr<int>() : nullptr, ip,
        (__nv_bfloat16*)y.data_ptr(), nullptr, B, T, D, K, nseq);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  // final states (the last K-1 inputs of every sequence), assembled on the device
  if (K > 1) {
    if (cu.has_value()) {
      auto cuc = cu->to(at::kLong);
      auto ends = cuc.slice(0, 1);
      for (int j = 0; j < K - 1; ++j) {
        auto idx = ends - (K - 1) + j;
        auto starts = cuc.slice(0, 0, nseq);
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
  const int B = x.size(0), T = x.size(1), D = x.size(2), K = w.size(-1);
  auto wf = w.reshape({D, K}).to(at::kFloat).contiguous();
  auto dx = torch::empty_like(x);
  auto dw = torch::zeros({D, K}, x.options().dtype(at::kFloat));
  const int nseq = cu.has_value() ? cu->numel() - 1 : B;
  torch::Tensor init_f;
  const float* ip = nullptr;
  if (init.has_value()) {
    init_f = init->to(at::kFloat).contiguous();
    ip = init_f.data_ptr<float>();
  }
  auto dyc = dy.to(at::kBFloat16).contiguous();
  if (x.numel() > 0) {
    conv1d_bwd_kernel<<<gdn_grid(x.numel()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        (const __nv_bfloat16*)dyc.data_ptr(), (const __nv_bfloat16*)x.data_ptr(), wf.data_ptr<float>(),
        cu.has_value() ? cu->data_ptr<int>() : nullptr, ip, (__nv_bfloat16*)dx.data_ptr(), dw.data_ptr<float>(), B, T,
        D, K, nseq);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {dx, dw.reshape(w.sizes())};
}

// Chunk offsets are computed on the device (no host synchronisation); total_chunks is the
// host-side upper bound T_total / C + num_seqs used to size the saved-state buffer.
static GdnGeom make_geom(const torch::Tensor& q, const torch::Tensor& v, const c10::optional<torch::Tensor>& cu,
                         torch::Tensor& chunk_off_dev, int& total_chunks) {
  GdnGeom g{};
  const int B = q.size(0), T = q.size(1), H = q.size(2);
  g.heads = H;
  g.row_q = (int64_t)H * q.size(3);
  g.row_v = (int64_t)H * v.size(3);
  g.dv = v.size(3);
  if (cu.has_value()) {
    TORCH_CHECK(B == 1 && cu->scalar_type() == at::kInt, "gdn: packed layout needs batch 1 and int32 cu_seqlens");
    const int n = cu->numel() - 1;
    g.num_seqs = n;
    g.cu = cu->data_ptr<int>();
    auto lens = cu->slice(0, 1) - cu->slice(0, 0, n);
    auto nch = torch::floor_divide(lens + (kC - 1), kC);
    chunk_off_dev = torch::cat({torch::zeros({1}, cu->options()), torch::cumsum(nch, 0, at::kInt)}).contiguous();
    total_chunks = (int)(((int64_t)T + kC - 1) / kC + n);
  } else {
    g.num_seqs = B;
    g.seq_len = T;
    const int per = (T + kC - 1) / kC;
    chunk_off_dev = (torch::arange(B + 1, q.options().dtype(at::kInt)) * per).contiguous();
    total_chunks = B * per;
  }
  g.chunk_off = chunk_off_dev.data_ptr<int>();
  return g;
}

std::vector<torch::Tensor> gdn_chunk_fwd_entry(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor gg,
                                               torch::Tensor beta, c10::optional<torch::Tensor> init,
                                               c10::optional<torch::Tensor> cu, bool per_channel) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(!per_channel, "gdn_chunk_fwd: per-channel (KDA) decay runs on the chunked PyTorch statement");
  TORCH_CHECK(q.size(3) == kDK && v.size(3) == 2 * kDVH && v.size(2) == q.size(2),
              "gdn_chunk_fwd: head_k_dim 128, head_v_dim 128, as many value heads as key heads");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "gdn_chunk_fwd: contiguous q/k/v");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "gdn_chunk_fwd: bf16 q/k/v");
  torch::Tensor chunk_off;
  int total_chunks = 0;
  GdnGeom g = make_geom(q, v, cu, chunk_off, total_chunks);
  const int H = g.heads;
  auto out = torch::empty_like(v);
  auto states = torch::empty({std::max(total_chunks, 1), H, kDK, g.dv}, q.options().dtype(at::kFloat));
  auto fin = torch::empty({g.num_seqs, H, kDK, g.dv}, q.options().dtype(at::kFloat));
  auto gf = gg.to(at::kFloat).contiguous();
  auto bf = beta.to(at::kFloat).contiguous();
  torch::Tensor init_f;
  if (init.has_value()) init_f = init->to(at::kFloat).contiguous();
  const int smem = FwdSm::TOTAL * 4;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  const float qscale = 1.f / std::sqrt((float)kDK);
  if (g.num_seqs > 0 && q.numel() > 0) {
    gdn_chunk_fwd_kernel<<<g.num_seqs * H * 2, kGdnThreads, smem, at::cuda::getCurrentCUDAStream()>>>(
        g, (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)v.data_ptr(),
        gf.data_ptr<float>(), bf.data_ptr<float>(), init.has_value() ? init_f.data_ptr<float>() : nullptr,
        (__nv_bfloat16*)out.data_ptr(), states.data_ptr<float>(), fin.data_ptr<float>(), qscale);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {out, fin, states};
}

std::vector<torch::Tensor> gdn_chunk_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                         torch::Tensor gg, torch::Tensor beta, c10::optional<torch::Tensor> init,
                                         c10::optional<torch::Tensor> cu, std::vector<torch::Tensor> saved,
                                         c10::optional<torch::Tensor> dfinal, bool per_channel) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(!per_channel, "gdn_chunk_bwd: per-channel decay unsupported");
  torch::Tensor chunk_off;
  int total_chunks = 0;
  GdnGeom g = make_geom(q, v, cu, chunk_off, total_chunks);
  const int H = g.heads;
  auto states = saved[0];
  auto gf = gg.to(at::kFloat).contiguous();
  auto bf = beta.to(at::kFloat).contiguous();
  auto doc = dout.to(at::kBFloat16).contiguous();
  const int64_t rows = (int64_t)q.size(0) * q.size(1);
  auto dq_acc = torch::zeros({rows, H, kDK}, q.options().dtype(at::kFloat));
  auto dk_acc = torch::zeros({rows, H, kDK}, q.options().dtype(at::kFloat));
  auto dv = torch::empty_like(v);
  auto dgam = torch::zeros({rows, H}, q.options().dtype(at::kFloat));
  auto db = torch::zeros({rows, H}, q.options().dtype(at::kFloat));
  auto dinit = torch::empty({g.num_seqs, H, kDK, g.dv}, q.options().dtype(at::kFloat));
  torch::Tensor dfin_f;
  if (dfinal.has_value()) dfin_f = dfinal->to(at::kFloat).contiguous();
  const int smem = BwdSm::TOTAL * 4;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  const float qscale = 1.f / std::sqrt((float)kDK);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (g.num_seqs > 0 && rows > 0) {
    gdn_chunk_bwd_kernel<<<g.num_seqs * H * 2, kGdnThreads, smem, st>>>(
        g, (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)v.data_ptr(),
        gf.data_ptr<float>(), bf.data_ptr<float>(), states.data_ptr<float>(), (const __nv_bfloat16*)doc.data_ptr(),
        dfinal.has_value() ? dfin_f.data_ptr<float>() : nullptr, dq_acc.data_ptr<float>(), dk_acc.data_ptr<float>(), (__nv_bfloat16*)dv.data_ptr(),
        dgam.data_ptr<float>(), db.data_ptr<float>(), dinit.data_ptr<float>(), qscale);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  auto dq = torch::empty_like(q), dk = torch::empty_like(k);
  auto dg = torch::empty_like(dgam);
  if (rows > 0) {
    gdn_post_bwd_kernel<<<(unsigned)((rows * H * 32 + 255) / 256), 256, 0, st>>>(
        g, (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)k.data_ptr(), dq_acc.data_ptr<float>(),
        dk_acc.data_ptr<float>(), (__nv_bfloat16*)dq.data_ptr(), (__nv_bfloat16*)dk.data_ptr(), rows, qscale);
    gdn_dg_kernel<<<(unsigned)(((int64_t)total_chunks * H + 255) / 256), 256, 0, st>>>(g, dgam.data_ptr<float>(),
                                                                                    dg.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return {dq, dk, dv, dg.view(gg.sizes()), db.view(beta.sizes()), dinit};
}

std::vector<torch::Tensor> gdn_recurrent(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor gg,
                                         torch::Tensor beta, c10::optional<torch::Tensor> init, bool per_channel) {
  c10::cuda::CUDAGuard guard(q.device());
  const int B = q.size(0), T = q.size(1), H = q.size(2), dk = q.size(3), dv = v.size(3);
  auto out = torch::empty_like(v);
  auto fin = torch::empty({B, H, dk, dv}, q.options().dtype(at::kFloat));
  auto gf = gg.to(at::kFloat).contiguous();
  auto bf = beta.to(at::kFloat).contiguous();
  torch::Tensor init_f;
  if (init.has_value()) init_f = init->to(at::kFloat).contiguous();
  const int smem = (dk * dv + 2 * dk + 32 + dv) * 4;
  TORCH_CHECK(smem <= 227 * 1024, "gdn_recurrent: state too large");
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_recurrent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    configured = true;
  }
  gdn_recurrent_kernel<<<B * H, kGdnThreads, smem, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)q.data_ptr(), (const __nv_bfloat16*)k.data_ptr(), (const __nv_bfloat16*)v.data_ptr(),
      gf.data_ptr<float>(), bf.data_ptr<float>(), init.has_value() ? init_f.data_ptr<float>() : nullptr,
      (__nv_bfloat16*)out.data_ptr(), fin.data_ptr<float>(), T, H, dk, dv, 1.f / std::sqrt((float)dk), per_channel);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {out, fin};
}

}  // namespace mykb
