// Split-KV attention for decoding over static KV caches (flash-decoding).
//
// A decode step has a handful of queries per sequence (the verify window of speculative
// decoding: 1 + drafts) against thousands of cached keys.  The prefill kernel gives one
// CTA per (128-query tile, head), so a decode step would run on batch x heads CTAs, each
// walking the whole cache.  Here the keys are split instead: a warp owns a run of 32-key
// tiles of one (sequence, KV head) and all the query rows of that KV head's group (GQA
// heads x queries, at most 16 rows = one MMA row tile); it streams the tiles through a
// double-buffered cp.async pipeline and computes S = Q K^T and P V on the tensor cores
// (bf16 MMA, fp32 accumulate) with an online softmax.  The 4 warps of a CTA merge their
// (m, l, O) in shared memory; the last CTA of a (sequence, KV head) to finish (atomic
// ticket, nothing waits) merges the CTAs in a fixed order, so results are deterministic.
// The number of tiles per warp is chosen so that the grid is about four CTAs per SM.
//
// Semantics match the prefill kernel's KV-cache path: queries are aligned to the end of
// the visible keys (query i of L sits at position seqused - L + i), window (left, right)
// with -1 meaning unbounded, rows that see no key output 0.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace mykb {
namespace fadec {

typedef __nv_bfloat16 bf16;
constexpr int ROWS = 16;        // query rows per KV head (GQA group x queries)
constexpr int KEYS = 32;        // keys per tile; a warp walks consecutive tiles
constexpr int WARPS = 4;
constexpr int STAGES = 3;       // tiles per warp in its shared-memory ring (two in flight while one is used)

struct Params {
  const bf16* q;       // (B, L, H, D) with strides
  const bf16* k;       // (B, cap, Hkv, D) contiguous
  const bf16* v;
  const int* seqused;  // (B) visible keys per sequence
  bf16* o;             // (B, L, H, D) contiguous
  float* work;         // [B][Hkv][splits][ROWS][D] per-CTA partial O, then [.][.][splits][ROWS] m, l
  float* ml;
  int* tickets;        // [B * Hkv]
  int64_t q_sb, q_st, q_sh;
  int B, L, H, Hkv, cap, splits;  // splits = CTAs per (b, hkv)
  int tiles;                      // key tiles per warp
  float scale_log2;
  int left, right;
};

__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
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
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Is key j visible from row r (r = g * L + i: GQA head g of the group, query i)?
__device__ __forceinline__ bool visible(const Params& p, int r, int j, int rows, int kv_len) {
  if (r >= rows || j >= kv_len) return false;
  const int qpos = kv_len - p.L + (r % p.L);
  if (p.right >= 0 && j > qpos + p.right) return false;
  if (p.left >= 0 && j < qpos - p.left) return false;
  return true;
}

// Shared-memory tiles are unpadded rows of D bf16 with the 16-byte chunks of row r stored
// at chunk index c ^ (r & 7): the eight rows an ldmatrix phase reads then hit eight
// different bank groups.
template <int D>
__device__ __forceinline__ int swz(int r, int col) {
  return r * D + ((((col >> 3) ^ (r & 7)) << 3) | (col & 7));
}

template <int D>
__global__ void __launch_bounds__(WARPS * 32) fa_decode_kernel(Params p) {
  extern __shared__ __align__(128) unsigned char smraw[];
  bf16* Qs = reinterpret_cast<bf16*>(smraw);  // [ROWS][D] (swizzled)
  bf16* KV = Qs + ROWS * D;                    // [WARPS][STAGES][K, V][KEYS][D] (swizzled)
  __shared__ int last;
  __shared__ float rowM[ROWS], rowL[ROWS];
  __shared__ float wM[WARPS][ROWS], wL[WARPS][ROWS];
  const int ctas = p.splits;
  const int bh = blockIdx.x / ctas, cta = blockIdx.x % ctas;
  const int b = bh / p.Hkv, hk = bh % p.Hkv;
  const int G = p.H / p.Hkv, rows = G * p.L;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kv_len = min(p.seqused[b], p.cap);
  // this warp's contiguous key range: the visible keys split evenly over all warps of (b, hk)
  const int T = (kv_len + ctas * WARPS * KEYS - 1) / (ctas * WARPS * KEYS);
  const int key0 = (cta * WARPS + warp) * KEYS * T;
  const int64_t kv_row = (int64_t)p.Hkv * D;
  const bf16* kb = p.k + ((int64_t)b * p.cap) * kv_row + (int64_t)hk * D;
  const bf16* vb = p.v + ((int64_t)b * p.cap) * kv_row + (int64_t)hk * D;
  for (int e = tid; e < ROWS * (D / 8); e += WARPS * 32) {
    const int r = e / (D / 8), c = (e % (D / 8)) * 8;
    const bool ok = r < rows;
    const int g = ok ? r / p.L : 0, i = ok ? r % p.L : 0;
    cp16(Qs + swz<D>(r, c), p.q + b * p.q_sb + i * p.q_st + (int64_t)(hk * G + g) * p.q_sh + c, ok);
  }
  bf16* wbuf = KV + warp * STAGES * 2 * KEYS * D;
  auto load_tile = [&](int t) {
    bf16* ks = wbuf + (t % STAGES) * 2 * KEYS * D;
    bf16* vs = ks + KEYS * D;
    const int base = key0 + t * KEYS;
#pragma unroll 4
    for (int e = lane; e < KEYS * (D / 8); e += 32) {
      const int r = e / (D / 8), c = (e % (D / 8)) * 8;
      const bool ok = base + r < kv_len;
      const int64_t off = (int64_t)(ok ? base + r : 0) * kv_row + c;
      cp16(ks + swz<D>(r, c), kb + off, ok);
      cp16(vs + swz<D>(r, c), vb + off, ok);
    }
  };
  asm volatile("cp.async.commit_group;" ::: "memory");  // group: Q
  // tiles past the visible keys are skipped (they would only be masked)
  const int nt = max(0, min(T, (kv_len - key0 + KEYS - 1) / KEYS));
  // prologue: STAGES - 1 tiles in flight (empty groups keep the group count uniform)
#pragma unroll
  for (int t = 0; t < STAGES - 1; ++t) {
    if (t < nt) load_tile(t);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  asm volatile("cp.async.wait_group %0;" ::"n"(STAGES - 1) : "memory");
  __syncthreads();  // Q is visible to every warp
  const int rr = lane & 7, mat = lane >> 3, gq = lane >> 2, cq = (lane & 3) * 2;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  for (int t = 0; t < nt; ++t) {
    if (t + STAGES - 1 < nt) load_tile(t + STAGES - 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group %0;" ::"n"(STAGES - 1) : "memory");  // tile t has landed
    __syncwarp();
    const bf16* ks = wbuf + (t % STAGES) * 2 * KEYS * D;
    const bf16* vs = ks + KEYS * D;
    float s[KEYS / 8][4];
#pragma unroll
    for (int j = 0; j < KEYS / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < D; k0 += 16) {
      uint32_t a[4];
      ldsm4(a, Qs + swz<D>(lane & 15, k0 + (lane >> 4) * 8));
#pragma unroll
      for (int j = 0; j < KEYS / 8; j += 2) {
        uint32_t bq[4];
        ldsm4(bq, ks + swz<D>(j * 8 + rr + (mat >> 1) * 8, k0 + (mat & 1) * 8));
        mma(s[j], a, bq[0], bq[1]);
        mma(s[j + 1], a, bq[2], bq[3]);
      }
    }
    const int base = key0 + t * KEYS;
    float mt[2] = {m[0], m[1]};
#pragma unroll
    for (int j = 0; j < KEYS / 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = gq + (e >> 1) * 8, col = base + j * 8 + cq + (e & 1);
        s[j][e] = visible(p, r, col, rows, kv_len) ? s[j][e] * p.scale_log2 : -INFINITY;
        mt[e >> 1] = fmaxf(mt[e >> 1], s[j][e]);
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffff, mt[h], 1));
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffff, mt[h], 2));
    }
    float corr[2], ls[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) corr[h] = (mt[h] == -INFINITY || m[h] == -INFINITY) ? (m[h] == -INFINITY ? 0.f : 1.f)
                                                                                      : exp2f(m[h] - mt[h]);
#pragma unroll
    for (int j = 0; j < KEYS / 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = mt[e >> 1];
        s[j][e] = mm == -INFINITY ? 0.f : exp2f(s[j][e] - mm);
        ls[e >> 1] += s[j][e];
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ls[h] += __shfl_xor_sync(0xffffffff, ls[h], 1);
      ls[h] += __shfl_xor_sync(0xffffffff, ls[h], 2);
      l[h] = l[h] * corr[h] + ls[h];
      m[h] = mt[h];
    }
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= corr[0], o[n][1] *= corr[0], o[n][2] *= corr[1], o[n][3] *= corr[1];
    }
#pragma unroll
    for (int kt = 0; kt < KEYS / 16; ++kt) {
      uint32_t a[4];
      a[0] = pack2(s[2 * kt][0], s[2 * kt][1]);
      a[1] = pack2(s[2 * kt][2], s[2 * kt][3]);
      a[2] = pack2(s[2 * kt + 1][0], s[2 * kt + 1][1]);
      a[3] = pack2(s[2 * kt + 1][2], s[2 * kt + 1][3]);
#pragma unroll
      for (int n = 0; n < D / 8; n += 2) {
        uint32_t bv[4];
        ldsm4t(bv, vs + swz<D>(kt * 16 + (mat & 1) * 8 + rr, n * 8 + (mat >> 1) * 8));
        mma(o[n], a, bv[0], bv[1]);
        mma(o[n + 1], a, bv[2], bv[3]);
      }
    }
    __syncwarp();  // this stage is refilled by the load STAGES - 1 tiles ahead
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  // merge the warps of this CTA through shared memory (reusing the K/V buffers)
  __syncthreads();
  float* Ow = reinterpret_cast<float*>(KV);  // [WARPS][ROWS][D]
  if ((lane & 3) == 0) {
    wM[warp][gq] = m[0], wL[warp][gq] = l[0];
    wM[warp][gq + 8] = m[1], wL[warp][gq + 8] = l[1];
  }
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    *reinterpret_cast<float2*>(Ow + (warp * ROWS + gq) * D + n * 8 + cq) = make_float2(o[n][0], o[n][1]);
    *reinterpret_cast<float2*>(Ow + (warp * ROWS + gq + 8) * D + n * 8 + cq) = make_float2(o[n][2], o[n][3]);
  }
  __syncthreads();
  if (tid < ROWS) {
    float M = -INFINITY;
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, wM[w][tid]);
    float L = 0.f;
    if (M != -INFINITY)
      for (int w = 0; w < WARPS; ++w)
        if (wM[w][tid] != -INFINITY) L += exp2f(wM[w][tid] - M) * wL[w][tid];
    rowM[tid] = M, rowL[tid] = L;
    float* wml = p.ml + ((int64_t)bh * ctas + cta) * ROWS * 2;
    wml[tid * 2] = M;
    wml[tid * 2 + 1] = L;
  }
  __syncthreads();
  float* wo = p.work + ((int64_t)bh * ctas + cta) * ROWS * D;
  for (int e = tid; e < ROWS * D; e += WARPS * 32) {
    const int r = e / D;
    const float M = rowM[r];
    float acc = 0.f;
    if (M != -INFINITY)
      for (int w = 0; w < WARPS; ++w)
        if (wM[w][r] != -INFINITY) acc += exp2f(wM[w][r] - M) * Ow[(w * ROWS) * D + e];
    wo[e] = acc;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = (atomicAdd(&p.tickets[bh], 1) == ctas - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  // merge the CTAs of (b, hk): O = sum_c e^{m_c - M} O_c / sum_c e^{m_c - M} l_c
  const float* ml = p.ml + (int64_t)bh * ctas * ROWS * 2;
  if (tid < ROWS) {
    float M = -INFINITY;
    for (int c = 0; c < ctas; ++c) M = fmaxf(M, __ldcg(ml + (c * ROWS + tid) * 2));
    float L = 0.f;
    if (M != -INFINITY)
      for (int c = 0; c < ctas; ++c) {
        const float mc = __ldcg(ml + (c * ROWS + tid) * 2);
        if (mc != -INFINITY) L += exp2f(mc - M) * __ldcg(ml + (c * ROWS + tid) * 2 + 1);
      }
    rowM[tid] = M;
    rowL[tid] = L;
  }
  __syncthreads();
  const float* wb = p.work + (int64_t)bh * ctas * ROWS * D;
  for (int e = tid; e < rows * D; e += WARPS * 32) {
    const int r = e / D, d = e % D;
    const float M = rowM[r], L = rowL[r];
    float acc = 0.f;
    if (L > 0.f)
      for (int c = 0; c < ctas; ++c) {
        const float mc = __ldcg(ml + (c * ROWS + r) * 2);
        if (mc != -INFINITY) acc += exp2f(mc - M) * __ldcg(wb + (c * ROWS + r) * D + d);
      }
    const int g = r / p.L, i = r % p.L;
    p.o[(((int64_t)b * p.L + i) * p.H + hk * G + g) * D + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
  }
  if (tid == 0) p.tickets[bh] = 0;
}

}  // namespace fadec

// q (B, L, H, D) bf16 with a contiguous last dim; k_cache / v_cache (B, cap, Hkv, D)
// contiguous bf16; seqused (B) int32 visible keys.  Needs (H / Hkv) * L <= 16.
torch::Tensor fa_decode(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor seqused,
                        double scale, int64_t left, int64_t right) {
  using namespace fadec;
  TORCH_CHECK(q.is_cuda() && q.dim() == 4 && k_cache.dim() == 4 && v_cache.sizes() == k_cache.sizes(),
              "fa_decode: q (B, L, H, D), caches (B, cap, Hkv, D)");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16 &&
                  v_cache.scalar_type() == at::kBFloat16,
              "fa_decode: bf16 tensors");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && q.stride(3) == 1, "fa_decode: layouts");
  TORCH_CHECK(seqused.scalar_type() == at::kInt && seqused.numel() == q.size(0), "fa_decode: int32 seqused (B)");
  const int B = q.size(0), L = q.size(1), H = q.size(2), D = q.size(3);
  const int cap = k_cache.size(1), Hkv = k_cache.size(2);
  TORCH_CHECK(k_cache.size(0) == B && k_cache.size(3) == D && H % Hkv == 0, "fa_decode: shapes");
  TORCH_CHECK((H / Hkv) * L <= ROWS, "fa_decode: (heads per KV head) x queries must be <= 16");
  TORCH_CHECK(D == 64 || D == 128, "fa_decode: head_dim 64 or 128");
  TORCH_CHECK(q.stride(2) % 8 == 0 && q.stride(1) % 8 == 0 && q.stride(0) % 8 == 0 &&
                  ((uintptr_t)q.data_ptr() % 16) == 0,
              "fa_decode: 16-byte aligned query rows");
  c10::cuda::CUDAGuard guard(q.device());
  auto o = torch::empty({B, L, H, D}, q.options());
  const int max_tiles = std::max(1, (cap + KEYS * WARPS - 1) / (KEYS * WARPS));  // tiles per warp at one CTA
  static int sms[64] = {0};
  if (!sms[q.get_device()]) cudaDeviceGetAttribute(&sms[q.get_device()], cudaDevAttrMultiProcessorCount, q.get_device());
  const int64_t target = 4LL * sms[q.get_device()];
  const int64_t want = ((int64_t)cap * B * Hkv + (int64_t)KEYS * WARPS * target - 1) / ((int64_t)KEYS * WARPS * target);
  const int tiles = (int)std::max<int64_t>(1, std::min<int64_t>(max_tiles, want));
  const int ctas = std::max(1, (cap + KEYS * WARPS * tiles - 1) / (KEYS * WARPS * tiles));
  Params p{};
  p.q = (const bf16*)q.data_ptr();
  p.k = (const bf16*)k_cache.data_ptr();
  p.v = (const bf16*)v_cache.data_ptr();
  p.seqused = seqused.data_ptr<int>();
  p.o = (bf16*)o.data_ptr();
  p.q_sb = q.stride(0), p.q_st = q.stride(1), p.q_sh = q.stride(2);
  p.B = B, p.L = L, p.H = H, p.Hkv = Hkv, p.cap = cap;
  p.splits = ctas;
  p.tiles = tiles;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.left = (int)left, p.right = (int)right;
  const int64_t slots = (int64_t)B * Hkv * p.splits;
  auto work = torch::empty({slots * ROWS * (D + 2)}, q.options().dtype(at::kFloat));
  p.work = work.data_ptr<float>();
  p.ml = p.work + slots * ROWS * D;
  p.tickets = ticket_region(B * Hkv);
  const int grid = B * Hkv * ctas;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  static SmemOptIn attr64, attr128;
  const size_t smem = (size_t)(ROWS + STAGES * 2 * WARPS * KEYS) * D * sizeof(bf16);
  if (D == 64) {
    C10_CUDA_CHECK(attr64.ensure(fa_decode_kernel<64>, (int)smem));
    fa_decode_kernel<64><<<grid, WARPS * 32, smem, st>>>(p);
  } else {
    C10_CUDA_CHECK(attr128.ensure(fa_decode_kernel<128>, (int)smem));
    fa_decode_kernel<128><<<grid, WARPS * 32, smem, st>>>(p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return o;
}

namespace fadec {
// k/v (B, T, Hkv, D) -> caches at positions seqlens[b] + t (one launch for both).
__global__ void kv_append_kernel(const uint4* __restrict__ k, const uint4* __restrict__ v, uint4* __restrict__ kc,
                                 uint4* __restrict__ vc, const int* __restrict__ seqlens, int T, int cap,
                                 int row_vec, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bt = i / row_vec;
    const int c = (int)(i % row_vec);
    const int b = (int)(bt / T), t = (int)(bt % T);
    const int pos = seqlens[b] + t;
    if (pos >= cap) continue;
    const int64_t dst = ((int64_t)b * cap + pos) * row_vec + c;
    kc[dst] = k[i];
    vc[dst] = v[i];
  }
}
}  // namespace fadec

void kv_append(torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor k, torch::Tensor v,
               torch::Tensor seqlens) {
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.sizes() == v_cache.sizes() &&
                  k_cache.dim() == 4,
              "kv_append: contiguous (B, cap, Hkv, D) caches");
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == k_cache.size(0) && k.size(2) == k_cache.size(2) &&
                  k.size(3) == k_cache.size(3) && k.scalar_type() == k_cache.scalar_type(),
              "kv_append: new keys/values must match the caches");
  TORCH_CHECK(seqlens.scalar_type() == at::kInt && seqlens.numel() == k.size(0), "kv_append: int32 seqlens (B)");
  c10::cuda::CUDAGuard guard(k.device());
  auto kk = k.contiguous(), vv = v.contiguous();
  const int64_t row_bytes = k.size(2) * k.size(3) * k.element_size();
  TORCH_CHECK(row_bytes % 16 == 0, "kv_append: rows must be multiples of 16 bytes");
  const int row_vec = (int)(row_bytes / 16);
  const int64_t total = k.size(0) * k.size(1) * row_vec;
  if (total == 0) return;
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((total + threads - 1) / threads, 4096);
  fadec::kv_append_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const uint4*)kk.data_ptr(), (const uint4*)vv.data_ptr(), (uint4*)k_cache.data_ptr(),
      (uint4*)v_cache.data_ptr(), seqlens.data_ptr<int>(), (int)k.size(1), (int)k_cache.size(1), row_vec, total);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
