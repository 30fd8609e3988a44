// Skinny GEMM for decode / small batches: D (M x N) = A (M x K) . W (N x K)^T with M <= 256.
//
// Decode-time linears multiply a handful of token rows by a large weight: the time is the
// weight read, and a 128 x 256 output tile leaves most SMs idle (N = 1024 gives four
// tiles).  Here a CTA owns 64 output columns and one slice of K; the K slices (split-K)
// are chosen so that about two CTAs per SM stream the weight once, each through a
// 4-stage cp.async pipeline of 64-wide K chunks.  Warps multiply on the tensor cores with
// bf16 MMAs (fp32 accumulate) fed by ldmatrix.  Split-K partials go to an fp32 workspace;
// the last CTA of a column tile to finish (atomic ticket, no waiting) adds them in a fixed
// order and writes D, so results are deterministic and the whole GEMM is one launch.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace mykb {
namespace skinny {

typedef __nv_bfloat16 bf16;
constexpr int BN = 64;       // output columns per CTA
constexpr int BK = 64;       // K chunk
constexpr int LDS = BK + 8;  // padded smem row (elements)
constexpr int STAGES = 4;
constexpr int THREADS = 128;

__device__ __forceinline__ void cp16(void* dst, const void* src, bool valid) {
  // zero-fills the 16 bytes when !valid (no bytes are read)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const bf16* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
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

struct Params {
  const bf16* A;
  const bf16* W;
  void* D;
  float* work;   // [tiles][splits][64 x 64] partials (splits > 1)
  int* tickets;  // [tiles], zero on entry, left zero on exit
  int64_t lda, ldw, ldd;
  int M, N, K;
  int splits, chunks_per_split;
  bool out_f32;
};

template <int MT, int WM>  // 16-row tiles per warp, warps along M (rows of the tile = WM * MT * 16)
__global__ void __launch_bounds__(THREADS * WM) skinny_gemm_kernel(Params p) {
  constexpr int RT = WM * MT * 16;
  extern __shared__ __align__(16) unsigned char smraw[];
  bf16* As = reinterpret_cast<bf16*>(smraw);  // [STAGES][RT][LDS]
  bf16* Ws = As + STAGES * RT * LDS;           // [STAGES][64][LDS]
  __shared__ int last;
  const int tile = blockIdx.x / p.splits, split = blockIdx.x % p.splits;
  const int n0 = tile * BN;
  const int nchunks = (p.K + BK - 1) / BK;
  const int c0 = split * p.chunks_per_split;
  const int c1 = min(nchunks, c0 + p.chunks_per_split);
  const int tid = threadIdx.x, lane = tid & 31;
  const int warp = (tid >> 5) & 3, wrow = tid >> 7;  // column group, row group
  const int m_base = wrow * MT * 16;

  auto load = [&](int chunk, int stage) {
    const int k0 = chunk * BK;
    bf16* a = As + stage * RT * LDS;
    bf16* w = Ws + stage * BN * LDS;
    for (int i = tid; i < RT * 8; i += THREADS * WM) {
      const int r = i >> 3, c = (i & 7) * 8;
      const bool ok = r < p.M && k0 + c < p.K;
      cp16(a + r * LDS + c, p.A + (ok ? (int64_t)r * p.lda + k0 + c : 0), ok);
    }
    for (int i = tid; i < BN * 8; i += THREADS * WM) {
      const int r = i >> 3, c = (i & 7) * 8;
      const bool ok = n0 + r < p.N && k0 + c < p.K;
      cp16(w + r * LDS + c, p.W + (ok ? (int64_t)(n0 + r) * p.ldw + k0 + c : 0), ok);
    }
  };

  float acc[MT][2][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 2; ++j) acc[m][j][0] = acc[m][j][1] = acc[m][j][2] = acc[m][j][3] = 0.f;

  const int n = max(c1 - c0, 0);
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < n) load(c0 + s, s);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  const int r = lane & 7, mat = lane >> 3;
  for (int i = 0; i < n; ++i) {
    if (i + STAGES - 1 < n) load(c0 + i + STAGES - 1, (i + STAGES - 1) % STAGES);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group %0;" ::"n"(STAGES - 1) : "memory");
    __syncthreads();
    const bf16* a = As + (i % STAGES) * RT * LDS;
    const bf16* w = Ws + (i % STAGES) * BN * LDS;
#pragma unroll
    for (int k = 0; k < BK; k += 16) {
      uint32_t b[4];  // columns warp*16 .. +15 (two n8 tiles), W stored [n][k]
      ldsm4(b, w + (warp * 16 + r + (mat >> 1) * 8) * LDS + k + (mat & 1) * 8);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        uint32_t af[4];
        ldsm4(af, a + (m_base + m * 16 + (lane & 15)) * LDS + k + (lane >> 4) * 8);
        mma(acc[m][0], af, b[0], b[1]);
        mma(acc[m][1], af, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");

  const int gq = lane >> 2, cq = (lane & 3) * 2;
  if (p.splits == 1) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int row = m_base + m * 16 + gq + hf * 8, col = n0 + warp * 16 + j * 8 + cq;
          if (row >= p.M || col >= p.N) continue;
          const float x = acc[m][j][2 * hf], y = acc[m][j][2 * hf + 1];
          if (p.out_f32) {
            float* d = reinterpret_cast<float*>(p.D) + (int64_t)row * p.ldd + col;
            d[0] = x;
            if (col + 1 < p.N) d[1] = y;
          } else {
            bf16* d = reinterpret_cast<bf16*>(p.D) + (int64_t)row * p.ldd + col;
            d[0] = __float2bfloat16(x);
            if (col + 1 < p.N) d[1] = __float2bfloat16(y);
          }
        }
    return;
  }
  // split-K: partial tile to the workspace, then the last CTA of the tile reduces
  float* part = p.work + ((int64_t)tile * p.splits + split) * (RT * BN);
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int row = m_base + m * 16 + gq + hf * 8, col = warp * 16 + j * 8 + cq;
        *reinterpret_cast<float2*>(part + row * BN + col) = make_float2(acc[m][j][2 * hf], acc[m][j][2 * hf + 1]);
      }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = (atomicAdd(&p.tickets[tile], 1) == p.splits - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* base = p.work + (int64_t)tile * p.splits * (RT * BN);
  for (int e = tid; e < p.M * BN; e += THREADS * WM) {
    const int row = e / BN, col = e % BN;
    if (n0 + col >= p.N) continue;
    float s = 0.f;
    for (int k = 0; k < p.splits; ++k) s += __ldcg(base + k * (RT * BN) + row * BN + col);
    if (p.out_f32) reinterpret_cast<float*>(p.D)[(int64_t)row * p.ldd + n0 + col] = s;
    else reinterpret_cast<bf16*>(p.D)[(int64_t)row * p.ldd + n0 + col] = __float2bfloat16(s);
  }
  if (tid == 0) p.tickets[tile] = 0;
}

}  // namespace skinny

static int skinny_sms(int dev) {
  static int cached[64] = {0};
  if (!cached[dev]) cudaDeviceGetAttribute(&cached[dev], cudaDevAttrMultiProcessorCount, dev);
  return cached[dev];
}

template <int MT, int WM>
static void skinny_launch(const skinny::Params& p, int grid, cudaStream_t st) {
  using namespace skinny;
  const size_t smem = (size_t)STAGES * (WM * MT * 16 + BN) * LDS * sizeof(bf16);
  static SmemOptIn attr;
  C10_CUDA_CHECK(attr.ensure(skinny_gemm_kernel<MT, WM>, (int)smem));
  skinny_gemm_kernel<MT, WM><<<grid, THREADS * WM, smem, st>>>(p);
}

// a (M, K) with M <= 256, w (N, K), both bf16 with contiguous K; d (M, N) bf16 or fp32.
void gemm_skinny(torch::Tensor a, torch::Tensor w, torch::Tensor d) {
  using namespace skinny;
  TORCH_CHECK(a.is_cuda() && w.is_cuda() && d.is_cuda() && a.dim() == 2 && w.dim() == 2 && d.dim() == 2,
              "gemm_skinny: 2-D CUDA tensors");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm_skinny: bf16 operands");
  TORCH_CHECK(d.scalar_type() == at::kBFloat16 || d.scalar_type() == at::kFloat, "gemm_skinny: bf16 or fp32 output");
  const int M = a.size(0), K = a.size(1), N = w.size(0);
  TORCH_CHECK(M >= 1 && M <= 256 && w.size(1) == K && d.size(0) == M && d.size(1) == N, "gemm_skinny: shapes");
  TORCH_CHECK(a.stride(1) == 1 && w.stride(1) == 1 && d.stride(1) == 1 && K % 8 == 0 && a.stride(0) % 8 == 0 &&
                  w.stride(0) % 8 == 0,
              "gemm_skinny: contiguous K, K and row strides multiples of 8");
  TORCH_CHECK(((uintptr_t)a.data_ptr() % 16) == 0 && ((uintptr_t)w.data_ptr() % 16) == 0,
              "gemm_skinny: 16-byte aligned operands");
  c10::cuda::CUDAGuard guard(a.device());
  const int MT = M <= 64 ? (M + 15) / 16 : 8;
  const int WM = M <= 128 ? 1 : 2;
  const int RT = WM * MT * 16;
  const int tiles = (N + BN - 1) / BN;
  const int nchunks = (K + BK - 1) / BK;
  const int target = 2 * skinny_sms(a.get_device());
  int splits = std::max(1, std::min(nchunks, (target + tiles - 1) / tiles));
  const int per = (nchunks + splits - 1) / splits;
  splits = (nchunks + per - 1) / per;
  Params p{};
  p.A = (const bf16*)a.data_ptr();
  p.W = (const bf16*)w.data_ptr();
  p.D = d.data_ptr();
  p.lda = a.stride(0);
  p.ldw = w.stride(0);
  p.ldd = d.stride(0);
  p.M = M, p.N = N, p.K = K;
  p.splits = splits;
  p.chunks_per_split = per;
  p.out_f32 = d.scalar_type() == at::kFloat;
  torch::Tensor work;
  if (splits > 1) {
    work = torch::empty({(int64_t)tiles * splits * RT * BN}, a.options().dtype(at::kFloat));
    p.work = work.data_ptr<float>();
    p.tickets = ticket_region(tiles);
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int grid = tiles * splits;
  if (WM == 2) skinny_launch<8, 2>(p, grid, st);
  else if (MT == 8) skinny_launch<8, 1>(p, grid, st);
  else if (MT == 1) skinny_launch<1, 1>(p, grid, st);
  else if (MT == 2) skinny_launch<2, 1>(p, grid, st);
  else if (MT == 3) skinny_launch<3, 1>(p, grid, st);
  else skinny_launch<4, 1>(p, grid, st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
