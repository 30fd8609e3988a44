// MXFP8 (OCP microscaling fp8) training kernels for sm100a:
//
//  * mx_quantize: one read of a bf16 matrix X (R x C) produces, as asked,
//      - dim0: X in fp8 (E4M3 or E5M2) with one E8M0 scale per 1 x 32 block along C, and
//      - dim1: X^T (C x R) in fp8 with one scale per 32 x 1 block along R,
//    i.e. the K-major operands of the forward GEMM and of the two backward GEMMs.  Scales
//    are rounded up to a power of two (RCEIL: 2^ceil(log2(amax / fp8_max))), so no value
//    overflows.
//  * mx_gemm: D = A . B^T on tcgen05 block-scaled MMAs (kind::mxf8f6f4, scale vector 1X:
//    one scale per 32 K elements), both operands K-major fp8, scale factors staged in
//    tensor memory, D bf16 / fp32 (store) or fp32 accumulate (reduce-add, wgrad).
//
// Scale-factor storage.  Scales of an (R x K) operand are kept as 512-byte atoms, one per
// (128-row block, 128-K block), in the order tcgen05.cp reads them: byte
// (r % 32) * 16 + ((r % 128) / 32) * 4 + (k / 32) % 4 of atom (r / 128, k / 128).  A
// 32x128b.warpx4 copy moves an atom into 4 TMEM columns (lanes replicated over the 4
// sub-partitions): column c, byte j holds the scale of row 32c + lane, K block j, which
// is the block-scaled MMA's operand layout; MMA j of the 4 in a 128-K block selects byte j
// through the scale-factor id.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.h"

namespace mykb {
namespace mx {

typedef __nv_bfloat16 bf16;

// E8M0 of 2^ceil(log2(v)) (round toward +inf, saturating), v >= 0.
__device__ __forceinline__ uint32_t e8m0_ceil(float v) {
  uint16_t d;
  asm("cvt.rp.satfinite.ue8m0x2.f32 %0, %1, %2;" : "=h"(d) : "f"(v), "f"(v));
  return d & 0xFF;
}
// 2^(127 - e): the reciprocal of the scale 2^(e - 127) (e in [0, 253]).
__device__ __forceinline__ float inv_scale(uint32_t e) { return __uint_as_float((254u - min(e, 253u)) << 23); }

// two floats -> two fp8 (x0 in the low byte)
template <bool E5M2>
__device__ __forceinline__ uint16_t to_fp8x2(float x0, float x1) {
  uint16_t d;
  if (E5M2) asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(d) : "f"(x1), "f"(x0));
  else asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(x1), "f"(x0));
  return d;
}

__device__ __forceinline__ int64_t sf_offset(int64_t r, int64_t k, int64_t katoms) {
  return ((r >> 7) * katoms + (k >> 7)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + ((k >> 5) & 3);
}

constexpr int QT_ROWS = 32, QT_COLS = 128, QT_THREADS = 128;

// One CTA per (32-row, 128-col) tile.  dim0: thread t quantizes row t/4, columns
// 32 (t % 4) .. +31; dim1: thread t quantizes column t over the 32 rows.
template <bool E5M2>
__global__ void __launch_bounds__(QT_THREADS) mx_quantize_kernel(const bf16* __restrict__ x, int R, int C, int64_t ldx,
                                                                uint8_t* __restrict__ q0, uint8_t* __restrict__ s0,
                                                                uint8_t* __restrict__ q1, uint8_t* __restrict__ s1,
                                                                int64_t ldq1) {
  __shared__ __align__(16) bf16 tile[QT_ROWS][QT_COLS + 8];
  const float fmax = E5M2 ? 57344.f : 448.f;
  const int r0 = blockIdx.y * QT_ROWS, c0 = blockIdx.x * QT_COLS;
  const int t = threadIdx.x;
  for (int i = t; i < QT_ROWS * QT_COLS / 8; i += QT_THREADS) {
    const int r = i / (QT_COLS / 8), c = (i % (QT_COLS / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r0 + r < R && c0 + c < C) v = *reinterpret_cast<const uint4*>(x + (int64_t)(r0 + r) * ldx + c0 + c);
    *reinterpret_cast<uint4*>(&tile[r][c]) = v;
  }
  __syncthreads();
  if (q0 != nullptr) {
    const int r = t >> 2, cb = (t & 3) * 32;
    float v[32], amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      v[i] = __bfloat162float(tile[r][cb + i]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
    const uint32_t e = e8m0_ceil(amax / fmax);
    const float inv = inv_scale(e);
    if (r0 + r < R && c0 + cb < C) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        w[i] = (uint32_t)to_fp8x2<E5M2>(v[4 * i] * inv, v[4 * i + 1] * inv) |
               ((uint32_t)to_fp8x2<E5M2>(v[4 * i + 2] * inv, v[4 * i + 3] * inv) << 16);
      uint4* dst = reinterpret_cast<uint4*>(q0 + (int64_t)(r0 + r) * C + c0 + cb);
      dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
      dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
      s0[sf_offset(r0 + r, c0 + cb, C / 128)] = (uint8_t)e;
    }
  }
  if (q1 != nullptr) {
    const int c = t;
    float v[32], amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      v[i] = __bfloat162float(tile[i][c]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
    const uint32_t e = e8m0_ceil(amax / fmax);
    const float inv = inv_scale(e);
    if (c0 + c < C) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        w[i] = (uint32_t)to_fp8x2<E5M2>(v[4 * i] * inv, v[4 * i + 1] * inv) |
               ((uint32_t)to_fp8x2<E5M2>(v[4 * i + 2] * inv, v[4 * i + 3] * inv) << 16);
      uint4* dst = reinterpret_cast<uint4*>(q1 + (int64_t)(c0 + c) * ldq1 + r0);
      dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
      dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
      s1[sf_offset(c0 + c, r0, ldq1 / 128)] = (uint8_t)e;
    }
  }
}

}  // namespace mx

// ------------------------------------------------------------------------------ GEMM
namespace mx {

constexpr int BM = 128, BN = 128, BK = 128;  // BK in fp8 elements (= bytes): one 128-byte swizzle row
constexpr int STAGES = 6;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, SF_BYTES = 512;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + 2 * SF_BYTES;
constexpr int STAGING_BYTES = 32 * 128;
constexpr int BAR_OFFSET = STAGES * STAGE_BYTES + EPI_WARPS * STAGING_BYTES;
constexpr int SMEM_TOTAL = BAR_OFFSET + 256 + 1024;
constexpr int TMEM_COLS = 512;   // accumulators [0, 256), scale factors from column 256
constexpr int SF_COL0 = 2 * BN;  // per stage: 4 columns of A scales, then 4 of B scales

struct GemmArgs {
  const uint8_t* sfa;  // atoms of A: [ceil(M/128)][K/128][512]
  const uint8_t* sfb;
  int M, N, K;
  int tiles_m, tiles_n, k_blocks, total_tiles;
  int* status;
  // optional dequantisation of per-tensor / per-row float8 operands, applied in the
  // epilogue: D[m, n] = acc[m, n] * row_scale[m or 0] * col_scale[n or 0]
  const float* row_scale;
  const float* col_scale;
  int row_scale_n, col_scale_n;  // 1 (scalar) or M / N
};

// block-scaled instruction descriptor (kind::mxf8f6f4, scale vector 1X, E8M0 scales)
__host__ __device__ constexpr uint32_t make_idesc_mx(int m, int n, bool a_e5m2, bool b_e5m2, uint32_t sf_id) {
  return (sf_id << 4)                      // B scale-factor id (byte in the TMEM word)
         | ((a_e5m2 ? 1u : 0u) << 7)       // A format: 0 E4M3, 1 E5M2
         | ((b_e5m2 ? 1u : 0u) << 10)      // B format
         | ((uint32_t)(n >> 3) << 17)      // N / 8
         | (1u << 23)                      // scale format E8M0
         | ((uint32_t)(m >> 4) << 24)      // M / 16
         | (sf_id << 29);                  // A scale-factor id
}

// no-swizzle K-major descriptor of a 32-row x 16-byte scale atom (8-row groups 128 B apart)
__device__ __forceinline__ uint64_t make_sf_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)(128 >> 4) << 32;  // SBO
  d |= (uint64_t)1 << 46;           // descriptor version
  return d;                          // layout type 0: no swizzle
}

__device__ __forceinline__ void sf_copy(uint32_t taddr, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
}

__device__ __forceinline__ void umma_mx(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(smem_dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tile_coords(const GemmArgs& p, int tile, int& mt, int& nt) {
  constexpr int G = 8;
  const int span = G * p.tiles_n;
  const int group = tile / span, first = group * G, gsize = min(p.tiles_m - first, G), in = tile % span;
  mt = first + in % gsize;
  nt = in / gsize;
}

template <bool A_E5M2, bool B_E5M2, bool OUT_F32, bool ACCUM>
__global__ void __launch_bounds__(THREADS, 1)
mx_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmD, const GemmArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFFSET);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int katoms = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], EPI_WARPS);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmD);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- producer (TMA + bulk)
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
        int mt, nt;
        tile_coords(p, tile, mt, nt);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, __LINE__)) { ok = false; break; }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          uint8_t* ssf = sb + B_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_3d(sa, &tmA, &full[stage], kb * BK, mt * BM, 0);
          tma_load_3d(sb, &tmB, &full[stage], kb * BK, nt * BN, 0);
          bulk_load(ssf, p.sfa + ((int64_t)mt * katoms + kb) * SF_BYTES, SF_BYTES, &full[stage]);
          bulk_load(ssf + SF_BYTES, p.sfb + ((int64_t)nt * katoms + kb) * SF_BYTES, SF_BYTES, &full[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        if (!mbar_wait(&acc_empty[buf], ((local >> 1) & 1) ^ 1, p.status, __LINE__)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, __LINE__)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
          const uint32_t sf_addr = b_addr + B_BYTES;
          const uint32_t sfa_t = tmem_base + SF_COL0 + stage * 8;
          const uint32_t sfb_t = sfa_t + 4;
          sf_copy(sfa_t, make_sf_desc(sf_addr));
          sf_copy(sfb_t, make_sf_desc(sf_addr + SF_BYTES));
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint64_t da = make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t db = make_sw128_desc(b_addr + kk * 32, 16, 1024);
            umma_mx(d_tmem, da, db, make_idesc_mx(BM, BN, A_E5M2, B_E5M2, kk), sfa_t | ((uint32_t)kk << 30),
                    sfb_t | ((uint32_t)kk << 30), (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int q = warp & 3;
    uint8_t* stage_buf = staging + (warp - 2) * STAGING_BYTES;
    const uint32_t stage_addr = smem_u32(stage_buf);
    int local = 0;
    for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++local) {
      int mt, nt;
      tile_coords(p, tile, mt, nt);
      const int buf = local & 1;
      if (!mbar_wait_warp(&acc_full[buf], (local >> 1) & 1, p.status, __LINE__)) break;
      tc_fence_after();
      constexpr int kSlab = OUT_F32 ? 32 : 64;
#pragma unroll 1
      for (int s = 0; s < BN / kSlab; ++s) {
        float v[kSlab];
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN + s * kSlab;
        tmem_ld32(taddr, *reinterpret_cast<float(*)[32]>(&v[0]));
        if constexpr (!OUT_F32) tmem_ld32(taddr + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
        if (p.row_scale != nullptr) {
          const int row = mt * BM + q * 32 + lane;
          const float rs = p.row_scale[p.row_scale_n == 1 ? 0 : min(row, p.M - 1)];
          const int c0 = nt * BN + s * kSlab;
#pragma unroll
          for (int i = 0; i < kSlab; ++i)
            v[i] *= rs * p.col_scale[p.col_scale_n == 1 ? 0 : min(c0 + i, p.N - 1)];
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t w0, w1, w2, w3;
          if (OUT_F32) {
            w0 = __float_as_uint(v[4 * j + 0]);
            w1 = __float_as_uint(v[4 * j + 1]);
            w2 = __float_as_uint(v[4 * j + 2]);
            w3 = __float_as_uint(v[4 * j + 3]);
          } else {
            w0 = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            w1 = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            w2 = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            w3 = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
          }
          const uint32_t addr = stage_addr + lane * 128 + ((j ^ (lane & 7)) * 16);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int x = nt * BN + s * kSlab, y = mt * BM + q * 32, z = 0;
          if (ACCUM) {
            asm volatile(
                "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];"
                ::"l"(reinterpret_cast<uint64_t>(&tmD)), "r"(stage_addr), "r"(x), "r"(y), "r"(z)
                : "memory");
          } else {
            asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                         ::"l"(reinterpret_cast<uint64_t>(&tmD)), "r"(stage_addr), "r"(x), "r"(y), "r"(z)
                         : "memory");
          }
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace mx

// ------------------------------------------------------------------------------ host
static int mx_sms(int dev) {
  static int cached[64] = {0};
  if (!cached[dev]) cudaDeviceGetAttribute(&cached[dev], cudaDevAttrMultiProcessorCount, dev);
  return cached[dev];
}

// x (R, C) bf16, C % 128 == 0.  Returns [q0, s0] (dim0) and/or [q1, s1] (dim1; needs
// R % 128 == 0): q0 (R, C) uint8 fp8 bits, s0 (ceil(R/128) * C/128 * 512) uint8 atoms;
// q1 (C, R), s1 (ceil(C/128) * R/128 * 512).
std::vector<torch::Tensor> mx_quantize(torch::Tensor x, bool e5m2, bool dim0, bool dim1) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.scalar_type() == at::kBFloat16 && x.stride(1) == 1,
              "mx_quantize: 2-D bf16 CUDA matrix with contiguous rows");
  const int R = x.size(0), C = x.size(1);
  TORCH_CHECK(C % 128 == 0 && x.stride(0) % 8 == 0 && ((uintptr_t)x.data_ptr() % 16) == 0,
              "mx_quantize: columns must be a multiple of 128 and rows 16-byte aligned");
  TORCH_CHECK(!dim1 || R % 128 == 0, "mx_quantize: dim1 needs rows a multiple of 128");
  c10::cuda::CUDAGuard guard(x.device());
  auto u8 = x.options().dtype(at::kByte);
  torch::Tensor q0, s0, q1, s1;
  if (dim0) {
    q0 = torch::empty({R, C}, u8);
    const int64_t n = (int64_t)((R + 127) / 128) * (C / 128) * 512;
    s0 = (R % 128) ? torch::zeros({n}, u8) : torch::empty({n}, u8);  // padded rows keep scale byte 0
  }
  if (dim1) {
    q1 = torch::empty({C, R}, u8);
    s1 = torch::empty({(int64_t)(C / 128) * (R / 128) * 512}, u8);
  }
  if (R > 0) {
    dim3 grid(C / mx::QT_COLS, (R + mx::QT_ROWS - 1) / mx::QT_ROWS);
    auto st = at::cuda::getCurrentCUDAStream();
    auto p = [](torch::Tensor& t) { return t.defined() ? t.data_ptr<uint8_t>() : nullptr; };
    if (e5m2)
      mx::mx_quantize_kernel<true><<<grid, mx::QT_THREADS, 0, st>>>(
          (const mx::bf16*)x.data_ptr(), R, C, x.stride(0), p(q0), p(s0), p(q1), p(s1), R);
    else
      mx::mx_quantize_kernel<false><<<grid, mx::QT_THREADS, 0, st>>>(
          (const mx::bf16*)x.data_ptr(), R, C, x.stride(0), p(q0), p(s0), p(q1), p(s1), R);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  std::vector<torch::Tensor> out;
  if (dim0) out.insert(out.end(), {q0, s0});
  if (dim1) out.insert(out.end(), {q1, s1});
  return out;
}

// mx_quantize into caller-given buffers (both copies): q0 (R, C) and q1 (C, R) uint8,
// s0 / s1 their scale atoms.  Used for the row shards of fp8-gathered weights, whose
// quantized copies live in symmetric memory that peers read.
void mx_quantize_into(torch::Tensor x, bool e5m2, torch::Tensor q0, torch::Tensor s0, torch::Tensor q1,
                      torch::Tensor s1) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.scalar_type() == at::kBFloat16 && x.is_contiguous(),
              "mx_quantize_into: contiguous 2-D bf16 CUDA matrix");
  const int R = x.size(0), C = x.size(1);
  TORCH_CHECK(C % 128 == 0 && R % 128 == 0, "mx_quantize_into: rows and columns must be multiples of 128");
  for (const auto& t : {q0, s0, q1, s1})
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kByte && t.is_contiguous() &&
                    ((uintptr_t)t.data_ptr() % 16) == 0,
                "mx_quantize_into: 16-byte aligned contiguous uint8 outputs");
  TORCH_CHECK(q0.numel() == (int64_t)R * C && q1.numel() == (int64_t)R * C &&
                  s0.numel() == (int64_t)R * C / 32 && s1.numel() == (int64_t)R * C / 32,
              "mx_quantize_into: output sizes");
  c10::cuda::CUDAGuard guard(x.device());
  if (R == 0) return;
  dim3 grid(C / mx::QT_COLS, (R + mx::QT_ROWS - 1) / mx::QT_ROWS);
  auto st = at::cuda::getCurrentCUDAStream();
  if (e5m2)
    mx::mx_quantize_kernel<true><<<grid, mx::QT_THREADS, 0, st>>>((const mx::bf16*)x.data_ptr(), R, C, C,
                                                                   q0.data_ptr<uint8_t>(), s0.data_ptr<uint8_t>(),
                                                                   q1.data_ptr<uint8_t>(), s1.data_ptr<uint8_t>(), R);
  else
    mx::mx_quantize_kernel<false><<<grid, mx::QT_THREADS, 0, st>>>((const mx::bf16*)x.data_ptr(), R, C, C,
                                                                    q0.data_ptr<uint8_t>(), s0.data_ptr<uint8_t>(),
                                                                    q1.data_ptr<uint8_t>(), s1.data_ptr<uint8_t>(), R);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <bool AE, bool BE, bool F32, bool ACC>
static void mx_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const mx::GemmArgs& p,
                      int grid, cudaStream_t st) {
  auto kern = mx::mx_gemm_kernel<AE, BE, F32, ACC>;
  static SmemOptIn configured;
  C10_CUDA_CHECK(configured.ensure(kern, mx::SMEM_TOTAL));
  kern<<<grid, mx::THREADS, mx::SMEM_TOTAL, st>>>(ta, tb, td, p);
}

// d (M, N) = a (M, K) . b (N, K)^T: a, b fp8 bits (uint8) with scale atoms sa, sb from
// mx_quantize; d bf16 or fp32; accumulate adds into fp32 d.  row_scale / col_scale
// (optional fp32, 1 or M / N entries) multiply the product in the epilogue.
static void mx_gemm_impl(torch::Tensor a, torch::Tensor sa, bool a_e5m2, torch::Tensor b, torch::Tensor sb,
                         bool b_e5m2, torch::Tensor d, bool accumulate, const torch::Tensor* row_scale,
                         const torch::Tensor* col_scale);

void mx_gemm(torch::Tensor a, torch::Tensor sa, bool a_e5m2, torch::Tensor b, torch::Tensor sb, bool b_e5m2,
             torch::Tensor d, bool accumulate) {
  mx_gemm_impl(a, sa, a_e5m2, b, sb, b_e5m2, d, accumulate, nullptr, nullptr);
}

// Per-tensor / per-row scaled float8 GEMM (the float8 training recipes' matmul):
// d = (a * row_scale) . (b * col_scale)^T with a (M, K), b (N, K) fp8 bits, K a multiple
// of 128.  The tensor cores run the block-scaled instruction with every block scale 2^0
// (unit atoms, built once per shape by the caller) and the epilogue applies the scales.
void fp8_scaled_gemm(torch::Tensor a, torch::Tensor unit_sa, bool a_e5m2, torch::Tensor b, torch::Tensor unit_sb,
                     bool b_e5m2, torch::Tensor row_scale, torch::Tensor col_scale, torch::Tensor d) {
  TORCH_CHECK(row_scale.scalar_type() == at::kFloat && col_scale.scalar_type() == at::kFloat &&
                  row_scale.is_contiguous() && col_scale.is_contiguous() && row_scale.is_cuda() && col_scale.is_cuda(),
              "fp8_scaled_gemm: fp32 CUDA scales");
  TORCH_CHECK(row_scale.numel() == 1 || row_scale.numel() == a.size(0), "fp8_scaled_gemm: row scale 1 or M");
  TORCH_CHECK(col_scale.numel() == 1 || col_scale.numel() == b.size(0), "fp8_scaled_gemm: column scale 1 or N");
  mx_gemm_impl(a, unit_sa, a_e5m2, b, unit_sb, b_e5m2, d, false, &row_scale, &col_scale);
}

static void mx_gemm_impl(torch::Tensor a, torch::Tensor sa, bool a_e5m2, torch::Tensor b, torch::Tensor sb,
                         bool b_e5m2, torch::Tensor d, bool accumulate, const torch::Tensor* row_scale,
                         const torch::Tensor* col_scale) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && d.is_cuda() && a.dim() == 2 && b.dim() == 2 && d.dim() == 2,
              "mx_gemm: 2-D CUDA tensors");
  TORCH_CHECK(a.scalar_type() == at::kByte && b.scalar_type() == at::kByte, "mx_gemm: uint8 fp8 operands");
  const int M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(b.size(1) == K && K % 128 == 0 && K > 0, "mx_gemm: K must match and be a multiple of 128");
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && d.stride(1) == 1 && d.size(0) == M && d.size(1) == N,
              "mx_gemm: contiguous operands, D (M, N)");
  TORCH_CHECK(sa.numel() >= (int64_t)((M + 127) / 128) * (K / 128) * 512 &&
                  sb.numel() >= (int64_t)((N + 127) / 128) * (K / 128) * 512,
              "mx_gemm: scale atoms do not cover the operands");
  const bool f32 = d.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || d.scalar_type() == at::kBFloat16, "mx_gemm: D bf16 or fp32");
  TORCH_CHECK(!accumulate || f32, "mx_gemm: accumulate needs fp32 D");
  c10::cuda::CUDAGuard guard(a.device());
  mx::GemmArgs p{};
  p.sfa = sa.data_ptr<uint8_t>();
  p.sfb = sb.data_ptr<uint8_t>();
  p.M = M, p.N = N, p.K = K;
  p.tiles_m = (M + mx::BM - 1) / mx::BM;
  p.tiles_n = (N + mx::BN - 1) / mx::BN;
  p.k_blocks = K / mx::BK;
  p.total_tiles = p.tiles_m * p.tiles_n;
  p.status = device_status();
  if (row_scale != nullptr) {
    p.row_scale = row_scale->data_ptr<float>();
    p.col_scale = col_scale->data_ptr<float>();
    p.row_scale_n = (int)row_scale->numel();
    p.col_scale_n = (int)col_scale->numel();
  }
  if (p.total_tiles == 0) return;
  CUtensorMap ta = make_tmap_3d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, 1, K, 0, mx::BK, mx::BM);
  CUtensorMap tb = make_tmap_3d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, 1, K, 0, mx::BK, mx::BN);
  CUtensorMap td = f32 ? make_tmap_3d(d.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, 1, d.stride(0), 0, 32, 32)
                       : make_tmap_3d(d.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 1, d.stride(0), 0, 64, 32);
  const int grid = std::min(p.total_tiles, mx_sms(a.get_device()));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int key = (a_e5m2 ? 8 : 0) | (b_e5m2 ? 4 : 0) | (f32 ? 2 : 0) | (accumulate ? 1 : 0);
  switch (key) {
    case 0: mx_launch<false, false, false, false>(ta, tb, td, p, grid, st); break;
    case 2: mx_launch<false, false, true, false>(ta, tb, td, p, grid, st); break;
    case 3: mx_launch<false, false, true, true>(ta, tb, td, p, grid, st); break;
    case 8: mx_launch<true, false, false, false>(ta, tb, td, p, grid, st); break;
    case 10: mx_launch<true, false, true, false>(ta, tb, td, p, grid, st); break;
    case 11: mx_launch<true, false, true, true>(ta, tb, td, p, grid, st); break;
    case 12: mx_launch<true, true, false, false>(ta, tb, td, p, grid, st); break;
    case 14: mx_launch<true, true, true, false>(ta, tb, td, p, grid, st); break;
    case 15: mx_launch<true, true, true, true>(ta, tb, td, p, grid, st); break;
    default: TORCH_CHECK(false, "mx_gemm: an E4M3 A with an E5M2 B is not instantiated");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
