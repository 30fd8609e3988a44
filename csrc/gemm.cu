// Persistent, warp-specialised bf16 GEMM on tcgen05 (sm_100a).
//
//   D[b, m, n] = alpha * sum_k A[b, m, k] * B[b, n, k] + beta * C[b, m, n]     (store mode)
//   D[b, m, n] += alpha * sum_k A[b, m, k] * B[b, n, k]                        (accumulate mode)
//
// Operands are bf16, each either K-major (reduction dim contiguous) or MN-major (output
// dim contiguous); D is bf16 or fp32.  Layout per CTA (one CTA per SM, persistent over
// output tiles in a grouped raster order for L2 reuse):
//
//   warp 0      TMA producer: streams 128x64 A and BNx64 B tiles (128-byte swizzle) into a
//               STAGES-deep shared-memory ring, one mbarrier pair per stage.
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma (M=128, N=BN, K=16) into
//               one of two tensor-memory accumulators, commits each stage back to the
//               producer and each finished tile to the epilogue.
//   warps 2-5   epilogue: tcgen05.ld the accumulator (each warp owns 32 TMEM lanes = 32 rows),
//               scale / add C, convert, write a 128-byte-swizzled staging tile and issue a
//               TMA store (or a TMA reduce-add into fp32 D in accumulate mode, which also
//               carries split-K partial sums).
//
// Two accumulators let the epilogue of tile i overlap the main loop of tile i+1.  Every TMA
// load is a plain per-CTA copy: this kernel may read operands that other ranks wrote into this GPU's
// memory, never another GPU's memory.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.h"

namespace mykb {

// All-gather fused into the GEMM (parameter-sharded data parallelism): the B operand is a
// weight whose rows are spread over `world` GPUs (rank r holds rows [r*R, (r+1)*R) in its
// shard buffer, at the same element offset on every rank).  Extra "gather" warps of every
// CTA copy 64-row chunks of it from the owners' memory (16-byte peer loads over NVLink,
// local loads for this rank's own rows) into a local full-size copy `dst`, which the TMA
// producer then reads; a chunk counter per 64 rows (release add by the gather warp,
// acquire load by the producer, proxy fences on both sides for the TMA read) orders them.
// The copy starts at this rank's own chunks and the tile order (forward: output columns;
// data gradient: the reduction loop) starts there too, so the first tiles run on rows that
// are local while the remote rows cross NVLink.
struct GatherParams {
  const int64_t* src_ptrs;  // [world] base addresses (bf16) of every rank's shard buffer
  int64_t src_offset;       // element offset of this weight's shard in each buffer (multiple of 8)
  int rows_per_rank;        // R
  int rows, cols;           // gathered weight: rows x cols, row-major (cols multiple of 8)
  __nv_bfloat16* dst;       // local full-size copy
  uint32_t* ready;          // [chunks] counters, one per 64 rows of dst
  uint32_t target;          // counter value once this call has copied the whole chunk
  int pieces_per_chunk, rows_per_piece;
  int first_chunk, chunks;
  int wait_b;  // 1: dst is this GEMM's B operand (the producer waits per chunk); 0: prefetch of a later GEMM's weight
};

constexpr int kGatherWarps = 4;
constexpr int kGatherUnroll = 8;

struct GemmParams {
  int M, N, K, batch;
  int tiles_m, tiles_n, k_blocks, split_k, kb_per_split;
  int total_units;
  const void* C;  // optional epilogue input, same layout/dtype as D
  int64_t ldc, c_batch_stride;
  float alpha, beta;
  int symmetric;  // D = D^T (M == N): tiles strictly above the diagonal are skipped, then mirrored
  int* status;
  int rot_n;      // gather mode, B K-major: output column tiles start at this one
  int rot_k;      // gather mode, B MN-major: the reduction loop starts at this K block
  GatherParams g;
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGroupM = 8;
constexpr int kEpiWarps = 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;

// A tile of a symmetric product whose every element lies above the diagonal (column > row).
__device__ __forceinline__ bool skip_tile(const GemmParams& p, int mt, int nt, int bn) {
  return p.symmetric && nt * bn >= (mt + 1) * kBM;
}

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagingBytes = 32 * 128;  // one epilogue slab: 32 rows x 128 B
  // two staging slabs per epilogue warp, so a slab's TMA store overlaps the next slab
  static constexpr int kBarOffset = STAGES * kStageBytes + kEpiWarps * 2 * kStagingBytes;
  static constexpr int kTotal = kBarOffset + 256 + 1024;  // barriers + alignment slack
};

__device__ __forceinline__ void unit_coords(const GemmParams& p, int unit, int& b, int& mt, int& nt, int& split) {
  int tiles = p.tiles_m * p.tiles_n;
  int tile = unit % tiles;
  int rest = unit / tiles;
  split = rest % p.split_k;
  b = rest / p.split_k;
  int group_span = kGroupM * p.tiles_n;
  int group = tile / group_span;
  int first_m = group * kGroupM;
  int gsize = min(p.tiles_m - first_m, kGroupM);
  int in_group = tile % group_span;
  mt = first_m + in_group % gsize;
  nt = in_group / gsize;
  if (p.rot_n) nt = (nt + p.rot_n) % p.tiles_n;
}

__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Gather warps: copy pieces (rows_per_piece whole rows) of the sharded weight into dst,
// chunk by chunk starting at this rank's first chunk, and count each finished piece on its
// chunk's counter.  gw / n_gw: this warp's index among all gather warps of the grid.
__device__ __forceinline__ void gather_rows(const GatherParams& g, int gw, int n_gw, int lane) {
  const int vpr = g.cols / 8;  // 16-byte vectors per row
  const int total = g.chunks * g.pieces_per_chunk;
  uint4* dst = reinterpret_cast<uint4*>(g.dst);
  for (int pi = gw; pi < total; pi += n_gw) {
    const int chunk = (g.first_chunk + pi / g.pieces_per_chunk) % g.chunks;
    const int row0 = chunk * 64 + (pi % g.pieces_per_chunk) * g.rows_per_piece;
    const int row1 = min(row0 + g.rows_per_piece, g.rows);
    const int nvec = max(0, row1 - row0) * vpr;
    for (int base = 0; base < nvec; base += 32 * kGatherUnroll) {
      uint4 v[kGatherUnroll];
      int64_t at[kGatherUnroll];
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u) {
        const int i = base + u * 32 + lane;
        at[u] = -1;
        if (i < nvec) {
          const int row = row0 + i / vpr, c = i % vpr;
          const int r = row / g.rows_per_rank, lr = row - r * g.rows_per_rank;
          const uint4* src = reinterpret_cast<const uint4*>(g.src_ptrs[r]) + (g.src_offset + (int64_t)lr * g.cols) / 8;
          v[u] = src[c];
          at[u] = (int64_t)row * vpr + c;
        }
      }
#pragma unroll
      for (int u = 0; u < kGatherUnroll; ++u)
        if (at[u] >= 0) dst[at[u]] = v[u];
    }
    // the copied rows are read next by TMA (the async proxy) in other CTAs
    fence_proxy_async_global();
    __syncwarp();
    if (lane == 0) {
      __threadfence();
      red_release_add(g.ready + chunk, 1u);
    }
  }
}

// Producer side: wait (bounded) until every chunk of rows [r0, r1) is complete in this call.
// `seen` caches chunks already found complete (the first 256).
__device__ __forceinline__ bool wait_rows_ready(const GatherParams& g, int r0, int r1, uint32_t* seen, int* status,
                                                int code) {
  const int c0 = r0 / 64, c1 = min(g.chunks, (r1 + 63) / 64);
  bool waited = false;
  for (int c = c0; c < c1; ++c) {
    if (c < 256 && (seen[c >> 5] >> (c & 31) & 1u)) continue;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_gpu(g.ready + c) - g.target) < 0) {
      if (status_failed(status)) return false;
      if (globaltimer_ns() - t0 > kWaitNs) {
        set_status(status, code);
        return false;
      }
    }
    if (c < 256) seen[c >> 5] |= 1u << (c & 31);
    waited = true;
  }
  if (waited) fence_proxy_async_global();
  return true;
}

template <bool GATHER>
constexpr int gemm_threads() {
  return kThreads + (GATHER ? 32 * kGatherWarps : 0);
}

template <int BN, int STAGES, bool A_MN, bool B_MN, bool OUT_F32, bool ACCUM, bool GATHER>
__global__ void __launch_bounds__(gemm_threads<GATHER>(), 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmD, const GemmParams p) {
  using S = GemmSmem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * S::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
  uint64_t* full = bars;                  // [STAGES]
  uint64_t* empty = bars + STAGES;        // [STAGES]
  uint64_t* acc_full = bars + 2 * STAGES; // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmD);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t seen[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += gridDim.x) {
        int b, mt, nt, split;
        unit_coords(p, unit, b, mt, nt, split);
        if (skip_tile(p, mt, nt, BN)) continue;
        int kb0 = split * p.kb_per_split;
        int kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
        if (GATHER && !B_MN && p.g.wait_b && !wait_rows_ready(p.g, nt * BN, nt * BN + BN, seen, p.status, __LINE__)) {
          ok = false;
          break;
        }
        const int nkb = kb1 - kb0;
        for (int it = 0; it < nkb; ++it) {
          const int kb = GATHER ? kb0 + (it + p.rot_k) % nkb : kb0 + it;
          if (GATHER && B_MN && p.g.wait_b && !wait_rows_ready(p.g, kb * kBK, kb * kBK + kBK, seen, p.status, __LINE__)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, __LINE__)) { ok = false; break; }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          const int k0 = kb * kBK;
          if (A_MN) {
            tma_load_3d(sa, &tmA, &full[stage], mt * kBM, k0, b);
            tma_load_3d(sa + 8192, &tmA, &full[stage], mt * kBM + 64, k0, b);
          } else {
            tma_load_3d(sa, &tmA, &full[stage], k0, mt * kBM, b);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_3d(sb + j * 8192, &tmB, &full[stage], nt * BN + j * 64, k0, b);
          } else {
            tma_load_3d(sb, &tmB, &full[stage], k0, nt * BN, b);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, A_MN, B_MN);
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += gridDim.x) {
        int b, mt, nt, split;
        unit_coords(p, unit, b, mt, nt, split);
        if (skip_tile(p, mt, nt, BN)) continue;
        int kb0 = split * p.kb_per_split;
        int kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
        const int buf = local & 1;
        if (!mbar_wait(&acc_empty[buf], ((local >> 1) & 1) ^ 1, p.status, __LINE__)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = kb0; kb < kb1; ++kb) {  // only the count matters here: the producer orders the K blocks
          if (!mbar_wait(&full[stage], phase, p.status, __LINE__)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t b_addr = a_addr + S::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            uint64_t da = A_MN ? make_sw128_desc(a_addr + kk * 2048, 8192, 1024)
                               : make_sw128_desc(a_addr + kk * 32, 16, 1024);
            uint64_t db = B_MN ? make_sw128_desc(b_addr + kk * 2048, 8192, 1024)
                               : make_sw128_desc(b_addr + kk * 32, 16, 1024);
            umma_bf16_ss(d_tmem, da, db, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
        ++local;
      }
    }
  } else if (GATHER && warp >= 2 + kEpiWarps) {
    // ---------------------------------------------------------------- gather warps
    gather_rows(p.g, blockIdx.x * kGatherWarps + (warp - 2 - kEpiWarps), gridDim.x * kGatherWarps, lane);
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t stage_base = smem_u32(staging + (warp - 2) * 2 * S::kStagingBytes);
    int local = 0, slab_ct = 0;
    for (int unit = blockIdx.x; unit < p.total_units; unit += gridDim.x) {
      int b, mt, nt, split;
      unit_coords(p, unit, b, mt, nt, split);
      if (skip_tile(p, mt, nt, BN)) continue;
      const int buf = local & 1;
      if (!mbar_wait_warp(&acc_full[buf], (local >> 1) & 1, p.status, __LINE__)) break;
      tc_fence_after();
      const int row = mt * kBM + q * 32 + lane;
      const int col0 = nt * BN;
      // Each slab is 128 bytes of output columns: 64 bf16 or 32 fp32.
      constexpr int kSlab = OUT_F32 ? 32 : 64;
#pragma unroll 1
      for (int s = 0; s < BN / kSlab; ++s, ++slab_ct) {
        const uint32_t stage_addr = stage_base + (slab_ct & 1) * S::kStagingBytes;
        float v[kSlab];
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN + s * kSlab;
        tmem_ld32_raw(taddr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        if constexpr (!OUT_F32) tmem_ld32_raw(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
        const bool add_c = !ACCUM && p.C != nullptr && p.beta != 0.f;
#pragma unroll
        for (int i = 0; i < kSlab; ++i) v[i] *= p.alpha;
        if (add_c && row < p.M) {
          const int cbase = col0 + s * kSlab;
          if (OUT_F32) {
            const float* c = reinterpret_cast<const float*>(p.C) + b * p.c_batch_stride + (int64_t)row * p.ldc;
            if (cbase + kSlab <= p.N) {  // whole slab in range: 16-byte loads (rows are 16-byte aligned)
#pragma unroll
              for (int i = 0; i < kSlab; i += 4) {
                const float4 cv = *reinterpret_cast<const float4*>(c + cbase + i);
                v[i] += p.beta * cv.x;
                v[i + 1] += p.beta * cv.y;
                v[i + 2] += p.beta * cv.z;
                v[i + 3] += p.beta * cv.w;
              }
            } else {
#pragma unroll
              for (int i = 0; i < kSlab; ++i)
                if (cbase + i < p.N) v[i] += p.beta * c[cbase + i];
            }
          } else {
            const __nv_bfloat16* c =
                reinterpret_cast<const __nv_bfloat16*>(p.C) + b * p.c_batch_stride + (int64_t)row * p.ldc;
            if (cbase + kSlab <= p.N) {
#pragma unroll
              for (int i = 0; i < kSlab; i += 8) {
                const uint4 u = *reinterpret_cast<const uint4*>(c + cbase + i);
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 f = __bfloat1622float2(h[j]);
                  v[i + 2 * j] += p.beta * f.x;
                  v[i + 2 * j + 1] += p.beta * f.y;
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < kSlab; ++i)
                if (cbase + i < p.N) v[i] += p.beta * __bfloat162float(c[cbase + i]);
            }
          }
        }
        // The TMA store issued from this staging buffer two slabs ago must have finished
        // reading it (at most one younger store may still be in flight).
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        __syncwarp();
        // Row `lane` of the staging tile: 8 chunks of 16 bytes, chunk j stored at j ^ (lane & 7)
        // (the 128-byte swizzle the store tensor map expects).
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
          const int x = col0 + s * kSlab;
          const int y = mt * kBM + q * 32;
          if (ACCUM) {
            asm volatile(
                "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];"
                ::"l"(reinterpret_cast<uint64_t>(&tmD)), "r"(stage_addr), "r"(x), "r"(y), "r"(b)
                : "memory");
          } else {
            asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                         ::"l"(reinterpret_cast<uint64_t>(&tmD)), "r"(stage_addr), "r"(x), "r"(y), "r"(b)
                         : "memory");
          }
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      // All TMEM reads of this accumulator are done: hand it back to the MMA warp.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      ++local;
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// -------------------------------------------------------------------------------------
// host side
// -------------------------------------------------------------------------------------
static int num_sms(int device) {
  static int cached[64] = {0};
  if (cached[device] == 0) {
    cudaDeviceGetAttribute(&cached[device], cudaDevAttrMultiProcessorCount, device);
  }
  return cached[device];
}

template <int BN, int STAGES, bool A_MN, bool B_MN, bool OUT_F32, bool ACCUM, bool GATHER>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const GemmParams& p,
                        int grid, cudaStream_t stream) {
  using S = GemmSmem<BN, STAGES>;
  auto kern = gemm_kernel<BN, STAGES, A_MN, B_MN, OUT_F32, ACCUM, GATHER>;
  static SmemOptIn configured;
  C10_CUDA_CHECK(configured.ensure(kern, S::kTotal));
  kern<<<grid, gemm_threads<GATHER>(), S::kTotal, stream>>>(ta, tb, td, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int BN, bool A_MN, bool B_MN, bool OUT_F32, bool ACCUM, bool GATHER = false>
static void dispatch_stages(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const GemmParams& p,
                            int grid, cudaStream_t stream) {
  // 4 stages for BN=256 (48 KB each), 6 for BN=128 (32 KB each).
  if constexpr (BN == 256) {
    launch_gemm<BN, 4, A_MN, B_MN, OUT_F32, ACCUM, GATHER>(ta, tb, td, p, grid, stream);
  } else {
    launch_gemm<BN, 6, A_MN, B_MN, OUT_F32, ACCUM, GATHER>(ta, tb, td, p, grid, stream);
  }
}

template <int BN>
static void dispatch_layout(bool a_mn, bool b_mn, bool out_f32, bool accum, const CUtensorMap& ta,
                            const CUtensorMap& tb, const CUtensorMap& td, const GemmParams& p, int grid,
                            cudaStream_t s) {
#define MYKB_GEMM_CASE(AM, BM)                                                       \
  if (a_mn == AM && b_mn == BM) {                                                    \
    if (accum) return dispatch_stages<BN, AM, BM, true, true>(ta, tb, td, p, grid, s); \
    if (out_f32) return dispatch_stages<BN, AM, BM, true, false>(ta, tb, td, p, grid, s); \
    return dispatch_stages<BN, AM, BM, false, false>(ta, tb, td, p, grid, s);          \
  }
  MYKB_GEMM_CASE(false, false)
  MYKB_GEMM_CASE(false, true)
  MYKB_GEMM_CASE(true, false)
  MYKB_GEMM_CASE(true, true)
#undef MYKB_GEMM_CASE
}

// Symmetric mode: copy the lower triangle onto the upper one (D[i][j] = D[j][i], j > i), which
// also fills the tiles the GEMM skipped.  A block moves one 64 x 64 tile: 16-byte vector loads
// of the source tile (below the diagonal) into shared memory, transposed 16-byte vector stores
// of the destination tile (above it).  Rows must be 16-byte aligned (checked by the caller).
template <typename T>
__global__ void __launch_bounds__(256) mirror_lower_kernel(T* __restrict__ d, int n, int64_t ld, int64_t bstride) {
  constexpr int V = 16 / sizeof(T);  // elements per vector
  __shared__ alignas(16) T tile[64][64 + V];
  const int bi = blockIdx.y, bj = blockIdx.x;  // destination tile: rows 64 bi.., cols 64 bj..
  if (bj < bi) return;
  T* m = d + (int64_t)blockIdx.z * bstride;
  constexpr int kVecRow = 64 / V;
  for (int v = threadIdx.x; v < 64 * kVecRow; v += blockDim.x) {  // source tile: rows 64 bj.., cols 64 bi..
    const int r = v / kVecRow, c = (v % kVecRow) * V;
    const int i = bj * 64 + r, j = bi * 64 + c;
    if (i < n && j + V <= n) {
      *reinterpret_cast<uint4*>(&tile[r][c]) = *reinterpret_cast<const uint4*>(m + (int64_t)i * ld + j);
    } else if (i < n) {
      for (int e = 0; e < V && j + e < n; ++e) tile[r][c + e] = m[(int64_t)i * ld + j + e];
    }
  }
  __syncthreads();
  for (int v = threadIdx.x; v < 64 * kVecRow; v += blockDim.x) {
    const int r = v / kVecRow, c = (v % kVecRow) * V;  // destination row 64 bi + r, cols 64 bj + c ..
    const int i = bi * 64 + r, j = bj * 64 + c;
    if (i >= n) continue;
    alignas(16) T out[V];
#pragma unroll
    for (int e = 0; e < V; ++e) out[e] = tile[c + e][r];
    if (j > i && j + V <= n) {
      *reinterpret_cast<uint4*>(m + (int64_t)i * ld + j) = *reinterpret_cast<const uint4*>(out);
    } else {
      for (int e = 0; e < V; ++e)
        if (j + e > i && j + e < n) m[(int64_t)i * ld + j + e] = out[e];
    }
  }
}

// a: (batch?, M, K) or (batch?, K, M); b: (batch?, N, K) or (batch?, K, N); d: (batch?, M, N)
// gather != nullptr: all-gather mode (2-D, A K-major, bf16 D, stored product); b is the local
// full-size copy the kernel fills from the shards while it multiplies.
static void run_gemm(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor& d, c10::optional<torch::Tensor> c,
                     bool a_mn, bool b_mn, double alpha, double beta, bool accumulate, bool symmetric,
                     const GatherParams* gather) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && d.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm: bf16 operands required");
  TORCH_CHECK(d.scalar_type() == at::kBFloat16 || d.scalar_type() == at::kFloat, "gemm: D must be bf16 or fp32");
  TORCH_CHECK(a.dim() == b.dim() && a.dim() == d.dim() && (a.dim() == 2 || a.dim() == 3), "gemm: rank mismatch");
  TORCH_CHECK(!accumulate || d.scalar_type() == at::kFloat, "gemm: accumulate needs fp32 D");
  const bool batched = a.dim() == 3;
  const int batch = batched ? a.size(0) : 1;
  const int M = a_mn ? a.size(-1) : a.size(-2);
  const int K = a_mn ? a.size(-2) : a.size(-1);
  const int N = b_mn ? b.size(-1) : b.size(-2);
  const int Kb = b_mn ? b.size(-2) : b.size(-1);
  TORCH_CHECK(K == Kb, "gemm: reduction sizes differ (", K, " vs ", Kb, ")");
  TORCH_CHECK(d.size(-2) == M && d.size(-1) == N, "gemm: D has the wrong shape");
  TORCH_CHECK(a.stride(-1) == 1 && b.stride(-1) == 1 && d.stride(-1) == 1, "gemm: inner dims must be contiguous");
  c10::cuda::CUDAGuard guard(a.device());
  const bool out_f32 = d.scalar_type() == at::kFloat;

  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = batch;
  const int BN = (N <= 128) ? 128 : 256;
  p.tiles_m = (M + kBM - 1) / kBM;
  p.tiles_n = (N + BN - 1) / BN;
  p.k_blocks = (K + kBK - 1) / kBK;
  const int sms = num_sms(a.get_device());
  int split = 1;
  const int tiles = batch * p.tiles_m * p.tiles_n;
  if (accumulate) {
    // Split K (partial sums meet in the fp32 reduce-add epilogue) when the tiles fill the
    // SMs' waves badly: the fewest splits whose waves are >= 95% full, else the best fill,
    // keeping >= 16 K blocks per split so the reduce epilogue stays amortised.
    auto fill = [&](int sp) {
      const int units = tiles * sp;
      return (double)units / ((double)((units + sms - 1) / sms) * sms);
    };
    double best = fill(1);
    for (int sp = 2; sp <= 16 && best < 0.95 && p.k_blocks / sp >= 16; ++sp) {
      const double f = fill(sp);
      if (f > best + 0.02) {
        best = f;
        split = sp;
      }
    }
  }
  p.kb_per_split = (p.k_blocks + split - 1) / split;
  p.split_k = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  p.total_units = tiles * p.split_k;
  p.alpha = (float)alpha;
  p.beta = (float)beta;
  p.C = nullptr;
  if (c.has_value() && c->defined() && beta != 0.0) {
    TORCH_CHECK(c->scalar_type() == d.scalar_type() && c->size(-1) == N && c->size(-2) == M && c->stride(-1) == 1,
                "gemm: C must match D");
    p.C = c->data_ptr();
    p.ldc = c->stride(-2);
    p.c_batch_stride = batched ? c->stride(0) : 0;
  }
  p.status = device_status();
  if (symmetric) {
    TORCH_CHECK(M == N && !accumulate && split == 1, "gemm: symmetric mode needs M == N and a stored product");
    p.symmetric = 1;
  }
  if (gather != nullptr) {
    const bool store_layout = !a_mn && !out_f32 && !accumulate;  // forward / data-gradient products
    const bool wgrad_layout = a_mn && b_mn && accumulate;        // weight-gradient products
    TORCH_CHECK(!batched && !symmetric && (store_layout || wgrad_layout),
                "gemm_gather: 2-D forward (A, B K-major), data-gradient (B MN-major) or weight-gradient layouts");
    TORCH_CHECK(!gather->wait_b || (store_layout && split == 1), "gemm_gather: B can be gathered only by a stored product");
    p.g = *gather;
    if (gather->wait_b) {  // start where this rank's own rows are
      if (b_mn) {
        p.rot_k = p.k_blocks > 0 ? gather->first_chunk % p.k_blocks : 0;  // a chunk is one 64-row K block
      } else {
        p.rot_n = p.tiles_n > 0 ? (gather->first_chunk * 64 / BN) % p.tiles_n : 0;
      }
    }
  }

  // Tensor maps (dims innermost first): A/B tiles of 64 elements (128 B) along the
  // contiguous dim; D boxes of 128 bytes x 32 rows.
  const int64_t a_bs = batched ? a.stride(0) : 0, b_bs = batched ? b.stride(0) : 0, d_bs = batched ? d.stride(0) : 0;
  CUtensorMap ta = a_mn ? make_tmap_3d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, batch, a.stride(-2),
                                       a_bs, 64, 64)
                        : make_tmap_3d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, batch, a.stride(-2),
                                       a_bs, 64, kBM);
  CUtensorMap tb = b_mn ? make_tmap_3d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, batch, b.stride(-2),
                                       b_bs, 64, 64)
                        : make_tmap_3d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, batch, b.stride(-2),
                                       b_bs, 64, BN);
  CUtensorMap td = out_f32 ? make_tmap_3d(d.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, batch,
                                          d.stride(-2), d_bs, 32, 32)
                           : make_tmap_3d(d.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, batch,
                                          d.stride(-2), d_bs, 64, 32);
  const int grid = std::min(p.total_units, sms);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (gather != nullptr) {
    if (BN == 128) {
      if (accumulate) dispatch_stages<128, true, true, true, true, true>(ta, tb, td, p, grid, stream);
      else if (b_mn) dispatch_stages<128, false, true, false, false, true>(ta, tb, td, p, grid, stream);
      else dispatch_stages<128, false, false, false, false, true>(ta, tb, td, p, grid, stream);
    } else {
      if (accumulate) dispatch_stages<256, true, true, true, true, true>(ta, tb, td, p, grid, stream);
      else if (b_mn) dispatch_stages<256, false, true, false, false, true>(ta, tb, td, p, grid, stream);
      else dispatch_stages<256, false, false, false, false, true>(ta, tb, td, p, grid, stream);
    }
    return;
  }
  if (BN == 128) {
    dispatch_layout<128>(a_mn, b_mn, out_f32, accumulate, ta, tb, td, p, grid, stream);
  } else {
    dispatch_layout<256>(a_mn, b_mn, out_f32, accumulate, ta, tb, td, p, grid, stream);
  }
  if (symmetric && M > 0) {
    const int tiles64 = (M + 63) / 64;
    dim3 mg(tiles64, tiles64, batch);
    if (out_f32)
      mirror_lower_kernel<float><<<mg, 256, 0, stream>>>(d.data_ptr<float>(), M, d.stride(-2), d_bs);
    else
      mirror_lower_kernel<__nv_bfloat16><<<mg, 256, 0, stream>>>((__nv_bfloat16*)d.data_ptr(), M, d.stride(-2), d_bs);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor d, c10::optional<torch::Tensor> c, bool a_mn, bool b_mn,
          double alpha, double beta, bool accumulate, bool symmetric) {
  run_gemm(a, b, d, c, a_mn, b_mn, alpha, beta, accumulate, symmetric, nullptr);
}

static GatherParams make_gather(const torch::Tensor& w, const torch::Tensor& src_ptrs, int64_t src_offset,
                                int64_t rows_per_rank, int64_t rank, const torch::Tensor& ready, int64_t epoch,
                                const char* who) {
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous() && w.scalar_type() == at::kBFloat16, who, ": gathered weight 2-D bf16");
  TORCH_CHECK(src_ptrs.scalar_type() == at::kLong && src_ptrs.is_cuda(), who, ": int64 CUDA src_ptrs");
  TORCH_CHECK(ready.scalar_type() == at::kInt && ready.is_cuda() && ready.is_contiguous(), who, ": ready counters");
  const int rows = w.size(0), cols = w.size(1);
  const int world = src_ptrs.numel();
  TORCH_CHECK(cols % 8 == 0 && src_offset % 8 == 0, who, ": rows and shards must be 16-byte aligned");
  TORCH_CHECK(rows_per_rank > 0 && rows_per_rank * world >= rows && rank >= 0 && rank < world, who,
              ": shards do not cover the weight");
  const int chunks = (rows + 63) / 64;
  TORCH_CHECK(ready.numel() >= chunks, who, ": ready needs one counter per 64 rows");
  GatherParams g{};
  g.src_ptrs = src_ptrs.data_ptr<int64_t>();
  g.src_offset = src_offset;
  g.rows_per_rank = (int)rows_per_rank;
  g.rows = rows;
  g.cols = cols;
  g.dst = (__nv_bfloat16*)w.data_ptr();
  g.ready = reinterpret_cast<uint32_t*>(ready.data_ptr<int>());
  // pieces of whole rows of about 16 KB, a power of two per 64-row chunk
  int rpp = 64;
  while (rpp > 1 && (int64_t)rpp * cols * 2 > 16384) rpp >>= 1;
  g.rows_per_piece = rpp;
  g.pieces_per_chunk = 64 / rpp;
  g.target = (uint32_t)((uint64_t)epoch * (uint64_t)g.pieces_per_chunk);
  g.chunks = chunks;
  g.first_chunk = chunks > 0 ? (int)((rank * rows_per_rank) / 64) % chunks : 0;
  return g;
}

// GEMM with an all-gather fused in.  `gw` (rows x cols bf16, local) receives a row-sharded
// weight: src_ptrs holds every rank's bf16 shard-buffer base address (int64 [world]), the
// weight's shard starts at element src_offset of each and holds rows_per_rank rows; ready
// are int32 counters owned by gw (one per 64 rows, zeroed once at allocation) and epoch
// counts the gathers into gw so far including this one.  When `b` is `gw` the product
// waits for the rows it reads (forward d = a gw^T, or data gradient d = a gw with b_mn);
// otherwise the gather is a prefetch for a later product and `b` is any operand, in the
// forward, data-gradient or weight-gradient layouts of `gemm`.
void gemm_gather(torch::Tensor a, torch::Tensor b, torch::Tensor d, bool a_mn, bool b_mn, bool accumulate,
                 torch::Tensor gw, torch::Tensor src_ptrs, int64_t src_offset, int64_t rows_per_rank, int64_t rank,
                 torch::Tensor ready, int64_t epoch) {
  GatherParams g = make_gather(gw, src_ptrs, src_offset, rows_per_rank, rank, ready, epoch, "gemm_gather");
  g.wait_b = b.data_ptr() == gw.data_ptr() ? 1 : 0;
  TORCH_CHECK(!g.wait_b || b.sizes() == gw.sizes(), "gemm_gather: b aliases gw with another shape");
  run_gemm(a, b, d, c10::nullopt, a_mn, b_mn, 1.0, 0.0, accumulate, false, &g);
}

// Gather only (no product): the same copy as gemm_gather's gather warps, with a grid of its
// own.  Used where a sharded weight is needed outside a large GEMM (decode-sized products,
// checkpoints) and as the unfused comparison in tests.
__global__ void __launch_bounds__(32 * kGatherWarps) shard_gather_kernel(const GatherParams g) {
  gather_rows(g, blockIdx.x * kGatherWarps + threadIdx.x / 32, gridDim.x * kGatherWarps, threadIdx.x % 32);
}

void shard_gather(torch::Tensor w, torch::Tensor src_ptrs, int64_t src_offset, int64_t rows_per_rank, int64_t rank,
                  torch::Tensor ready, int64_t epoch) {
  GatherParams g = make_gather(w, src_ptrs, src_offset, rows_per_rank, rank, ready, epoch, "shard_gather");
  if (g.rows == 0) return;
  c10::cuda::CUDAGuard guard(w.device());
  const int pieces = g.chunks * g.pieces_per_chunk;
  const int blocks = std::max(1, std::min((pieces + kGatherWarps - 1) / kGatherWarps, 4 * num_sms(w.get_device())));
  shard_gather_kernel<<<blocks, 32 * kGatherWarps, 0, at::cuda::getCurrentCUDAStream()>>>(g);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mykb
