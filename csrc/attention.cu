// FlashAttention forward / backward on tcgen05 (sm_100a).
//
// Forward, one CTA per (sequence, head, 128-query tile) work item, persistent over items:
//   warp 0      TMA producer: Q tile once per item, then K/V tiles of 128 keys into a
//               two-stage ring (128-byte swizzle, plain per-CTA copies).
//   warp 1      MMA issuer: S = Q K^T into tensor memory (M=128, N=128, K=d), then
//               O_j = P_j V_j into tensor memory (M=128, N=d, K=128) once the softmax
//               warps have written P_j.
//   warps 2-5   softmax: thread t owns query row t.  Reads its S row from TMEM, applies
//               scale and masks (causal / window / sequence end), updates the running max
//               and sum in base 2, writes P (bf16) into a 128-byte-swizzled shared tile,
//               and folds O_{j-1} (read from TMEM) into a register accumulator rescaled by
//               exp2(m_{j-1} - m_j).  At the end: O / l to global, LSE (natural log).
// Two CTAs fit on one SM for head_dim 64, so one CTA's softmax overlaps the other's MMAs.
//
// Backward, kernel 1 (dK/dV per 128-key tile), per work item (sequence, kv head, key
// tile), looping over the query tiles and the query heads of the GQA group:
//   S^T  = K Q^T          (M=128 keys, N=64 queries, K=d)
//   dP^T = V dO^T         (M=128 keys, N=64 queries, K=d)
//   P^T  = exp(S^T - lse), dS^T = P^T * (dP^T - Delta)   (registers; thread = key row)
//   dV  += P^T dO         (M=128, N=d, K=queries; A = P^T from TMEM)
//   dK  += dS^T Q         (M=128, N=d, K=queries; A = dS^T from TMEM)
// over 64-query sub-tiles with double-buffered S^T / dP^T so MMAs overlap the softmax.
// Kernel 2 (dQ per 128-query tile) recomputes S and dP over 64-key sub-tiles the same way
// and accumulates dQ += dS K in TMEM (A = dS from TMEM): no atomics, a deterministic result.
// Both backward kernels run eight softmax-gradient warps (two per SM sub-partition, each
// owning half of the tile's columns).  Delta = rowsum(dO * O) comes from a small pre-kernel.
//
// Semantics follow the reference (src/myk_llm/ops/flash_attn.py): queries end-aligned to
// the keys, window (left, right) with -1 unbounded, empty rows output 0 with LSE +inf.
#include <type_traits>

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.h"

namespace mykb {

constexpr int kFaThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct FaParams {
  int num_seqs;      // batch size, or number of packed documents
  int heads, kv_heads, group;
  int q_tiles;       // ceil(max_q / 128)
  int total_items;
  int max_q, max_k;
  const int* cu_q;   // packed offsets (nullptr for batch layout)
  const int* cu_k;
  const int* seqused_k;  // per-sequence key count (static caches), or nullptr
  int left, right;   // window; -1 unbounded
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* out;
  int64_t out_row_stride;  // elements between consecutive token rows (= heads * d)
  float* lse;        // (heads, total_q) packed or (batch, heads, max_q)
  int* status;
};

struct SeqGeom {
  int q_start, k_start;  // first row of this sequence in the 2-D (token, head*d) view
  int len_q, len_k;
};

__device__ __forceinline__ SeqGeom seq_geom(const FaParams& p, int s) {
  SeqGeom g;
  if (p.cu_q != nullptr) {
    g.q_start = p.cu_q[s];
    g.len_q = p.cu_q[s + 1] - g.q_start;
    g.k_start = p.cu_k[s];
    g.len_k = p.cu_k[s + 1] - g.k_start;
  } else {
    g.q_start = s * p.max_q;
    g.len_q = p.max_q;
    g.k_start = s * p.max_k;
    g.len_k = p.max_k;
  }
  if (p.seqused_k != nullptr) g.len_k = p.seqused_k[s];
  return g;
}

struct Item {
  int seq, head, qt;
  SeqGeom g;
  int q0;        // first query of the tile (within the sequence)
  int rows;      // valid query rows in the tile
  int kv_lo, kv_hi;  // key range [lo, hi) the tile needs
  int n_kv;      // number of 128-key tiles
};

// Work items: CTA c takes items c, c + grid, c + 2 grid, ...  The tiles of every (sequence,
// head) column are cut into bands of kBand tiles, heaviest band first (so every CTA starts
// on heavy tiles and the tail is light); inside a band the items run column by column, and
// band b is rotated by b * kBand items.  So the tiles of one long document go to different
// CTAs whatever the number of columns: numbering by tile first sends every tile of a
// column to the same CTA whenever the column count is a multiple of the grid, and one long
// packed document then serialises there.
constexpr int kBand = 4;
__host__ __device__ __forceinline__ int fa_item_count(int tiles, int cols) {
  return (tiles + kBand - 1) / kBand * kBand * cols;
}
// (band-ordered tile index from the heavy end, column) of item w
__device__ __forceinline__ void fa_item_coords(int w, int cols, int& t, int& col) {
  const int band = kBand * cols;
  const int b = w / band;
  const int r = (w % band + b * kBand) % band;
  col = r / kBand;
  t = b * kBand + r % kBand;
}

__device__ __forceinline__ bool decode_item(const FaParams& p, int w, Item& it) {
  int t, col;
  fa_item_coords(w, p.num_seqs * p.heads, t, col);
  if (t >= p.q_tiles) return false;
  it.qt = p.q_tiles - 1 - t;  // heaviest (last) query tiles first
  it.seq = col / p.heads;
  it.head = col % p.heads;
  it.g = seq_geom(p, it.seq);
  it.q0 = it.qt * 128;
  if (it.q0 >= it.g.len_q) return false;
  it.rows = min(128, it.g.len_q - it.q0);
  const int off = it.g.len_k - it.g.len_q;  // end alignment
  const int qlo = it.q0 + off, qhi = it.q0 + it.rows - 1 + off;
  int lo = 0, hi = it.g.len_k;
  if (p.left >= 0) lo = max(lo, qlo - p.left);
  if (p.right >= 0) hi = min(hi, qhi + p.right + 1);
  it.kv_lo = lo;
  it.kv_hi = hi;
  it.n_kv = hi > lo ? (hi - lo + 127) / 128 : 0;
  return true;
}

template <int D>
struct FaSmem {
  static constexpr int kTile = 128 * D * 2;  // one 128-row tile of head_dim D (bf16)
  static constexpr int kQ = 0;
  static constexpr int kK0 = kQ + kTile;
  static constexpr int kV0 = kK0 + 2 * kTile;
  static constexpr int kP = kV0 + 2 * kTile;
  static constexpr int kBars = kP + 128 * 128 * 2;
  // The dynamic shared window of a CTA without static shared memory starts 1024-byte
  // aligned; the kernel checks this (status word) instead of paying 1 KB of slack, which
  // would keep two head_dim-64 CTAs from sharing an SM.
  static constexpr int kTotal = kBars + 128;
};

// Loads a 128-row x D tile: D/64 boxes of {64, 128}, each 16 KB.
template <int D>
__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int col0, int row0) {
#pragma unroll
  // the token maps are 3-D (batch extent 1), so the 3-D form of the copy is required
  for (int part = 0; part < D / 64; ++part) tma_load_3d(dst + part * 16384, map, bar, col0 + part * 64, row0, 0);
}

// K-major operand descriptor for 16-wide K step kk of a tile whose K dimension is split
// into 64-element atoms 16 KB apart.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return make_sw128_desc(base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}
// MN-major operand descriptor (atoms of 64 along N, 16 KB apart), K step kk of 16 rows.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk) {
  return make_sw128_desc(base + kk * 2048, 16384, 1024);
}

template <int D>
__global__ void __launch_bounds__(kFaThreads, (D == 64 ? 2 : 1))
fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV, const FaParams p) {
  using S = FaSmem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem) & 1023) != 0) {
    if (threadIdx.x == 0) set_status(p.status, kMisaligned);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBars);
  uint64_t* kv_full = bars;       // [2]
  uint64_t* kv_empty = bars + 2;  // [2]
  uint64_t* q_full = bars + 4;
  uint64_t* q_empty = bars + 5;
  uint64_t* s_full = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* o_full = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  constexpr int kTmemCols = 256;  // S: columns [0,128), O: [128, 128+D)

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int items = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < p.total_items && ok; w += gridDim.x) {
        Item it;
        if (!decode_item(p, w, it) || it.n_kv == 0) continue;
        if (!mbar_wait(q_empty, (items & 1) ^ 1, p.status, __LINE__)) break;
        mbar_arrive_expect_tx(q_full, S::kTile);
        load_tile<D>(smem + S::kQ, &tmQ, q_full, it.head * D, it.g.q_start + it.q0);
        const int kvh = it.head / p.group;
        for (int j = 0; j < it.n_kv; ++j) {
          if (!mbar_wait(&kv_empty[stage], phase ^ 1, p.status, __LINE__)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[stage], 2 * S::kTile);
          const int row = it.g.k_start + it.kv_lo + j * 128;
          load_tile<D>(smem + S::kK0 + stage * S::kTile, &tmK, &kv_full[stage], kvh * D, row);
          load_tile<D>(smem + S::kV0 + stage * S::kTile, &tmV, &kv_full[stage], kvh * D, row);
          if (++stage == 2) { stage = 0; phase ^= 1; }
        }
        ++items;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16(128, D, false, true);
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int items = 0, ntile = 0;
      bool ok = true;
      const uint32_t q_addr = smem_u32(smem + S::kQ);
      const uint32_t p_addr = smem_u32(smem + S::kP);
      for (int w = blockIdx.x; w < p.total_items && ok; w += gridDim.x) {
        Item it;
        if (!decode_item(p, w, it) || it.n_kv == 0) continue;
        if (!mbar_wait(q_full, items & 1, p.status, __LINE__)) break;
        tc_fence_after();
        for (int j = 0; j < it.n_kv && ok; ++j, ++ntile) {
          // S_j = Q K_j^T
          if (!mbar_wait(&kv_full[stage], phase, p.status, __LINE__)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + S::kK0 + stage * S::kTile);
          const uint32_t v_addr = smem_u32(smem + S::kV0 + stage * S::kTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_bf16_ss(tmem, kmajor_desc(q_addr, kk), kmajor_desc(k_addr, kk), idesc_s, kk > 0);
          umma_commit(s_full);
          if (j == it.n_kv - 1) umma_commit(q_empty);
          // O_j = P_j V_j once the softmax warps have written P_j
          if (!mbar_wait(p_full, ntile & 1, p.status, __LINE__)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16_ss(tmem + 128, kmajor_desc(p_addr, kk), mnmajor_desc(v_addr, kk), idesc_o,
                         (j > 0 || kk > 0) ? 1u : 0u);  // O accumulates in TMEM over the KV tiles
          umma_commit(o_full);
          umma_commit(&kv_empty[stage]);
          if (++stage == 2) { stage = 0; phase ^= 1; }
        }
        ++items;
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax
    // One pass per KV tile: the 128 scores of this thread's row are loaded into registers,
    // the row max taken on the raw scores, and p = exp2(s * scale_log2 - m_ref) computed
    // with one FFMA + one EX2.  O accumulates in TMEM (PV MMAs with accumulate); the
    // reference max m_ref only moves when the row max grows by more than 2^8 (lazy
    // rescale), and then this warp rescales its 32 rows of O in TMEM before the next PV.
    const int q = warp & 3;
    const int row = q * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t p_base = smem_u32(smem + S::kP) + row * 128;
    const uint32_t swz = row & 7;
    constexpr float kRescaleThreshold = 8.f;  // log2 units
    int ntile = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.total_items && ok; w += gridDim.x) {
      Item it;
      if (!decode_item(p, w, it)) continue;
      const int off = it.g.len_k - it.g.len_q;
      const int qpos = it.q0 + row + off;  // absolute key-space position of this query
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j, ++ntile) {
        if (!mbar_wait_warp(s_full, ntile & 1, p.status, __LINE__)) { ok = false; break; }
        tc_fence_after();
        const int k0 = it.kv_lo + j * 128;
        const bool edge = (k0 + 127 >= it.g.len_k) || (p.right >= 0 && k0 + 127 > it.q0 + off + p.right) ||
                          (p.left >= 0 && k0 < it.q0 + it.rows - 1 + off - p.left);
        // keys visible to this row form one range [kmin, kmax); as offsets into this tile:
        const int kmin = (p.left >= 0 ? max(0, qpos - p.left) : 0) - k0;
        const int kspan = max(0, min(it.g.len_k, p.right >= 0 ? qpos + p.right + 1 : it.g.len_k) - k0 - kmin);
        // pass 1 over TMEM: row max of the raw scores (masked on edge tiles)
        float mx = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t cr[32];
          tmem_ld32_raw(tmem + lane_base + c * 32, cr);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float sc = __uint_as_float(cr[i]);
            if (edge && (unsigned)(c * 32 + i - kmin) >= (unsigned)kspan) sc = -INFINITY;
            mx = fmaxf(mx, sc);
          }
        }
        const float m_tile = mx * p.scale_log2;  // scale > 0: max commutes with it
        const bool grow = m_tile > m_ref + kRescaleThreshold;
        bool o_ready = false;
        if (__any_sync(0xffffffffu, grow)) {
          // rescale: every lane adopts its current max (a no-op factor for lanes that
          // did not grow beyond it)
          const float m_new = fmaxf(m_ref, m_tile);
          const float alpha = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - m_new);
          l *= alpha;
          m_ref = m_new;
          if (j > 0) {
            if (!mbar_wait_warp(o_full, (ntile - 1) & 1, p.status, __LINE__)) { ok = false; break; }
            tc_fence_after();
            o_ready = true;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              uint32_t ov[32];
              tmem_ld32_raw(tmem + lane_base + 128 + c * 32, ov);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
              tmem_st32(tmem + lane_base + 128 + c * 32, ov);
            }
          }
        }
        // pass 2 over TMEM: exponentials (overlapping the previous PV MMA), bf16 pairs
        const float neg = (m_ref == -INFINITY) ? 0.f : -m_ref;
        float rs = 0.f;
        uint32_t sr[64];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t cr[32];
          tmem_ld32_raw(tmem + lane_base + c * 32, cr);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float s0 = __uint_as_float(cr[i]), s1 = __uint_as_float(cr[i + 1]);
            if (edge) {
              if ((unsigned)(c * 32 + i - kmin) >= (unsigned)kspan) s0 = -INFINITY;
              if ((unsigned)(c * 32 + i + 1 - kmin) >= (unsigned)kspan) s1 = -INFINITY;
            }
            const float p0 = exp2f(fmaf(s0, p.scale_log2, neg));
            const float p1 = exp2f(fmaf(s1, p.scale_log2, neg));
            rs += p0 + p1;
            sr[(c * 32 + i) >> 1] = pack_bf16x2(p0, p1);
          }
        }
        l += rs;
        if (j > 0 && !o_ready) {
          // PV_{j-1} must be done before P is overwritten
          if (!mbar_wait_warp(o_full, (ntile - 1) & 1, p.status, __LINE__)) { ok = false; break; }
        }
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          const uint32_t addr = p_base + (ch >> 3) * 16384 + (((ch & 7) ^ swz) * 16);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(sr[ch * 4 + 0]),
                       "r"(sr[ch * 4 + 1]), "r"(sr[ch * 4 + 2]), "r"(sr[ch * 4 + 3])
                       : "memory");
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      if (!ok) break;
      // epilogue: O / l and LSE
      float inv = l > 0.f ? 1.f / l : 0.f;
      const int64_t tok = it.g.q_start + it.q0 + row;
      __nv_bfloat16* dst = p.out + tok * p.out_row_stride + (int64_t)it.head * D;
      if (it.n_kv > 0) {
        if (!mbar_wait_warp(o_full, (ntile - 1) & 1, p.status, __LINE__)) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ov[32];
          tmem_ld32_raw(tmem + lane_base + 128 + c * 32, ov);
          tmem_wait_ld();
          if (row < it.rows) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 v;
              v.x = pack_bf16x2(__uint_as_float(ov[8 * i + 0]) * inv, __uint_as_float(ov[8 * i + 1]) * inv);
              v.y = pack_bf16x2(__uint_as_float(ov[8 * i + 2]) * inv, __uint_as_float(ov[8 * i + 3]) * inv);
              v.z = pack_bf16x2(__uint_as_float(ov[8 * i + 4]) * inv, __uint_as_float(ov[8 * i + 5]) * inv);
              v.w = pack_bf16x2(__uint_as_float(ov[8 * i + 6]) * inv, __uint_as_float(ov[8 * i + 7]) * inv);
              reinterpret_cast<uint4*>(dst + c * 32)[i] = v;
            }
          }
        }
        tc_fence_before();
      } else if (row < it.rows) {
        for (int i = 0; i < D / 8; ++i) reinterpret_cast<uint4*>(dst)[i] = make_uint4(0, 0, 0, 0);
      }
      if (row < it.rows) {
        const float lse = l > 0.f ? (m_ref + log2f(l)) * kLn2 : INFINITY;
        if (p.cu_q != nullptr)
          p.lse[(int64_t)it.head * p.cu_q[p.num_seqs] + tok] = lse;
        else
          p.lse[((int64_t)it.seq * p.heads + it.head) * p.max_q + it.q0 + row] = lse;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// -------------------------------------------------------------------------------------
// Forward for GQA groups of even size: one work item = the same 128-query tile of two
// query heads that share a KV head (tiles A and B), so every K / V tile is loaded once
// for both.  Warp 0 loads, warp 1 issues MMAs, warps 2-5 run the softmax of tile A and
// warps 6-9 that of tile B.  The MMA warp interleaves the tiles,
//     S_A(0) S_B(0) | PV_A(0) S_A(1) | PV_B(0) S_B(1) | PV_A(1) S_A(2) | ...
// so the tensor pipe computes one tile while the other tile's softmax runs.  P is written
// back into the first 64 columns of its S region as packed bf16 and O += P V takes A from
// TMEM.  A commit after S_T(j) also covers PV_T(j - 1) (issued before it), so when a
// softmax warp sees S_T(j) it may rescale O_T and overwrite P_T.
//
// TMEM columns: S_A [0, 128), S_B [128, 256), O_A [256, 256 + D), O_B [256 + D, 256 + 2 D).
// -------------------------------------------------------------------------------------
template <int D>
struct FaPairSmem {
  static constexpr int kStages = D == 64 ? 3 : 2;  // K / V ring depth
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kQ = 0;                      // Q_A, then Q_B
  static constexpr int kKV0 = 2 * kTile;            // stage s: K at kKV0 + 2 s kTile, V after it
  static constexpr int kBars = kKV0 + kStages * 2 * kTile;
  static constexpr int kTotal = kBars + 256;
};

constexpr int kFaPairThreads = 64 + 32 * 8;

struct PairItem {
  int seq, kvh, pair, qt;
  SeqGeom g;
  int q0, rows, kv_lo, n_kv;
};

__device__ __forceinline__ bool decode_pair(const FaParams& p, int w, PairItem& it) {
  // banded, rotated order of decode_item; heaviest query tiles first
  const int pairs = p.group / 2;
  int t, rem;
  fa_item_coords(w, p.num_seqs * p.kv_heads * pairs, t, rem);
  if (t >= p.q_tiles) return false;
  it.qt = p.q_tiles - 1 - t;
  it.seq = rem / (p.kv_heads * pairs);
  rem %= p.kv_heads * pairs;
  it.kvh = rem / pairs;
  it.pair = rem % pairs;
  it.g = seq_geom(p, it.seq);
  it.q0 = it.qt * 128;
  if (it.q0 >= it.g.len_q) return false;
  it.rows = min(128, it.g.len_q - it.q0);
  const int off = it.g.len_k - it.g.len_q;
  const int qlo = it.q0 + off, qhi = it.q0 + it.rows - 1 + off;
  int lo = 0, hi = it.g.len_k;
  if (p.left >= 0) lo = max(lo, qlo - p.left);
  if (p.right >= 0) hi = min(hi, qhi + p.right + 1);
  it.kv_lo = lo;
  it.n_kv = hi > lo ? (hi - lo + 127) / 128 : 0;
  return true;
}

template <int D>
__global__ void __launch_bounds__(kFaPairThreads, 1)
fa_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const FaParams p) {
  using S = FaPairSmem<D>;
  constexpr int ST = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem) & 1023) != 0) {
    if (threadIdx.x == 0) set_status(p.status, kMisaligned);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBars);
  uint64_t* kv_full = bars;            // [ST]
  uint64_t* kv_empty = bars + ST;      // [ST]
  uint64_t* q_full = bars + 2 * ST;
  uint64_t* q_empty = q_full + 1;
  uint64_t* s_full = q_full + 2;       // [2] per tile
  uint64_t* p_full = q_full + 4;       // [2]
  uint64_t* o_full = q_full + 6;       // [2] last PV of the item done
  uint64_t* o_free = q_full + 8;       // [2] epilogue read O
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_full + 10);
  constexpr int kCols = 512;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int total = fa_item_count(p.q_tiles, p.num_seqs * p.kv_heads * (p.group / 2));
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_full[t], 1);
      mbar_init(&o_free[t], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0, items = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        PairItem it;
        if (!decode_pair(p, w, it) || it.n_kv == 0) continue;
        if (!mbar_wait(q_empty, (items & 1) ^ 1, p.status, __LINE__)) break;
        mbar_arrive_expect_tx(q_full, 2 * S::kTile);
        const int h0 = it.kvh * p.group + 2 * it.pair;
        load_tile<D>(smem + S::kQ, &tmQ, q_full, h0 * D, it.g.q_start + it.q0);
        load_tile<D>(smem + S::kQ + S::kTile, &tmQ, q_full, (h0 + 1) * D, it.g.q_start + it.q0);
        for (int j = 0; j < it.n_kv; ++j) {
          if (!mbar_wait(&kv_empty[stage], phase ^ 1, p.status, __LINE__)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[stage], 2 * S::kTile);
          const int row = it.g.k_start + it.kv_lo + j * 128;
          uint8_t* kd = smem + S::kKV0 + stage * 2 * S::kTile;
          load_tile<D>(kd, &tmK, &kv_full[stage], it.kvh * D, row);
          load_tile<D>(kd + S::kTile, &tmV, &kv_full[stage], it.kvh * D, row);
          if (++stage == ST) { stage = 0; phase ^= 1; }
        }
        ++items;
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16(128, D, false, true);  // A = P from TMEM
    if (elect_one()) {
      int stage = 0, items = 0;
      uint32_t phase = 0, ntile = 0;  // KV tiles processed so far (all items)
      bool ok = true;
      const uint32_t qa = smem_u32(smem + S::kQ), qb = qa + S::kTile;
      auto k_addr = [&](int st) { return smem_u32(smem + S::kKV0 + st * 2 * S::kTile); };
      auto issue_s = [&](int t, int st) {
        const uint32_t q = t == 0 ? qa : qb;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_bf16_ss(tmem + t * 128, kmajor_desc(q, kk), kmajor_desc(k_addr(st), kk), idesc_s, kk > 0);
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int st, bool acc) {
        const uint32_t v = k_addr(st) + S::kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16_ts(tmem + 256 + t * D, tmem + t * 128 + kk * 8, mnmajor_desc(v, kk), idesc_o,
                       (acc || kk > 0) ? 1u : 0u);
      };
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        PairItem it;
        if (!decode_pair(p, w, it) || it.n_kv == 0) continue;
        if (!mbar_wait(q_full, items & 1, p.status, __LINE__)) break;
        if (!mbar_wait(&kv_full[stage], phase, p.status, __LINE__)) break;
        tc_fence_after();
        issue_s(0, stage);
        issue_s(1, stage);
        if (it.n_kv == 1) umma_commit(q_empty);
        for (int j = 0; j < it.n_kv && ok; ++j, ++ntile) {
          const int cur = stage;
          int nxt = stage + 1;
          uint32_t nphase = phase;
          if (nxt == ST) { nxt = 0; nphase ^= 1; }
          const bool more = j + 1 < it.n_kv;
          for (int t = 0; t < 2; ++t) {
            if (j == 0 && !mbar_wait(&o_free[t], (items & 1) ^ 1, p.status, __LINE__)) { ok = false; break; }
            if (!mbar_wait(&p_full[t], ntile & 1, p.status, __LINE__)) { ok = false; break; }
            tc_fence_after();
            issue_pv(t, cur, j > 0);
            if (!more) umma_commit(&o_full[t]);
            if (t == 1) umma_commit(&kv_empty[cur]);
            if (more) {
              if (t == 0 && !mbar_wait(&kv_full[nxt], nphase, p.status, __LINE__)) { ok = false; break; }
              tc_fence_after();
              issue_s(t, nxt);
              if (t == 1 && j + 2 == it.n_kv) umma_commit(q_empty);
            }
          }
          stage = nxt;
          phase = nphase;
        }
        ++items;
      }
    }
  } else {
    // softmax: thread = query row of tile t; same online softmax as fa_fwd_kernel (row
    // max over the raw scores, lazy rescale when the max grows by more than 2^8)
    const int t = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t s_col = t * 128, o_col = 256 + t * D;
    constexpr float kRescaleThreshold = 8.f;  // log2 units
    uint32_t ntile = 0;
    int items = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
      PairItem it;
      if (!decode_pair(p, w, it)) continue;
      const int h = it.kvh * p.group + 2 * it.pair + t;
      const int off = it.g.len_k - it.g.len_q;
      const int qpos = it.q0 + row + off;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j, ++ntile) {
        if (!mbar_wait_warp(&s_full[t], ntile & 1, p.status, __LINE__)) { ok = false; break; }
        tc_fence_after();
        const int k0 = it.kv_lo + j * 128;
        const bool edge = (k0 + 127 >= it.g.len_k) || (p.right >= 0 && k0 + 127 > it.q0 + off + p.right) ||
                          (p.left >= 0 && k0 < it.q0 + it.rows - 1 + off - p.left);
        const int kmin = (p.left >= 0 ? max(0, qpos - p.left) : 0) - k0;
        const int kspan = max(0, min(it.g.len_k, p.right >= 0 ? qpos + p.right + 1 : it.g.len_k) - k0 - kmin);
        float mx = -INFINITY;
        // two 32-column TMEM loads in flight per wait
#pragma unroll 1
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t cr[2][32];
          tmem_ld32_raw(tmem + lane_base + s_col + c2 * 64, cr[0]);
          tmem_ld32_raw(tmem + lane_base + s_col + c2 * 64 + 32, cr[1]);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = 2 * c2 + h;
            if (edge) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                float sc = __uint_as_float(cr[h][i]);
                if ((unsigned)(c * 32 + i - kmin) >= (unsigned)kspan) sc = -INFINITY;
                mx = fmaxf(mx, sc);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; i += 2) mx = fmax3(mx, __uint_as_float(cr[h][i]), __uint_as_float(cr[h][i + 1]));
            }
          }
        }
        const float m_tile = mx * p.scale_log2;
        const bool grow = m_tile > m_ref + kRescaleThreshold;
        if (__any_sync(0xffffffffu, grow)) {
          const float m_new = fmaxf(m_ref, m_tile);
          const float alpha = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - m_new);
          l *= alpha;
          m_ref = m_new;
          if (j > 0) {  // PV_t(j - 1) is complete: the commit of S_t(j) covers it
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              uint32_t ov[32];
              tmem_ld32_raw(tmem + lane_base + o_col + c * 32, ov);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
              tmem_st32(tmem + lane_base + o_col + c * 32, ov);
            }
          }
        }
        const float neg = (m_ref == -INFINITY) ? 0.f : -m_ref;
        const float2 scale2 = make_float2(p.scale_log2, p.scale_log2), neg2 = make_float2(neg, neg);
        float2 rs2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t cr[2][32];
          tmem_ld32_raw(tmem + lane_base + s_col + c2 * 64, cr[0]);
          tmem_ld32_raw(tmem + lane_base + s_col + c2 * 64 + 32, cr[1]);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = 2 * c2 + h;
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float s0 = __uint_as_float(cr[h][i]), s1 = __uint_as_float(cr[h][i + 1]);
              if (edge) {
                if ((unsigned)(c * 32 + i - kmin) >= (unsigned)kspan) s0 = -INFINITY;
                if ((unsigned)(c * 32 + i + 1 - kmin) >= (unsigned)kspan) s1 = -INFINITY;
              }
              const float2 a = ffma2(make_float2(s0, s1), scale2, neg2);  // both exponents in one FMA
              const float2 pv = make_float2(exp2f(a.x), exp2f(a.y));
              rs2 = fadd2(rs2, pv);
              pk[i >> 1] = pack_bf16x2(pv.x, pv.y);
            }
            // P columns [16 c, 16 c + 16) lie in S columns this thread has already read
            tmem_st16_raw(tmem + lane_base + s_col + c * 16, pk);
          }
        }
        l += rs2.x + rs2.y;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int64_t tok = it.g.q_start + it.q0 + row;
      __nv_bfloat16* dst = p.out + tok * p.out_row_stride + (int64_t)h * D;
      if (it.n_kv > 0) {
        if (!mbar_wait_warp(&o_full[t], items & 1, p.status, __LINE__)) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ov[32];
          tmem_ld32_raw(tmem + lane_base + o_col + c * 32, ov);
          tmem_wait_ld();
          if (row < it.rows) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 v;
              v.x = pack_bf16x2(__uint_as_float(ov[8 * i + 0]) * inv, __uint_as_float(ov[8 * i + 1]) * inv);
              v.y = pack_bf16x2(__uint_as_float(ov[8 * i + 2]) * inv, __uint_as_float(ov[8 * i + 3]) * inv);
              v.z = pack_bf16x2(__uint_as_float(ov[8 * i + 4]) * inv, __uint_as_float(ov[8 * i + 5]) * inv);
              v.w = pack_bf16x2(__uint_as_float(ov[8 * i + 6]) * inv, __uint_as_float(ov[8 * i + 7]) * inv);
              reinterpret_cast<uint4*>(dst + c * 32)[i] = v;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[t]);
        ++items;
      } else if (row < it.rows) {
        for (int i = 0; i < D / 8; ++i) reinterpret_cast<uint4*>(dst)[i] = make_uint4(0, 0, 0, 0);
      }
      if (row < it.rows) {
        const float lse = l > 0.f ? (m_ref + log2f(l)) * kLn2 : INFINITY;
        if (p.cu_q != nullptr)
          p.lse[(int64_t)h * p.cu_q[p.num_seqs] + tok] = lse;
        else
          p.lse[((int64_t)it.seq * p.heads + h) * p.max_q + it.q0 + row] = lse;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// -------------------------------------------------------------------------------------
// host
// -------------------------------------------------------------------------------------
static int sm_count() {
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// 2-D (token rows, head*d cols) tensor map of a (.., tokens, heads, d) tensor.
static CUtensorMap token_map(const torch::Tensor& t) {
  const int64_t d = t.size(-1), h = t.size(-2);
  // size-1 dimensions may carry any stride: only strides that address data are checked
  TORCH_CHECK(t.stride(-1) == 1 && (h == 1 || t.stride(-2) == d), "attention: heads must be packed (stride d)");
  int64_t row_stride = t.stride(-3);
  int64_t rows = t.size(-3);
  if (t.dim() == 4) {
    if (t.size(1) == 1)
      row_stride = t.stride(0);  // one token per sequence: rows step over the batch
    else
      TORCH_CHECK(t.size(0) == 1 || t.stride(0) == t.size(1) * row_stride,
                  "attention: batch rows must be uniformly strided");
    rows *= t.size(0);
  }
  if (rows == 1) row_stride = h * d;
  return make_tmap_3d(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, h * d, rows, 1, row_stride, 0, 64, 128);
}

template <int D>
static void launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const FaParams& p,
                       cudaStream_t st) {
  using S = FaSmem<D>;
  auto kern = fa_fwd_kernel<D>;
  static SmemOptIn configured;
  C10_CUDA_CHECK(configured.ensure(kern, S::kTotal));
  if (p.group % 2 == 0) {
    // GQA with an even group: two query heads per work item sharing each K / V tile
    using SP = FaPairSmem<D>;
    auto pk = fa_fwd_pair_kernel<D>;
    static SmemOptIn pair_configured;
    C10_CUDA_CHECK(pair_configured.ensure(pk, SP::kTotal));
    const int items = fa_item_count(p.q_tiles, p.num_seqs * p.kv_heads * (p.group / 2));
    pk<<<std::max(1, std::min(items, sm_count())), kFaPairThreads, SP::kTotal, st>>>(tq, tk, tv, p);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const int per_sm = D == 64 ? 2 : 1;
  const int grid = std::max(1, std::min(p.total_items, sm_count() * per_sm));
  kern<<<grid, kFaThreads, S::kTotal, st>>>(tq, tk, tv, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

std::vector<torch::Tensor> fa_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, c10::optional<torch::Tensor> cu_q,
                                  c10::optional<torch::Tensor> cu_k, c10::optional<torch::Tensor> seqused_k,
                                  int64_t max_q, int64_t max_k, double scale, int64_t left, int64_t right) {
  c10::cuda::CUDAGuard guard(q.device());
  const bool packed = cu_q.has_value();
  const int D = q.size(-1);
  TORCH_CHECK(D == 64 || D == 128, "fa_fwd: head_dim 64 or 128");
  FaParams p{};
  p.heads = q.size(-2);
  p.kv_heads = k.size(-2);
  p.group = p.heads / p.kv_heads;
  p.max_q = max_q;
  p.max_k = max_k;
  p.left = left;
  p.right = right;
  p.scale_log2 = (float)scale * kLog2e;
  torch::Tensor out, lse;
  if (packed) {
    TORCH_CHECK(cu_k.has_value() && cu_q->scalar_type() == at::kInt, "fa_fwd: int32 cu_seqlens");
    p.num_seqs = cu_q->numel() - 1;
    p.cu_q = cu_q->data_ptr<int>();
    p.cu_k = cu_k->data_ptr<int>();
    out = torch::empty({q.size(0), p.heads, D}, q.options());
    lse = torch::empty({p.heads, q.size(0)}, q.options().dtype(at::kFloat));
  } else {
    p.num_seqs = q.size(0);
    TORCH_CHECK(q.size(1) == max_q && k.size(1) == max_k, "fa_fwd: batch layout sizes");
    out = torch::empty({q.size(0), q.size(1), p.heads, D}, q.options());
    lse = torch::empty({q.size(0), p.heads, q.size(1)}, q.options().dtype(at::kFloat));
  }
  if (seqused_k.has_value()) {
    TORCH_CHECK(seqused_k->scalar_type() == at::kInt, "fa_fwd: int32 seqused_k");
    p.seqused_k = seqused_k->data_ptr<int>();
  }
  p.q_tiles = (int)((max_q + 127) / 128);
  p.total_items = fa_item_count(p.q_tiles, p.num_seqs * p.heads);
  p.out = (__nv_bfloat16*)out.data_ptr();
  p.out_row_stride = (int64_t)p.heads * D;
  p.lse = lse.data_ptr<float>();
  p.status = device_status();
  if (q.numel() == 0 || p.total_items == 0) return {out, lse};
  CUtensorMap tq = token_map(q), tk = token_map(k), tv = token_map(v);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (D == 64) launch_fwd<64>(tq, tk, tv, p, st);
  else launch_fwd<128>(tq, tk, tv, p, st);
  return {out, lse};
}

// =====================================================================================
// backward: two kernels, each built from the operand patterns of the forward pass
// =====================================================================================
struct FaBwdParams {
  FaParams f;          // geometry (heads, seqs, window, ...); f.out / f.lse unused
  int k_tiles;         // ceil(max_k / 128)
  const float2* ld;    // {base-2 LSE, Delta = rowsum(dO * O)} per (query, head), in the LSE layout
  __nv_bfloat16* dq;   // (tokens, heads, d)
  __nv_bfloat16* dk;   // (tokens_k, kv_heads, d)
  __nv_bfloat16* dv;
  float scale;         // softmax scale (natural units)
};

__device__ __forceinline__ int64_t lse_index(const FaParams& f, int seq, int h, int q_start, int qi, int64_t total_q) {
  return f.cu_q != nullptr ? (int64_t)h * total_q + q_start + qi : ((int64_t)seq * f.heads + h) * f.max_q + qi;
}

// ------------------------------------------------------------------ dK / dV per key tile
struct BwdItem {
  int seq, kvh, kt;
  SeqGeom g;
  int k0, keys;
  int qt_lo, qt_hi;  // query tiles that can see this key tile
};

__device__ __forceinline__ bool decode_bwd(const FaBwdParams& p, int w, BwdItem& it) {
  // banded, rotated order of decode_item; early key tiles (most work under a causal
  // mask) first
  int t, col;
  fa_item_coords(w, p.f.num_seqs * p.f.kv_heads, t, col);
  if (t >= p.k_tiles) return false;
  it.kt = t;
  it.seq = col / p.f.kv_heads;
  it.kvh = col % p.f.kv_heads;
  it.g = seq_geom(p.f, it.seq);
  it.k0 = it.kt * 128;
  if (it.k0 >= it.g.len_k || it.g.len_q == 0) return false;
  it.keys = min(128, it.g.len_k - it.k0);
  const int off = it.g.len_k - it.g.len_q;
  int qlo = 0, qhi = it.g.len_q;
  if (p.f.right >= 0) qlo = max(qlo, it.k0 - p.f.right - off);
  if (p.f.left >= 0) qhi = min(qhi, it.k0 + it.keys - 1 + p.f.left - off + 1);
  if (qhi <= qlo) {
    it.qt_lo = it.qt_hi = 0;
  } else {
    it.qt_lo = qlo / 128;
    it.qt_hi = (qhi + 127) / 128;
  }
  return true;
}

template <int D>
struct DkvSmem {
  static constexpr int kStages = D == 64 ? 4 : 2;  // Q / dO ring depth
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kK = 0;
  static constexpr int kV = kK + kTile;
  static constexpr int kQ0 = kV + kTile;
  static constexpr int kDO0 = kQ0 + kStages * kTile;
  static constexpr int kLd = kDO0 + kStages * kTile;  // [stages][128] {base-2 LSE, Delta} of the query tile
  static constexpr int kBars = kLd + kStages * 1024;
  static constexpr int kTotal = kBars + 256;
};

// Backward kernels: producer warp, MMA warp, and two groups of four softmax-gradient warps
// (each SM sub-partition runs one warp of each group, so one hides the other's latency).
constexpr int kBwdSoftmaxWarps = 8;
constexpr int kFaBwdThreads = 64 + 32 * kBwdSoftmaxWarps;

// dK / dV kernel.  Each 128-query tile is processed as two 64-query sub-tiles u whose
// S^T / dP^T accumulators alternate between two TMEM buffers, so the tensor pipe computes
// sub-tile u + 1 (and the dV / dK products of u - 1) while the softmax warps work on u.
// The softmax warps write P^T and dS^T back into TMEM as packed bf16 over the columns
// they read, and dV += P^T dO, dK += dS^T Q take their A operand from TMEM.
//
// TMEM columns (b = u & 1):  S^T [128 b, 128 b + 64), dP^T [128 b + 64, 128 b + 128),
// dV [256, 256 + D), dK [256 + D, 256 + 2 D).  Softmax group h (of 2) owns queries
// [32 h, 32 h + 32) of a sub-tile and writes its 16 packed columns at the start of its own
// 32 columns, so A for K step kk (16 queries) is at column (kk / 2) * 32 + (kk % 2) * 8.
template <int D>
__global__ void __launch_bounds__(kFaBwdThreads, 1)
fa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                   const FaBwdParams p) {
  using S = DkvSmem<D>;
  constexpr int ST = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem) & 1023) != 0) {
    if (threadIdx.x == 0) set_status(p.f.status, kMisaligned);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBars);
  uint64_t* kv_full = bars + 0;
  uint64_t* kv_empty = bars + 1;
  uint64_t* q_full = bars + 2;        // [ST]
  uint64_t* q_empty = bars + 2 + ST;  // [ST]
  uint64_t* s_full = bars + 2 + 2 * ST;  // [2] per TMEM buffer
  uint64_t* ds_full = s_full + 2;        // [2]
  uint64_t* kk_done = s_full + 4;
  uint64_t* dkv_free = s_full + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 6);
  constexpr int kCols = 512;
  constexpr uint32_t kColDV = 256, kColDK = 256 + D;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int group = p.f.group;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int i = 0; i < ST; ++i) {
      mbar_init(&q_full[i], 1 + 32);  // the TMA transaction plus the producer lanes' cp.async
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&ds_full[i], kBwdSoftmaxWarps);
    }
    mbar_init(kk_done, 1);
    mbar_init(dkv_free, kBwdSoftmaxWarps);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = fa_item_count(p.k_tiles, p.f.num_seqs * p.f.kv_heads);

  if (warp == 0) {
    // Producer warp: lane 0 issues the TMA copies of Q / dO; every lane copies the
    // {LSE, Delta} pairs of four query rows with cp.async, whose completion the stage's
    // mbarrier tracks (one no-increment arrival per lane), so no load latency sits on the
    // producer's path.  Rows past the document are zero-filled (the masks drop them).
    const uint32_t s_ld = smem_u32(smem + S::kLd);
    const int64_t total_q = p.f.cu_q != nullptr ? (int64_t)p.f.cu_q[p.f.num_seqs] : 0;
    int stage = 0, items = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
      BwdItem it;
      if (!decode_bwd(p, w, it) || it.qt_hi <= it.qt_lo) continue;
      bool good = true;
      if (lane == 0) good = mbar_wait(kv_empty, (items & 1) ^ 1, p.f.status, __LINE__);
      if (!__shfl_sync(0xffffffffu, good, 0)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(kv_full, 2 * S::kTile);
        load_tile<D>(smem + S::kK, &tmK, kv_full, it.kvh * D, it.g.k_start + it.k0);
        load_tile<D>(smem + S::kV, &tmV, kv_full, it.kvh * D, it.g.k_start + it.k0);
      }
      for (int hh = 0; hh < group && ok; ++hh) {
        const int h = it.kvh * group + hh;
        for (int qt = it.qt_lo; qt < it.qt_hi; ++qt) {
          if (lane == 0) good = mbar_wait(&q_empty[stage], phase ^ 1, p.f.status, __LINE__);
          if (!__shfl_sync(0xffffffffu, good, 0)) { ok = false; break; }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int c = lane * 4 + i;
            const int qi = qt * 128 + c;
            const bool in = qi < it.g.len_q;
            const float2* src = in ? p.ld + lse_index(p.f, it.seq, h, it.g.q_start, qi, total_q) : p.ld;
            cp_async_8(s_ld + (uint32_t)(stage * 128 + c) * 8u, src, in);
          }
          cp_async_mbar_arrive_noinc(&q_full[stage]);
          if (lane == 0) {
            mbar_arrive_expect_tx(&q_full[stage], 2 * S::kTile);
            const int row = it.g.q_start + qt * 128;
            load_tile<D>(smem + S::kQ0 + stage * S::kTile, &tmQ, &q_full[stage], h * D, row);
            load_tile<D>(smem + S::kDO0 + stage * S::kTile, &tmDO, &q_full[stage], h * D, row);
          }
          if (++stage == ST) { stage = 0; phase ^= 1; }
        }
      }
      ++items;
    }
  } else if (warp == 1) {
    // MMA warp.  Per sub-tile u: S^T(u), dP^T(u) into buffer u & 1, then the dV / dK
    // products of u - 1 (whose P^T / dS^T the softmax warps have written by then).
    constexpr uint32_t idesc_s = make_idesc_bf16(128, 64, false, false);  // K Q^T, V dO^T (N = 64 queries)
    constexpr uint32_t idesc_kv = make_idesc_bf16(128, D, false, true);   // P^T dO, dS^T Q (A from TMEM)
    if (elect_one()) {
      int stage = 0, items = 0;
      uint32_t phase = 0;
      uint32_t u = 0;  // sub-tiles issued so far (all items)
      bool ok = true;
      const uint32_t k_addr = smem_u32(smem + S::kK), v_addr = smem_u32(smem + S::kV);
      // the pending sub-tile whose dV / dK products are not issued yet
      int pend_stage = 0, pend_j = 0;
      bool pend_last = false, pend_first = false, have_pend = false;
      auto issue_kv = [&](uint32_t uu) -> bool {
        const uint32_t b = uu & 1;
        if (!mbar_wait(&ds_full[b], (uu >> 1) & 1, p.f.status, __LINE__)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + S::kQ0 + pend_stage * S::kTile);
        const uint32_t do_addr = smem_u32(smem + S::kDO0 + pend_stage * S::kTile);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acol = b * 128 + (kk >> 1) * 32 + (kk & 1) * 8;
          umma_bf16_ts(tmem + kColDV, tmem + acol, mnmajor_desc(do_addr, pend_j * 4 + kk), idesc_kv,
                       (!pend_first || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acol = b * 128 + 64 + (kk >> 1) * 32 + (kk & 1) * 8;
          umma_bf16_ts(tmem + kColDK, tmem + acol, mnmajor_desc(q_addr, pend_j * 4 + kk), idesc_kv,
                       (!pend_first || kk > 0) ? 1u : 0u);
        }
        if (pend_last) umma_commit(&q_empty[pend_stage]);
        return true;
      };
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        BwdItem it;
        if (!decode_bwd(p, w, it) || it.qt_hi <= it.qt_lo) continue;
        if (!mbar_wait(kv_full, items & 1, p.f.status, __LINE__)) break;
        if (!mbar_wait(dkv_free, (items & 1) ^ 1, p.f.status, __LINE__)) break;
        tc_fence_after();
        bool first = true;
        for (int hh = 0; hh < group && ok; ++hh) {
          for (int qt = it.qt_lo; qt < it.qt_hi && ok; ++qt) {
            if (!mbar_wait(&q_full[stage], phase, p.f.status, __LINE__)) { ok = false; break; }
            tc_fence_after();
            const uint32_t q_addr = smem_u32(smem + S::kQ0 + stage * S::kTile);
            const uint32_t do_addr = smem_u32(smem + S::kDO0 + stage * S::kTile);
            for (int j = 0; j < 2; ++j, ++u) {
              const uint32_t b = u & 1;
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk)
                umma_bf16_ss(tmem + b * 128, kmajor_desc(k_addr, kk), kmajor_desc(q_addr + j * 8192, kk), idesc_s,
                             kk > 0);
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk)
                umma_bf16_ss(tmem + b * 128 + 64, kmajor_desc(v_addr, kk), kmajor_desc(do_addr + j * 8192, kk),
                             idesc_s, kk > 0);
              umma_commit(&s_full[b]);
              if (have_pend && !issue_kv(u - 1)) { ok = false; break; }
              pend_stage = stage;
              pend_j = j;
              pend_last = j == 1;
              pend_first = first && j == 0;
              have_pend = true;
            }
            first = false;
            if (++stage == ST) { stage = 0; phase ^= 1; }
          }
        }
        if (!ok) break;
        if (!issue_kv(u - 1)) break;
        have_pend = false;
        umma_commit(kk_done);
        umma_commit(kv_empty);
        ++items;
      }
    }
  } else {
    const int qw = warp & 3;
    const int half = (warp - 2) >> 2;  // queries [32 half, 32 half + 32) of each 64-query sub-tile
    const int r = qw * 32 + lane;      // TMEM lane = key row within the tile
    const uint32_t lane_base = (uint32_t)(qw * 32) << 16;
    const float4* s_ld = reinterpret_cast<const float4*>(smem + S::kLd);  // two queries per float4
    uint32_t u = 0;
    int n = 0, items = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
      BwdItem it;
      if (!decode_bwd(p, w, it)) continue;
      const int off = it.g.len_k - it.g.len_q;
      const int kp = it.k0 + r;
      if (it.qt_hi > it.qt_lo) {
        for (int hh = 0; hh < group && ok; ++hh) {
          for (int qt = it.qt_lo; qt < it.qt_hi && ok; ++qt, ++n) {
            const int st_idx = n % ST;
            for (int j = 0; j < 2; ++j, ++u) {
              const uint32_t b = u & 1;
              const int q0 = qt * 128 + 64 * j;  // first query of the sub-tile
              if (!mbar_wait_warp(&s_full[b], (u >> 1) & 1, p.f.status, __LINE__)) { ok = false; break; }
              tc_fence_after();
              float sv[32], dp[32];
              tmem_ld32_raw(tmem + lane_base + b * 128 + 32 * half, *reinterpret_cast<uint32_t(*)[32]>(sv));
              tmem_ld32_raw(tmem + lane_base + b * 128 + 64 + 32 * half, *reinterpret_cast<uint32_t(*)[32]>(dp));
              // every (key, query) pair of the sub-tile visible: no per-element masks
              const bool edge = (it.k0 + 127 >= it.g.len_k) || (q0 + 63 >= it.g.len_q) ||
                                (p.f.right >= 0 && it.k0 + 127 > q0 + off + p.f.right) ||
                                (p.f.left >= 0 && it.k0 < q0 + 63 + off - p.f.left);
              // the queries this key row sees form one range [lo, lo + span) of the 32 columns
              const int qb = q0 + 32 * half;
              int lo = 0, hi = min(32, it.g.len_q - qb);
              if (p.f.right >= 0) lo = max(lo, kp - off - p.f.right - qb);
              if (p.f.left >= 0) hi = min(hi, kp - off + p.f.left - qb + 1);
              const int span = kp < it.g.len_k ? max(0, hi - lo) : 0;
              // the stage's {LSE, Delta} pairs landed with its Q / dO tiles
              if (j == 0 && !mbar_wait_warp(&q_full[st_idx], (n / ST) & 1, p.f.status, __LINE__)) {
                ok = false;
                break;
              }
              const float4* c_ld = s_ld + (st_idx * 128 + 64 * j + 32 * half) / 2;
              tmem_wait_ld();
              uint32_t pk[16], dk[16];
              const float2 sc2 = make_float2(p.f.scale_log2, p.f.scale_log2), ps2 = make_float2(p.scale, p.scale);
              // one straight-line body per case, so the compiler can interleave all 32 columns
              auto body = [&](auto masked) {
#pragma unroll
                for (int i4 = 0; i4 < 16; ++i4) {
                  const float4 v = c_ld[i4];  // {lse2, delta} of queries 2 i4 and 2 i4 + 1
                  const int i = 2 * i4;
                  const float2 a = ffma2(make_float2(sv[i], sv[i + 1]), sc2, make_float2(-v.x, -v.z));
                  float2 pv = make_float2(exp2f(a.x), exp2f(a.y));
                  if constexpr (decltype(masked)::value) {
                    if ((unsigned)(i - lo) >= (unsigned)span) pv.x = 0.f;
                    if ((unsigned)(i + 1 - lo) >= (unsigned)span) pv.y = 0.f;
                  }
                  sv[i] = pv.x;
                  sv[i + 1] = pv.y;
                  const float2 d = fmul2(fmul2(pv, ps2), fadd2(make_float2(dp[i], dp[i + 1]), make_float2(-v.y, -v.w)));
                  dp[i] = d.x;
                  dp[i + 1] = d.y;
                }
              };
              if (edge)
                body(std::true_type{});
              else
                body(std::false_type{});
#pragma unroll
              for (int m = 0; m < 16; ++m) {
                pk[m] = pack_bf16x2(sv[2 * m], sv[2 * m + 1]);
                dk[m] = pack_bf16x2(dp[2 * m], dp[2 * m + 1]);
              }
              // packed P^T / dS^T over the first 16 of the 32 columns this warp group read
              tmem_st16_raw(tmem + lane_base + b * 128 + 32 * half, pk);
              tmem_st16_raw(tmem + lane_base + b * 128 + 64 + 32 * half, dk);
              tmem_wait_st();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&ds_full[b]);
            }
          }
        }
        if (!ok) break;
        if (!mbar_wait_warp(kk_done, items & 1, p.f.status, __LINE__)) break;
        tc_fence_after();
        const bool valid = r < it.keys;
        const int64_t krow = it.g.k_start + it.k0 + r;
        __nv_bfloat16* dkp = p.dk + (krow * p.f.kv_heads + it.kvh) * D;
        __nv_bfloat16* dvp = p.dv + (krow * p.f.kv_heads + it.kvh) * D;
#pragma unroll
        for (int c = half * (D / 64); c < (half + 1) * (D / 64); ++c) {
          float a[32], bv[32];
          tmem_ld32(tmem + lane_base + kColDK + c * 32, a);
          tmem_ld32(tmem + lane_base + kColDV + c * 32, bv);
          if (valid) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 ka, va;
              ka.x = pack_bf16x2(a[8 * i + 0], a[8 * i + 1]);
              ka.y = pack_bf16x2(a[8 * i + 2], a[8 * i + 3]);
              ka.z = pack_bf16x2(a[8 * i + 4], a[8 * i + 5]);
              ka.w = pack_bf16x2(a[8 * i + 6], a[8 * i + 7]);
              va.x = pack_bf16x2(bv[8 * i + 0], bv[8 * i + 1]);
              va.y = pack_bf16x2(bv[8 * i + 2], bv[8 * i + 3]);
              va.z = pack_bf16x2(bv[8 * i + 4], bv[8 * i + 5]);
              va.w = pack_bf16x2(bv[8 * i + 6], bv[8 * i + 7]);
              reinterpret_cast<uint4*>(dkp + c * 32)[i] = ka;
              reinterpret_cast<uint4*>(dvp + c * 32)[i] = va;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dkv_free);
        ++items;
      } else if (r < it.keys) {
        const int64_t krow = it.g.k_start + it.k0 + r;
        __nv_bfloat16* dkp = p.dk + (krow * p.f.kv_heads + it.kvh) * D;
        __nv_bfloat16* dvp = p.dv + (krow * p.f.kv_heads + it.kvh) * D;
        for (int i = half * (D / 16); i < (half + 1) * (D / 16); ++i) {
          reinterpret_cast<uint4*>(dkp)[i] = make_uint4(0, 0, 0, 0);
          reinterpret_cast<uint4*>(dvp)[i] = make_uint4(0, 0, 0, 0);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// ------------------------------------------------------------------ dQ per query tile
// Same item walk as the forward.  Each 128-key tile is processed as two 64-key sub-tiles u
// with S = Q K^T and dP = dO V^T (A, B K-major) double-buffered in TMEM; the softmax
// warps (thread = query row) write dS = P (dP - Delta) back over the S columns they read
// as packed bf16, and dQ += dS K takes A from TMEM (B = K sub-tile, MN-major).
//
// TMEM columns (b = u & 1): S [128 b, 128 b + 64), dP [128 b + 64, 128 b + 128),
// dQ [256, 256 + D).  Softmax group h owns keys [32 h, 32 h + 32) of a sub-tile.
template <int D>
struct DqSmem {
  static constexpr int kStages = D == 64 ? 4 : 2;  // K / V ring depth
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kQ = 0;
  static constexpr int kDO = kQ + kTile;
  static constexpr int kK0 = kDO + kTile;
  static constexpr int kV0 = kK0 + kStages * kTile;
  static constexpr int kBars = kV0 + kStages * kTile;
  static constexpr int kTotal = kBars + 256;
};

template <int D>
__global__ void __launch_bounds__(kFaBwdThreads, 1)
fa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                 const FaBwdParams p) {
  using S = DqSmem<D>;
  constexpr int ST = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem) & 1023) != 0) {
    if (threadIdx.x == 0) set_status(p.f.status, kMisaligned);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBars);
  uint64_t* kv_full = bars;             // [ST]
  uint64_t* kv_empty = bars + ST;       // [ST]
  uint64_t* q_full = bars + 2 * ST;
  uint64_t* q_empty = q_full + 1;
  uint64_t* s_full = q_full + 2;        // [2]
  uint64_t* ds_full = q_full + 4;       // [2]
  uint64_t* dq_done = q_full + 6;
  uint64_t* dq_free = q_full + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_full + 8);
  constexpr int kCols = 512;
  constexpr uint32_t kColDQ = 256;
  const FaParams& f = p.f;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&ds_full[i], kBwdSoftmaxWarps);
    }
    mbar_init(dq_done, 1);
    mbar_init(dq_free, kBwdSoftmaxWarps);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0, items = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < f.total_items && ok; w += gridDim.x) {
        Item it;
        if (!decode_item(f, w, it) || it.n_kv == 0) continue;
        if (!mbar_wait(q_empty, (items & 1) ^ 1, f.status, __LINE__)) break;
        mbar_arrive_expect_tx(q_full, 2 * S::kTile);
        load_tile<D>(smem + S::kQ, &tmQ, q_full, it.head * D, it.g.q_start + it.q0);
        load_tile<D>(smem + S::kDO, &tmDO, q_full, it.head * D, it.g.q_start + it.q0);
        const int kvh = it.head / f.group;
        for (int j = 0; j < it.n_kv; ++j) {
          if (!mbar_wait(&kv_empty[stage], phase ^ 1, f.status, __LINE__)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[stage], 2 * S::kTile);
          const int row = it.g.k_start + it.kv_lo + j * 128;
          load_tile<D>(smem + S::kK0 + stage * S::kTile, &tmK, &kv_full[stage], kvh * D, row);
          load_tile<D>(smem + S::kV0 + stage * S::kTile, &tmV, &kv_full[stage], kvh * D, row);
          if (++stage == ST) { stage = 0; phase ^= 1; }
        }
        ++items;
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = make_idesc_bf16(128, 64, false, false);  // Q K^T, dO V^T (N = 64 keys)
    constexpr uint32_t idesc_q = make_idesc_bf16(128, D, false, true);    // dS K (A from TMEM)
    if (elect_one()) {
      int stage = 0, items = 0;
      uint32_t phase = 0, u = 0;
      bool ok = true;
      const uint32_t q_addr = smem_u32(smem + S::kQ), do_addr = smem_u32(smem + S::kDO);
      int pend_stage = 0, pend_j = 0;
      bool pend_last = false, pend_first = false, have_pend = false;
      auto issue_dq = [&](uint32_t uu) -> bool {
        const uint32_t b = uu & 1;
        if (!mbar_wait(&ds_full[b], (uu >> 1) & 1, f.status, __LINE__)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + S::kK0 + pend_stage * S::kTile);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acol = b * 128 + (kk >> 1) * 32 + (kk & 1) * 8;
          umma_bf16_ts(tmem + kColDQ, tmem + acol, mnmajor_desc(k_addr, pend_j * 4 + kk), idesc_q,
                       (!pend_first || kk > 0) ? 1u : 0u);
        }
        if (pend_last) umma_commit(&kv_empty[pend_stage]);
        return true;
      };
      for (int w = blockIdx.x; w < f.total_items && ok; w += gridDim.x) {
        Item it;
        if (!decode_item(f, w, it) || it.n_kv == 0) continue;
        if (!mbar_wait(q_full, items & 1, f.status, __LINE__)) break;
        if (!mbar_wait(dq_free, (items & 1) ^ 1, f.status, __LINE__)) break;
        tc_fence_after();
        for (int jt = 0; jt < it.n_kv && ok; ++jt) {
          if (!mbar_wait(&kv_full[stage], phase, f.status, __LINE__)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + S::kK0 + stage * S::kTile);
          const uint32_t v_addr = smem_u32(smem + S::kV0 + stage * S::kTile);
          for (int j = 0; j < 2; ++j, ++u) {
            const uint32_t b = u & 1;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              umma_bf16_ss(tmem + b * 128, kmajor_desc(q_addr, kk), kmajor_desc(k_addr + j * 8192, kk), idesc_s,
                           kk > 0);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              umma_bf16_ss(tmem + b * 128 + 64, kmajor_desc(do_addr, kk), kmajor_desc(v_addr + j * 8192, kk),
                           idesc_s, kk > 0);
            umma_commit(&s_full[b]);
            if (jt == it.n_kv - 1 && j == 1) umma_commit(q_empty);
            if (have_pend && !issue_dq(u - 1)) { ok = false; break; }
            pend_stage = stage;
            pend_j = j;
            pend_last = j == 1;
            pend_first = jt == 0 && j == 0;
            have_pend = true;
          }
          if (++stage == ST) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (!issue_dq(u - 1)) break;
        have_pend = false;
        umma_commit(dq_done);
        ++items;
      }
    }
  } else {
    const int qw = warp & 3;
    const int half = (warp - 2) >> 2;  // keys [32 half, 32 half + 32) of each 64-key sub-tile
    const int row = qw * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qw * 32) << 16;
    const int64_t total_q = f.cu_q != nullptr ? (int64_t)f.cu_q[f.num_seqs] : 0;
    uint32_t u = 0;
    int items = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < f.total_items && ok; w += gridDim.x) {
      Item it;
      if (!decode_item(f, w, it)) continue;
      const int off = it.g.len_k - it.g.len_q;
      const int qi = it.q0 + row;
      const int qpos = qi + off;
      const bool qvalid = row < it.rows;
      const bool qvalid_tile = it.rows == 128;
      float lse2 = INFINITY, dl = 0.f;
      if (qvalid) {
        const float2 v = p.ld[lse_index(f, it.seq, it.head, it.g.q_start, qi, total_q)];
        lse2 = v.x;
        dl = v.y;
      }
      for (int jt = 0; jt < it.n_kv && ok; ++jt) {
        for (int j = 0; j < 2; ++j, ++u) {
          const uint32_t b = u & 1;
          if (!mbar_wait_warp(&s_full[b], (u >> 1) & 1, f.status, __LINE__)) { ok = false; break; }
          tc_fence_after();
          float sv[32], dp[32];
          tmem_ld32_raw(tmem + lane_base + b * 128 + 32 * half, *reinterpret_cast<uint32_t(*)[32]>(sv));
          tmem_ld32_raw(tmem + lane_base + b * 128 + 64 + 32 * half, *reinterpret_cast<uint32_t(*)[32]>(dp));
          const int k0 = it.kv_lo + jt * 128 + 64 * j;  // first key of the sub-tile
          const bool edge = !qvalid_tile || (k0 + 63 >= it.g.len_k) ||
                            (f.right >= 0 && k0 + 63 > it.q0 + off + f.right) ||
                            (f.left >= 0 && k0 < it.q0 + it.rows - 1 + off - f.left);
          // keys visible to this row form one range; as offsets from k0:
          const int kmin = (f.left >= 0 ? max(0, qpos - f.left) : 0) - k0;
          const int kspan =
              qvalid ? max(0, min(it.g.len_k, f.right >= 0 ? qpos + f.right + 1 : it.g.len_k) - k0 - kmin) : 0;
          const float ps = p.scale;
          tmem_wait_ld();
          uint32_t dk[16];
          const float2 sc2 = make_float2(f.scale_log2, f.scale_log2), nl2 = make_float2(-lse2, -lse2);
          const float2 ps2 = make_float2(ps, ps), nd2 = make_float2(-dl, -dl);
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 a = ffma2(make_float2(sv[i], sv[i + 1]), sc2, nl2);
            float2 pv = make_float2(exp2f(a.x), exp2f(a.y));
            if (edge) {
              if ((unsigned)(32 * half + i - kmin) >= (unsigned)kspan) pv.x = 0.f;
              if ((unsigned)(32 * half + i + 1 - kmin) >= (unsigned)kspan) pv.y = 0.f;
            }
            const float2 d = fmul2(fmul2(pv, ps2), fadd2(make_float2(dp[i], dp[i + 1]), nd2));
            dk[i >> 1] = pack_bf16x2(d.x, d.y);
          }
          tmem_st16_raw(tmem + lane_base + b * 128 + 32 * half, dk);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ds_full[b]);
        }
      }
      if (!ok) break;
      const int64_t tok = it.g.q_start + it.q0 + row;
      __nv_bfloat16* dst = p.dq + (tok * f.heads + it.head) * D;
      if (it.n_kv > 0) {
        if (!mbar_wait_warp(dq_done, items & 1, f.status, __LINE__)) break;
        tc_fence_after();
#pragma unroll
        for (int c = half * (D / 64); c < (half + 1) * (D / 64); ++c) {
          float v[32];
          tmem_ld32(tmem + lane_base + kColDQ + c * 32, v);
          if (qvalid) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 o;
              o.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
              o.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
              o.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
              o.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
              reinterpret_cast<uint4*>(dst + c * 32)[i] = o;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_free);
        ++items;
      } else if (qvalid) {
        for (int i = half * (D / 16); i < (half + 1) * (D / 16); ++i)
          reinterpret_cast<uint4*>(dst)[i] = make_uint4(0, 0, 0, 0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// ld[row, h] = {LSE * log2(e), Delta = sum_d dO * O} (fp32), in the LSE layout: what the
// backward kernels read per query, one 8-byte load.
__global__ void fa_delta_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                const float* __restrict__ lse, float2* __restrict__ ld, int64_t rows, int heads,
                                int D, bool packed, int max_q) {
  // D / 8 consecutive lanes share one (token, head) row: one 16-byte load of each tensor
  // per lane, then a shuffle reduction within the group.
  const int per = D / 8;
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t gw = t / per;
  const int sub = (int)(t % per);
  const bool active = gw < rows * heads;
  float s = 0.f;
  if (active) {
    const uint4 x = *reinterpret_cast<const uint4*>(dout + gw * D + sub * 8);
    const uint4 y = *reinterpret_cast<const uint4*>(out + gw * D + sub * 8);
    const __nv_bfloat162* xa = reinterpret_cast<const __nv_bfloat162*>(&x);
    const __nv_bfloat162* ya = reinterpret_cast<const __nv_bfloat162*>(&y);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = __bfloat1622float2(xa[i]), b = __bfloat1622float2(ya[i]);
      s = fmaf(a.x, b.x, fmaf(a.y, b.y, s));
    }
  }
  for (int o = per / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
  if (active && sub == 0) {
    const int64_t tok = gw / heads;
    const int h = (int)(gw % heads);
    const int64_t li = packed ? (int64_t)h * rows + tok : ((tok / max_q) * heads + h) * max_q + tok % max_q;
    ld[li] = make_float2(lse[li] * kLog2e, s);
  }
}

template <int D>
static void launch_bwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                       const FaBwdParams& p, cudaStream_t st) {
  {
    using S = DkvSmem<D>;
    auto kern = fa_bwd_dkdv_kernel<D>;
    static SmemOptIn configured;
    C10_CUDA_CHECK(configured.ensure(kern, S::kTotal));
    const int total = fa_item_count(p.k_tiles, p.f.num_seqs * p.f.kv_heads);
    kern<<<std::max(1, std::min(total, sm_count())), kFaBwdThreads, S::kTotal, st>>>(tq, tk, tv, tdo, p);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  {
    using S = DqSmem<D>;
    auto kern = fa_bwd_dq_kernel<D>;
    static SmemOptIn configured;
    C10_CUDA_CHECK(configured.ensure(kern, S::kTotal));
    kern<<<std::max(1, std::min(p.f.total_items, sm_count())), kFaBwdThreads, S::kTotal, st>>>(tq, tk, tv, tdo, p);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

std::vector<torch::Tensor> fa_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                  torch::Tensor out, torch::Tensor lse, c10::optional<torch::Tensor> cu_q,
                                  c10::optional<torch::Tensor> cu_k, int64_t max_q, int64_t max_k, double scale,
                                  int64_t left, int64_t right) {
  c10::cuda::CUDAGuard guard(q.device());
  const bool packed = cu_q.has_value();
  const int D = q.size(-1);
  FaBwdParams p{};
  FaParams& f = p.f;
  f.heads = q.size(-2);
  f.kv_heads = k.size(-2);
  f.group = f.heads / f.kv_heads;
  f.max_q = max_q;
  f.max_k = max_k;
  f.left = left;
  f.right = right;
  f.scale_log2 = (float)scale * kLog2e;
  f.status = device_status();
  if (packed) {
    f.num_seqs = cu_q->numel() - 1;
    f.cu_q = cu_q->data_ptr<int>();
    f.cu_k = cu_k->data_ptr<int>();
  } else {
    f.num_seqs = q.size(0);
  }
  f.q_tiles = (int)((max_q + 127) / 128);
  f.total_items = fa_item_count(f.q_tiles, f.num_seqs * f.heads);
  p.k_tiles = (int)((max_k + 127) / 128);
  p.scale = (float)scale;
  auto dout_c = dout.contiguous();
  const int64_t q_rows = packed ? q.size(0) : q.size(0) * q.size(1);
  const int64_t k_rows = packed ? k.size(0) : k.size(0) * k.size(1);
  auto dq = torch::empty({q_rows, f.heads, D}, q.options());
  auto dk = torch::empty({k_rows, f.kv_heads, D}, q.options());
  auto dv = torch::empty({k_rows, f.kv_heads, D}, q.options());
  TORCH_CHECK(lse.is_contiguous() && lse.scalar_type() == at::kFloat, "fa_bwd: contiguous fp32 lse");
  auto ld = torch::empty({lse.numel(), 2}, lse.options());  // {base-2 LSE, Delta} per (query, head)
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (q_rows > 0) {
    const int64_t threads = q_rows * f.heads * (D / 8);
    fa_delta_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
        (const __nv_bfloat16*)dout_c.data_ptr(), (const __nv_bfloat16*)out.data_ptr(), lse.data_ptr<float>(),
        reinterpret_cast<float2*>(ld.data_ptr<float>()), q_rows, f.heads, D, packed, (int)max_q);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  p.ld = reinterpret_cast<const float2*>(ld.data_ptr<float>());
  p.dq = (__nv_bfloat16*)dq.data_ptr();
  p.dk = (__nv_bfloat16*)dk.data_ptr();
  p.dv = (__nv_bfloat16*)dv.data_ptr();
  if (k_rows > 0 && q_rows > 0) {
    auto dout4 = packed ? dout_c.view({q_rows, f.heads, D}) : dout_c;
    CUtensorMap tq = token_map(q), tk = token_map(k), tv = token_map(v), tdo = token_map(dout4);
    if (D == 64) launch_bwd<64>(tq, tk, tv, tdo, p, st);
    else launch_bwd<128>(tq, tk, tv, tdo, p, st);
  } else {
    dq.zero_();
    dk.zero_();
    dv.zero_();
  }
  if (!packed) {
    dq = dq.view(q.sizes());
    dk = dk.view(k.sizes());
    dv = dv.view(v.sizes());
  }
  return {dq, dk, dv};
}

}  // namespace mykb

// =====================================================================================
// C entry point without device allocation (declared in noalloc.h).  No counterpart in
// the reference project: see noalloc.h for who needs it and the contract.
// =====================================================================================
#include "noalloc.h"

namespace mykb {
namespace {
// Working memory of mykb_flash_attn_bwd_noalloc: {base-2 LSE, Delta} (two floats per query
// row and head) and the status word its bounded waits write.  Every GPU that loads this
// library holds these (8 MB + 256 B) until the process exits.
static __device__ __align__(256) float2 g_noalloc_ld[MYKB_NOALLOC_MAX_ROWS_X_HEADS];
static __device__ __align__(256) int g_noalloc_status[64];

thread_local char g_noalloc_err[256] = {0};

struct NoallocScratch {
  float2* ld = nullptr;
  int* status = nullptr;
};

// Host-side stand-ins of the arrays are not device addresses: look the addresses up once
// per device (with that device current) and pass them to the kernels.  The mutex makes
// first calls from several host threads safe.
NoallocScratch noalloc_scratch(int dev, cudaError_t* err) {
  static std::mutex mu;
  static NoallocScratch cache[64];
  static bool ready[64] = {false};
  *err = cudaSuccess;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return {};
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ready[dev]) {
    NoallocScratch s;
    *err = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.ld), g_noalloc_ld);
    if (*err != cudaSuccess) return {};
    *err = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.status), g_noalloc_status);
    if (*err != cudaSuccess) return {};
    cache[dev] = s;
    ready[dev] = true;
  }
  return cache[dev];
}

int noalloc_fail(int code, const char* msg) {
  snprintf(g_noalloc_err, sizeof(g_noalloc_err), "%s", msg);
  return code;
}

CUtensorMap raw_token_map(const void* base, int64_t rows, int heads, int d) {
  return make_tmap_3d(const_cast<void*>(base), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (int64_t)heads * d, rows, 1,
                      (int64_t)heads * d, 0, 64, 128);
}
}  // namespace
}  // namespace mykb

extern "C" int mykb_flash_attn_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v,
                                           const void* out, const float* lse, void* dq, void* dk, void* dv,
                                           const int* cu_seqlens, int num_seqs, int rows_q, int rows_k, int max_q,
                                           int max_k, int heads, int kv_heads, int head_dim, float softmax_scale,
                                           int window_left, int window_right, cudaStream_t stream) {
  using namespace mykb;
  g_noalloc_err[0] = 0;
  if (head_dim != 64 && head_dim != 128) return noalloc_fail(1, "head_dim must be 64 or 128");
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads) return noalloc_fail(2, "heads must be a multiple of kv_heads");
  if (rows_q <= 0 || rows_k <= 0 || num_seqs <= 0 || max_q <= 0 || max_k <= 0)
    return noalloc_fail(4, "empty problem");
  const bool packed = cu_seqlens != nullptr;
  if (packed) {
    // One cu_seqlens serves queries and keys, so both sides hold the same documents.
    if (rows_k != rows_q) return noalloc_fail(9, "packed layout: q and k share cu_seqlens, so rows_k must equal rows_q");
  } else {
    if ((int64_t)num_seqs * max_q != rows_q || (int64_t)num_seqs * max_k != rows_k)
      return noalloc_fail(10, "batch layout: rows_q must equal num_seqs * max_q and rows_k num_seqs * max_k");
  }
  // Delta holds one float per (query row, head) in either layout.
  if ((int64_t)rows_q * heads > MYKB_NOALLOC_MAX_ROWS_X_HEADS)
    return noalloc_fail(3, "rows_q * heads exceeds MYKB_NOALLOC_MAX_ROWS_X_HEADS (the built-in scratch size)");
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return noalloc_fail(5, cudaGetErrorString(err));
  NoallocScratch sc = noalloc_scratch(dev, &err);
  if (err != cudaSuccess) return noalloc_fail(6, cudaGetErrorString(err));
  // A wait that gave up in an earlier call must not make this call's waits give up too.
  err = cudaMemsetAsync(sc.status, 0, sizeof(int), stream);
  if (err != cudaSuccess) return noalloc_fail(7, cudaGetErrorString(err));
  try {
    FaBwdParams p{};
    FaParams& f = p.f;
    f.heads = heads;
    f.kv_heads = kv_heads;
    f.group = heads / kv_heads;
    f.max_q = max_q;
    f.max_k = max_k;
    f.left = window_left;
    f.right = window_right;
    f.scale_log2 = softmax_scale * kLog2e;
    f.status = sc.status;
    f.num_seqs = num_seqs;
    f.cu_q = cu_seqlens;
    f.cu_k = cu_seqlens;
    f.q_tiles = (max_q + 127) / 128;
    f.total_items = fa_item_count(f.q_tiles, f.num_seqs * f.heads);
    p.k_tiles = (max_k + 127) / 128;
    p.scale = softmax_scale;
    p.ld = sc.ld;
    p.dq = static_cast<__nv_bfloat16*>(dq);
    p.dk = static_cast<__nv_bfloat16*>(dk);
    p.dv = static_cast<__nv_bfloat16*>(dv);
    const int64_t threads = (int64_t)rows_q * heads * (head_dim / 8);
    fa_delta_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(dout), static_cast<const __nv_bfloat16*>(out), lse, sc.ld, rows_q, heads,
        head_dim, packed, max_q);
    err = cudaGetLastError();
    if (err != cudaSuccess) return noalloc_fail(7, cudaGetErrorString(err));
    CUtensorMap tq = raw_token_map(q, rows_q, heads, head_dim), tk = raw_token_map(k, rows_k, kv_heads, head_dim),
                tv = raw_token_map(v, rows_k, kv_heads, head_dim), tdo = raw_token_map(dout, rows_q, heads, head_dim);
    if (head_dim == 64) launch_bwd<64>(tq, tk, tv, tdo, p, stream);
    else launch_bwd<128>(tq, tk, tv, tdo, p, stream);
  } catch (const std::exception& e) {
    return noalloc_fail(8, e.what());
  }
  err = cudaGetLastError();
  if (err != cudaSuccess) return noalloc_fail(7, cudaGetErrorString(err));
  return 0;
}

extern "C" const char* mykb_noalloc_last_error(void) { return mykb::g_noalloc_err; }

extern "C" int mykb_noalloc_status(int clear) {
  using namespace mykb;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return -noalloc_fail(5, cudaGetErrorString(err));
  NoallocScratch sc = noalloc_scratch(dev, &err);
  if (err != cudaSuccess) return -noalloc_fail(6, cudaGetErrorString(err));
  int h = 0;
  err = cudaMemcpy(&h, sc.status, sizeof(int), cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return -noalloc_fail(7, cudaGetErrorString(err));
  if (clear && h != 0) {
    err = cudaMemset(sc.status, 0, sizeof(int));
    if (err != cudaSuccess) return -noalloc_fail(7, cudaGetErrorString(err));
  }
  return h;
}

extern "C" void* mykb_noalloc_status_address(void) {
  using namespace mykb;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return nullptr;
  NoallocScratch sc = noalloc_scratch(dev, &err);
  return err == cudaSuccess ? sc.status : nullptr;
}
