// Tensor-core building blocks of the Gated DeltaNet chunk kernels (sm_100a, tcgen05).
//
// Every operand tile is bf16 in shared memory in the 128-byte-swizzled layout the tensor
// core reads: a tile of R rows x (64 * nb) columns is stored as nb column blocks of R rows
// x 128 bytes (R * 128 bytes apart), and inside a block the 16-byte chunk j of row r sits
// at chunk position j ^ (r % 8).  The same tile serves as a K-major operand (its rows are
// the M / N index, its columns the reduction index) and as an MN-major operand (its
// columns are the M / N index, its rows the reduction index), so a product and its
// transpose read one copy.  TMA loads with 128-byte swizzle write exactly this layout.
//
// Chunk products have 64 rows (one chunk of tokens).  A 64-row tcgen05 accumulator
// occupies TMEM lanes 0-15 of each 32-lane sub-partition; these kernels split an N-column
// product into two N/2-column MMAs whose accumulators sit at lane offsets 0 and 16 of the
// same columns, so a warp's 32x32b load returns 16 rows of each half: lane l of warp w
// holds row 16 (w % 4) + (l % 16), column half l / 16, and warps w and w + 4 split the
// half's columns.
#pragma once

#include "common.cuh"

namespace mykb {
namespace gtc {

typedef __nv_bfloat16 bf16;

// K-major operand: tile rows [row0, row0 + M/N) are the M / N index, K step kk (16
// columns) of the reduction over the tile's columns.
__device__ __forceinline__ uint64_t desc_k(uint32_t base, int R, int row0, int kk) {
  return make_sw128_desc(base + (uint32_t)((kk >> 2) * R * 128 + row0 * 128 + (kk & 3) * 32), 16, 1024);
}
// MN-major operand: tile columns [col0, ...) are the M / N index (col0 a multiple of 64,
// or 32 for a 32-wide operand inside one block), K step kk (16 rows) of the reduction over
// the tile's rows.
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int R, int col0, int kk) {
  return make_sw128_desc(base + (uint32_t)((col0 >> 6) * R * 128 + (col0 & 63) * 2 + kk * 2048), (uint32_t)(R * 128),
                         1024);
}

// Byte offset of element (r, c) in a swizzled tile of R rows.
__device__ __forceinline__ uint32_t sw_off(int R, int r, int c) {
  return (uint32_t)((c >> 6) * R * 128 + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}

// Stores 8 consecutive columns [c, c + 8) of row r (c a multiple of 8) as bf16.
__device__ __forceinline__ void st8(uint8_t* tile, int R, int r, int c, const float* v) {
  uint4 w;
  w.x = pack_bf16x2(v[0], v[1]);
  w.y = pack_bf16x2(v[2], v[3]);
  w.z = pack_bf16x2(v[4], v[5]);
  w.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(tile + sw_off(R, r, c)) = w;
}
// Loads 8 consecutive bf16 columns [c, c + 8) of row r as floats.
__device__ __forceinline__ void ld8(const uint8_t* tile, int R, int r, int c, float* v) {
  const uint4 w = *reinterpret_cast<const uint4*>(tile + sw_off(R, r, c));
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// 4-byte asynchronous global -> shared copy (cp.async); zero-filled when !valid.
__device__ __forceinline__ void cp_async_4(uint32_t dst_smem, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst_smem), "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (warp-collective, no wait).
__device__ __forceinline__ void tmem_ld16_raw(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// One 64-row product D (+)= A B^T of N = 2 * NH columns and K = 16 * KS, issued by one
// thread as two NH-column MMAs per K step (accumulators at TMEM lane offsets 0 and 16 of
// columns [col, col + NH)).  a(kk) gives the A descriptor; b(half, kk) the B descriptor of
// columns [half * NH, half * NH + NH).
template <int NH, int KS, bool A_MN, bool B_MN, typename FA, typename FB>
__device__ __forceinline__ void mma64(uint32_t tmem, uint32_t col, FA a, FB b, bool accumulate) {
  constexpr uint32_t idesc = make_idesc_bf16(64, NH, A_MN, B_MN);
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    const uint64_t da = a(kk);
#pragma unroll
    for (int half = 0; half < 2; ++half)
      umma_bf16_ss(tmem + ((uint32_t)(16 * half) << 16) + col, da, b(half, kk), idesc,
                   (accumulate || kk > 0) ? 1u : 0u);
  }
}

// TMEM address of this thread's part of a 64-row accumulator at column `col` whose halves
// are NH wide: lanes of the warp's sub-partition, columns [col + (w / 4) NH / 2, + NH / 2).
__device__ __forceinline__ uint32_t acc_addr(uint32_t tmem, uint32_t col, int NH) {
  const int w = threadIdx.x >> 5;
  return tmem + ((uint32_t)(32 * (w & 3)) << 16) + col + (uint32_t)((w >> 2) * (NH / 2));
}

// This thread's accumulator row and first output column (for halves NH wide).
__device__ __forceinline__ int acc_row() { return 16 * ((threadIdx.x >> 5) & 3) + (threadIdx.x & 15); }
__device__ __forceinline__ int acc_col0(int NH) {
  return ((threadIdx.x & 31) >> 4) * NH + ((threadIdx.x >> 5) >> 2) * (NH / 2);
}

}  // namespace gtc
}  // namespace mykb
