// Chunk geometry of the Gated DeltaNet kernels: which token rows a global 64-token chunk
// covers, for packed documents (cu_seqlens) or a batch of equal-length rows.
#pragma once

#include <stdint.h>

namespace mykb {
namespace gdnk {

constexpr int kChunk = 64;  // tokens per chunk

struct Geo {
  const int* cu;         // packed document offsets or nullptr (batch layout)
  const int* chunk_off;  // first global chunk of every sequence; [num_seqs] = total
  const int* order;      // sequences by decreasing length (sequential kernels start long ones first)
  int num_seqs, heads, seq_len;
  int64_t rows;          // token rows (batch x time); per-token scalars are head-major [heads][rows]
  int64_t row_q, row_v;  // elements between consecutive token rows of q/k and of v
};

__device__ __forceinline__ void seq_span(const Geo& g, int s, int& t0, int& len) {
  if (g.cu != nullptr) {
    t0 = g.cu[s];
    len = g.cu[s + 1] - t0;
  } else {
    t0 = s * g.seq_len;
    len = g.seq_len;
  }
}

// Global chunk -> (first token row, valid rows).  False for chunk indices past the end.
__device__ __forceinline__ bool locate(const Geo& g, int chunk, int& row0, int& n) {
  if (chunk >= g.chunk_off[g.num_seqs]) return false;
  int lo = 0, hi = g.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (g.chunk_off[mid] <= chunk) lo = mid; else hi = mid - 1;
  }
  int t0, len;
  seq_span(g, lo, t0, len);
  const int a = (chunk - g.chunk_off[lo]) * kChunk;
  row0 = t0 + a;
  n = min(kChunk, len - a);
  return n > 0;
}

}  // namespace gdnk
}  // namespace mykb
