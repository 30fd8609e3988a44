// Bucket function of the hashed n-gram tables (a checkpoint contract: the same token
// window must address the same table row as in the reference model,
// src/myk_llm/model/embeddings.py).  For the order-n window ending at position t (tok[0]
// is the token at t, tok[-o] the one o places before; missing left context is the
// sentinel id):  h = n;  for o in 0..n-1:  h = h * M[o % 4] + tok[-o] + 1;  h ^= h >> 29
// (wrapping int64, arithmetic shift);  row = h mod buckets, in [0, buckets).
#pragma once

#include <stdint.h>

namespace mykb {

static __constant__ uint64_t kNgramMul[4] = {0x1F3D5B79A2C4E681ull, 0x0DDC0FFEEBADF00Dull, 0x1B873593CC9E2D51ull,
                                      0x0000000100000001B3ull};

__device__ __forceinline__ int64_t ngram_bucket(const int64_t* tok, int order, int64_t buckets) {
  int64_t h = order;
  for (int o = 0; o < order; ++o) {
    const uint64_t u = (uint64_t)h * kNgramMul[o & 3] + (uint64_t)tok[-o] + 1ull;
    h = (int64_t)u;
    h ^= h >> 29;
  }
  const int64_t r = h % buckets;
  return r < 0 ? r + buckets : r;
}

}  // namespace mykb
