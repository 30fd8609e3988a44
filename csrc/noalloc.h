// C entry point of the FlashAttention backward that allocates no device memory.
//
// This entry point has no counterpart in the reference project.  It exists for callers
// that cannot allocate GPU memory themselves: code running while a CUDA graph is being
// captured into a memory pool it does not own, inference runtimes and plugins that only
// receive pre-allocated buffers from their host framework, and processes whose memory is
// budgeted up front so that a cudaMalloc in the middle of a step would fail or stall.
// The caller passes every input and output buffer; the only working memory (the
// per-row Delta = rowsum(dO * O) and a status word) lives in file-scope device arrays of
// a fixed maximum size inside this library.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest rows * heads the built-in scratch holds (two floats per query row and head).
#define MYKB_NOALLOC_MAX_ROWS_X_HEADS (1 << 20)

// FlashAttention backward for packed (cu_seqlens != NULL, num_seqs documents) or batch
// (cu_seqlens == NULL, num_seqs sequences of max_q / max_k tokens) layouts.  q / out / dout /
// dq are (rows_q, heads, head_dim) bf16, k / v / dk / dv are (rows_k, kv_heads, head_dim)
// bf16, all contiguous; lse is the forward's natural-log LSE laid out (heads, rows_q)
// (packed) or (num_seqs, heads, max_q) (batch).  window_left / window_right: -1 = unbounded
// (causal is window_right = 0).  head_dim must be 64 or 128.
//
// Packed layout: the one cu_seqlens array gives the document boundaries of both queries
// and keys, so rows_k must equal rows_q.  Batch layout: rows_q must equal num_seqs * max_q
// and rows_k must equal num_seqs * max_k.  Calls that break either rule are rejected.
//
// Returns 0 when the work was enqueued on `stream`.  A non-zero return is an error code
// and mykb_noalloc_last_error() describes it (the message is kept per host thread); sizes
// beyond MYKB_NOALLOC_MAX_ROWS_X_HEADS are rejected without launching anything.
//
// The kernels' waits are bounded: a wait that gives up records a non-zero code in this
// device's status word and the kernels wind down, leaving dq / dk / dv incomplete.  The
// call itself cannot see that (it does not synchronise), so read the word with
// mykb_noalloc_status() after synchronising the stream.  Each call clears the word on its
// stream before its kernels run.
//
// The first call on a device looks up the device address of the scratch arrays
// (cudaGetSymbolAddress) for that device; make that first call before any stream
// capture.  All calls share the one scratch array of a device, so calls that overlap on
// the GPU (different streams, no ordering between them) race; serialise them.  The array
// keeps the previous call's contents: every element a call reads is written by that call
// first.
int mykb_flash_attn_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v, const void* out,
                                const float* lse, void* dq, void* dk, void* dv, const int* cu_seqlens,
                                int num_seqs, int rows_q, int rows_k, int max_q, int max_k, int heads,
                                int kv_heads, int head_dim, float softmax_scale, int window_left,
                                int window_right, cudaStream_t stream);

const char* mykb_noalloc_last_error(void);

// Status word of the current device's allocation-free calls: 0 when every wait of the
// calls since the last clear completed, else the code of the wait that gave up.  It
// synchronises with the device (a blocking copy), so call it after the stream sync.
// clear != 0 also resets the word.  A negative value is an error (see
// mykb_noalloc_last_error).
int mykb_noalloc_status(int clear);

// Device address of the current device's status word (NULL on error), for callers that
// read it asynchronously into their own pinned memory.
void* mykb_noalloc_status_address(void);

#ifdef __cplusplus
}
#endif
