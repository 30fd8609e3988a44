"""FlashAttention on tcgen05: causal / bidirectional, sliding window, GQA, packed varlen,
static KV-cache decode.

API and semantics follow the reference's Triton FlashAttention
(``src/myk_llm/ops/flash_attn.py:442-489``): queries are aligned to the end of the keys,
``window_size=(left, right)`` with -1 meaning unbounded, rows with no visible key output
0 (and an LSE of +inf), ``flash_attn_with_kvcache`` writes the new keys/values into a
static cache at ``cache_seqlens[b]`` before attending (no host sync, so it can be captured
in a CUDA graph).

The kernels (``csrc/attention.cu``) keep S and the P·V product in tensor memory, stage
K/V tiles with TMA (plain loads of local memory) and write the output plus a natural-log LSE.  The
backward pass computes dK/dV per key tile and accumulates dQ in fp32.
"""

from __future__ import annotations

import math

import torch

from . import reference as ref
from ._ext import ext

SUPPORTED_HEAD_DIMS = (64, 128)
# KV-cache steps whose (query heads per KV head) x new tokens fit one 16-row MMA tile take
# the split-KV decode kernel (keys spread over CTAs, partials merged by the last one).
DECODE_MAX_ROWS = 16


def _window(causal: bool, window_size: tuple[int, int]) -> tuple[int, int]:
    left, right = window_size
    left = -1 if left < 0 else left
    right = 0 if causal else (-1 if right < 0 else right)
    return left, right


def _check(q, k, v):
    d = q.shape[-1]
    if q.dtype not in (torch.bfloat16,) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"flash attention needs bf16 q, k, v; got {q.dtype}, {k.dtype}, {v.dtype}")
    if d not in SUPPORTED_HEAD_DIMS or k.shape[-1] != d or v.shape[-1] != d:
        raise ValueError(f"head_dim must be one of {SUPPORTED_HEAD_DIMS}; got {q.shape[-1]}, {k.shape[-1]}, {v.shape[-1]}")
    if q.shape[-2] % k.shape[-2] or k.shape[-2] != v.shape[-2]:
        raise ValueError(f"query heads ({q.shape[-2]}) must be a multiple of key/value heads ({k.shape[-2]})")


def _inner(x):
    return x if x.stride(-1) == 1 else x.contiguous()


class _FlashAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_q, cu_k, max_q, max_k, scale, left, right):
        o, lse = ext().fa_fwd(q, k, v, cu_q, cu_k, None, int(max_q), int(max_k), float(scale), int(left), int(right))
        ctx.save_for_backward(q, k, v, o, lse, cu_q, cu_k)
        ctx.args = (int(max_q), int(max_k), float(scale), int(left), int(right))
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, cu_q, cu_k = ctx.saved_tensors
        max_q, max_k, scale, left, right = ctx.args
        dq, dk, dv = ext().fa_bwd(_inner(do), q, k, v, o, lse, cu_q, cu_k, max_q, max_k, scale, left, right)
        return dq, dk, dv, None, None, None, None, None, None, None


def flash_attn_func(q, k, v, causal: bool = False, window_size=(-1, -1), softmax_scale=None):
    """q (batch, Lq, heads, d), k/v (batch, Lk, kv_heads, d)."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    left, right = _window(causal, window_size)
    if not q.is_cuda:
        out, _ = ref.attention_ref(q, k, v, causal=causal, window=(left, right), softmax_scale=scale)
        return out
    _check(q, k, v)
    q, k, v = _inner(q), _inner(k), _inner(v)
    return _FlashAttn.apply(q, k, v, None, None, q.shape[1], k.shape[1], scale, left, right)


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, causal: bool = False,
                           window_size=(-1, -1), softmax_scale=None):
    """Packed q (total_q, heads, d), k/v (total_k, kv_heads, d); document b spans rows
    cu_seqlens[b]:cu_seqlens[b+1]."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    left, right = _window(causal, window_size)
    if not q.is_cuda:
        out, _ = ref.attention_varlen_ref(q, k, v, cu_seqlens_q, cu_seqlens_k, causal=causal, window=(left, right),
                                          softmax_scale=scale)
        return out
    _check(q, k, v)
    q, k, v = _inner(q), _inner(k), _inner(v)
    return _FlashAttn.apply(q, k, v, cu_seqlens_q.int(), cu_seqlens_k.int(), max_seqlen_q, max_seqlen_k, scale,
                            left, right)


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, *, cache_seqlens, causal: bool = False,
                            window_size=(-1, -1), softmax_scale=None):
    """Append k/v (batch, new, kv_heads, d) to static caches (batch, capacity, kv_heads, d)
    at ``cache_seqlens[b]``, then attend q over ``cache_seqlens[b] + new`` keys.  The
    caller advances ``cache_seqlens``.  Forward only."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    left, right = _window(causal, window_size)
    seqused = cache_seqlens if cache_seqlens.dtype == torch.int32 else cache_seqlens.to(torch.int32)
    if k is not None and v is not None:
        bsz, new = k.shape[:2]
        if k.is_cuda and k_cache.is_contiguous() and v_cache.is_contiguous():
            ext().kv_append(k_cache, v_cache, k, v, seqused)
        else:
            rows = torch.arange(bsz, device=k.device)[:, None]
            cols = cache_seqlens.long()[:, None] + torch.arange(new, device=k.device)
            k_cache[rows, cols] = k
            v_cache[rows, cols] = v
        seqused = seqused + new
    if not q.is_cuda:
        out, _ = ref.attention_ref(q, k_cache, v_cache, causal=causal, window=(left, right), softmax_scale=scale,
                                   seqused_k=seqused)
        return out
    _check(q, k_cache, v_cache)
    q = _inner(q)
    if (q.shape[2] // k_cache.shape[2]) * q.shape[1] <= DECODE_MAX_ROWS and k_cache.is_contiguous() \
            and v_cache.is_contiguous() and q.stride(2) % 8 == 0 and q.stride(1) % 8 == 0:
        return ext().fa_decode(q, k_cache, v_cache, seqused, float(scale), left, right)
    o, _ = ext().fa_fwd(q, k_cache, v_cache, None, None, seqused, q.shape[1], k_cache.shape[1], float(scale),
                        left, right)
    return o
