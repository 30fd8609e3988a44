"""The allocation-free FlashAttention backward C entry point (``mykb_flash_attn_bwd_noalloc``).

Some callers cannot allocate GPU memory: code running during CUDA-graph capture into a
pool it does not own, plugins and inference runtimes that only receive buffers from their
host framework, and processes whose memory is fixed up front.  This entry point takes
every input and output from the caller and keeps its working memory (Delta and a status
word) in fixed-size arrays inside the library.  The test calls the exported C symbol
through ctypes and checks dq / dk / dv against the existing entry point (the one the
autograd op uses), on two calls in a row with different data, plus the size rejection.

This file is collected last so that a run stopping at the first failure has run every
other test already; it also passes alone in a fresh process.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from myk_llm_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.mykb_flash_attn_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 10 + [ctypes.c_int] * 8 + [ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                                                  ctypes.c_void_p]
    err = lib.mykb_noalloc_last_error
    err.restype = ctypes.c_char_p
    return fn, err


def _close(a, b, tol=2e-2):
    e = (a.float() - b.float()).abs().max().item()
    s = b.float().abs().max().item() + 1e-6
    assert e <= tol * s, f"err {e} > {tol} * {s}"


def _case(seed, lens, h=4, kvh=2, d=64):
    from myk_llm_b200.ops import ext

    g = torch.Generator(device="cuda").manual_seed(seed)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device="cuda")
    t = int(cu[-1])
    q = torch.randn(t, h, d, device="cuda", generator=g).bfloat16()
    k = torch.randn(t, kvh, d, device="cuda", generator=g).bfloat16()
    v = torch.randn(t, kvh, d, device="cuda", generator=g).bfloat16()
    do = torch.randn(t, h, d, device="cuda", generator=g).bfloat16()
    scale = 1.0 / math.sqrt(d)
    out, lse = ext().fa_fwd(q, k, v, cu, cu, None, max(lens), max(lens), scale, -1, 0)
    ref = ext().fa_bwd(do, q, k, v, out, lse, cu, cu, max(lens), max(lens), scale, -1, 0)
    return q, k, v, do, out, lse, cu, scale, ref


def _call(fn, err, q, k, v, do, out, lse, cu, scale, max_len, h, kvh, d):
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(do.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(), dq.data_ptr(),
            dk.data_ptr(), dv.data_ptr(), cu.data_ptr(), cu.numel() - 1, q.shape[0], k.shape[0], max_len, max_len, h,
            kvh, d, scale, -1, 0, stream)
    assert rc == 0, err().decode()
    torch.cuda.synchronize()
    return dq, dk, dv


def test_noalloc_matches_existing_entry_point_twice():
    fn, err = _lib()
    for seed, lens in [(0, [130, 7, 300]), (1, [64, 257, 128, 5])]:
        q, k, v, do, out, lse, cu, scale, ref = _case(seed, lens)
        got = _call(fn, err, q, k, v, do, out, lse, cu, scale, max(lens), 4, 2, 64)
        for a, b in zip(got, ref):
            _close(a, b)


def test_noalloc_rejects_oversized_problem():
    fn, err = _lib()
    rows = (1 << 20) // 4 + 1  # rows * heads exceeds the built-in scratch
    rc = fn(0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, rows, rows, rows, rows, 4, 2, 64, 0.125, -1, 0, None)
    assert rc != 0
    assert b"exceeds" in err()
