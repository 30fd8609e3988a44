"""The allocation-free FlashAttention backward C entry point (``mykb_flash_attn_bwd_noalloc``).

Some callers cannot allocate GPU memory: code running during CUDA-graph capture into a
pool it does not own, plugins and inference runtimes that only receive buffers from their
host framework, and processes whose memory is fixed up front.  This entry point takes
every input and output from the caller and keeps its working memory (Delta and a status
word) in fixed-size arrays inside the library.  The tests call the exported C symbol
through ctypes and check dq / dk / dv against the existing entry point (the one the
autograd op uses) on two calls in a row with different data, in both layouts (packed
documents and a plain batch), at head_dim 64 and 128, causal, non-causal and windowed;
that a status word left set by an earlier call does not spoil the next call; and that
inconsistent or oversized problems are rejected.

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
    status = lib.mykb_noalloc_status
    status.restype = ctypes.c_int
    status.argtypes = [ctypes.c_int]
    addr = lib.mykb_noalloc_status_address
    addr.restype = ctypes.c_void_p
    return fn, err, status, addr


def _close(a, b, tol=2e-2):
    e = (a.float() - b.float()).abs().max().item()
    s = b.float().abs().max().item() + 1e-6
    assert e <= tol * s, f"err {e} > {tol} * {s}"


class _Case:
    """Inputs of one backward problem and the existing entry point's dq / dk / dv."""

    def __init__(self, seed, lens, *, packed=True, h=4, kvh=2, d=64, left=-1, right=0):
        from myk_llm_b200.ops import ext

        g = torch.Generator(device="cuda").manual_seed(seed)
        self.h, self.kvh, self.d, self.left, self.right = h, kvh, d, left, right
        self.packed = packed
        self.max_len = max(lens)
        self.scale = 1.0 / math.sqrt(d)
        if packed:
            self.cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device="cuda")
            shape_q, shape_k = (int(self.cu[-1]), h, d), (int(self.cu[-1]), kvh, d)
            self.num_seqs = len(lens)
        else:
            self.cu = None
            shape_q, shape_k = (len(lens), self.max_len, h, d), (len(lens), self.max_len, kvh, d)
            self.num_seqs = len(lens)
        self.q = torch.randn(*shape_q, device="cuda", generator=g).bfloat16()
        self.k = torch.randn(*shape_k, device="cuda", generator=g).bfloat16()
        self.v = torch.randn(*shape_k, device="cuda", generator=g).bfloat16()
        self.do = torch.randn(*shape_q, device="cuda", generator=g).bfloat16()
        self.out, self.lse = ext().fa_fwd(self.q, self.k, self.v, self.cu, self.cu, None, self.max_len, self.max_len,
                                          self.scale, left, right)
        self.ref = ext().fa_bwd(self.do, self.q, self.k, self.v, self.out, self.lse, self.cu, self.cu, self.max_len,
                                self.max_len, self.scale, left, right)

    @property
    def rows_q(self):
        return self.q.numel() // (self.h * self.d)

    @property
    def rows_k(self):
        return self.k.numel() // (self.kvh * self.d)

    def call(self, fn, err, *, rows_q=None, rows_k=None, num_seqs=None):
        dq, dk, dv = torch.empty_like(self.q), torch.empty_like(self.k), torch.empty_like(self.v)
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(self.do.data_ptr(), self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.out.data_ptr(),
                self.lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                self.cu.data_ptr() if self.cu is not None else None,
                self.num_seqs if num_seqs is None else num_seqs,
                self.rows_q if rows_q is None else rows_q, self.rows_k if rows_k is None else rows_k,
                self.max_len, self.max_len, self.h, self.kvh, self.d, self.scale, self.left, self.right, stream)
        return rc, (dq, dk, dv)

    def check(self, fn, err, status):
        rc, got = self.call(fn, err)
        assert rc == 0, err().decode()
        torch.cuda.synchronize()
        assert status(1) == 0
        for a, b in zip(got, self.ref):
            _close(a, b)


_LAYOUTS = [
    # (packed, d, left, right)
    (True, 64, -1, 0),
    (True, 128, -1, 0),
    (True, 64, -1, -1),
    (True, 128, 96, 0),
    (False, 64, -1, 0),
    (False, 128, -1, -1),
    (False, 64, 200, 0),
]


@pytest.mark.parametrize("packed,d,left,right", _LAYOUTS)
def test_noalloc_matches_existing_entry_point_twice(packed, d, left, right):
    fn, err, status, _ = _lib()
    runs = [(0, [130, 7, 300]), (1, [64, 257, 128, 5])] if packed else [(0, [300, 300]), (1, [129, 129, 129])]
    for seed, lens in runs:
        _Case(seed, lens, packed=packed, d=d, left=left, right=right).check(fn, err, status)


def test_noalloc_status_left_set_does_not_spoil_the_next_call():
    """An earlier call whose wait gave up leaves a non-zero word; the next call clears it
    on its stream first, so its own waits run normally."""
    fn, err, status, addr = _lib()
    case = _Case(3, [200, 77])
    case.check(fn, err, status)  # first call on this device: also does the symbol lookup
    ptr = addr()
    assert ptr
    cudart = ctypes.CDLL("libcudart.so.12")
    word = ctypes.c_int(1234)
    assert cudart.cudaMemcpy(ctypes.c_void_p(ptr), ctypes.byref(word), ctypes.c_size_t(4), ctypes.c_int(1)) == 0
    assert status(0) == 1234  # the query sees the word without clearing it
    case.check(fn, err, status)  # still correct, and the word reads 0 after the call


def test_noalloc_rejects_oversized_problem():
    fn, err, _, _ = _lib()
    rows = (1 << 20) // 4 + 1  # rows * heads exceeds the built-in scratch
    rc = fn(0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, rows, rows, rows, rows, 4, 2, 64, 0.125, -1, 0, None)
    assert rc != 0
    assert b"exceeds" in err()


def test_noalloc_rejects_inconsistent_sizes():
    fn, err, _, _ = _lib()
    batch = _Case(4, [128, 128], packed=False)
    rc, _ = batch.call(fn, err, rows_q=batch.rows_q + 1, rows_k=batch.rows_k + 1)
    assert rc != 0 and b"num_seqs * max_q" in err()
    rc, _ = batch.call(fn, err, num_seqs=3)
    assert rc != 0 and b"num_seqs * max_q" in err()
    packed = _Case(5, [100, 50])
    rc, _ = packed.call(fn, err, rows_k=packed.rows_k - 10)
    assert rc != 0 and b"rows_k must equal rows_q" in err()
    torch.cuda.synchronize()
