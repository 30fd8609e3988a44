"""FlashAttention kernels vs the fp32 masked-softmax reference: forward output and
q/k/v gradients over partial tiles, GQA, sliding windows, bidirectional attention,
Lq < Lk (decode) and Lq > Lk (empty rows), packed documents and static KV caches.
Tolerance: 2% of max |reference| (the reference test's criterion)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(out, ref, tol=2e-2):
    err = (out.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item() + 1e-6
    assert err <= tol * scale, f"err {err} > {tol} * {scale}"


CASES = [
    # (batch, lq, lk, heads, kv_heads, d, causal, window)
    (2, 128, 128, 2, 1, 64, True, (-1, -1)),
    (2, 200, 200, 4, 2, 64, True, (-1, -1)),
    (1, 333, 333, 4, 1, 128, True, (-1, -1)),
    (2, 300, 300, 2, 2, 64, True, (63, 0)),
    (1, 257, 257, 2, 1, 64, False, (-1, -1)),
    (2, 16, 300, 4, 2, 64, True, (-1, -1)),
    (2, 300, 100, 2, 1, 64, True, (-1, -1)),
    (1, 512, 512, 2, 1, 128, True, (127, 0)),
    (1, 100, 260, 2, 2, 128, False, (50, 30)),
    # several work items per CTA, many KV tiles, two head pairs per KV head
    (2, 1100, 1100, 8, 2, 64, True, (-1, -1)),
    (1, 700, 700, 16, 4, 128, True, (300, 0)),
]


@pytest.mark.parametrize("case", CASES)
def test_flash_attn_dense(case):
    from myk_llm_b200.ops import flash_attn_func
    from myk_llm_b200.ops.reference import attention_ref

    b, lq, lk, h, kvh, d, causal, window = case
    torch.manual_seed(0)
    q = torch.randn(b, lq, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(b, lk, kvh, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(b, lk, kvh, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    out = flash_attn_func(q, k, v, causal=causal, window_size=window)
    g = torch.randn_like(out)
    (out.float() * g.float()).sum().backward()
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    left, right = window
    right = 0 if causal else right
    ref, _ = attention_ref(qr, kr, vr, causal=causal, window=(left, right))
    (ref.float() * g.float()).sum().backward()
    from myk_llm_b200.ops import ext

    assert ext().take_status() == 0
    _close(out, ref)
    _close(q.grad, qr.grad)
    _close(k.grad, kr.grad)
    _close(v.grad, vr.grad)


@pytest.mark.parametrize("d", [64, 128])
def test_flash_attn_varlen_documents(d):
    from myk_llm_b200.ops import flash_attn_varlen_func
    from myk_llm_b200.ops.reference import attention_varlen_ref

    torch.manual_seed(1)
    lens = [1, 130, 77, 256, 3, 300]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device="cuda")
    t = int(cu[-1])
    h, kvh = 4, 2
    q = torch.randn(t, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(t, kvh, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(t, kvh, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    out = flash_attn_varlen_func(q, k, v, cu, cu, max(lens), max(lens), causal=True)
    g = torch.randn_like(out)
    (out.float() * g.float()).sum().backward()
    qr, kr, vr = (x.detach().float().requires_grad_(True) for x in (q, k, v))
    ref, _ = attention_varlen_ref(qr, kr, vr, cu, cu, causal=True)
    (ref * g.float()).sum().backward()
    _close(out, ref)
    _close(q.grad, qr.grad)
    _close(k.grad, kr.grad)
    _close(v.grad, vr.grad)
    # documents never mix: each document alone gives the same rows
    s, e = int(cu[3]), int(cu[4])
    alone = flash_attn_varlen_func(q[s:e].detach(), k[s:e].detach(), v[s:e].detach(),
                                   torch.tensor([0, e - s], dtype=torch.int32, device="cuda"),
                                   torch.tensor([0, e - s], dtype=torch.int32, device="cuda"), e - s, e - s, causal=True)
    _close(alone, out[s:e].detach(), 1e-2)


def test_flash_attn_strided_qkv_view():
    """q/k/v as views into one fused projection output (no copies)."""
    from myk_llm_b200.ops import flash_attn_func
    from myk_llm_b200.ops.reference import attention_ref

    torch.manual_seed(2)
    b, l, h, kvh, d = 2, 190, 4, 1, 64
    qkv = torch.randn(b, l, (h + 2 * kvh) * d, device="cuda", dtype=torch.bfloat16)
    q, k, v = qkv.split([h * d, kvh * d, kvh * d], dim=-1)
    q, k, v = q.view(b, l, h, d), k.view(b, l, kvh, d), v.view(b, l, kvh, d)
    out = flash_attn_func(q, k, v, causal=True)
    ref, _ = attention_ref(q.float(), k.float(), v.float(), causal=True, window=(-1, 0))
    _close(out, ref)


def test_flash_attn_with_kvcache():
    from myk_llm_b200.ops import flash_attn_with_kvcache
    from myk_llm_b200.ops.reference import attention_ref

    torch.manual_seed(3)
    b, cap, h, kvh, d = 3, 400, 4, 2, 64
    kc = torch.zeros(b, cap, kvh, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    lens = torch.tensor([5, 130, 257], device="cuda", dtype=torch.int32)
    for i, n in enumerate(lens.tolist()):
        kc[i, :n] = torch.randn(n, kvh, d, device="cuda").bfloat16()
        vc[i, :n] = torch.randn(n, kvh, d, device="cuda").bfloat16()
    q = torch.randn(b, 3, h, d, device="cuda", dtype=torch.bfloat16)
    kn = torch.randn(b, 3, kvh, d, device="cuda", dtype=torch.bfloat16)
    vn = torch.randn(b, 3, kvh, d, device="cuda", dtype=torch.bfloat16)
    out = flash_attn_with_kvcache(q, kc, vc, kn, vn, cache_seqlens=lens, causal=True)
    for i, n in enumerate(lens.tolist()):
        kk = kc[i:i + 1, : n + 3].float()
        vv = vc[i:i + 1, : n + 3].float()
        ref, _ = attention_ref(q[i:i + 1].float(), kk, vv, causal=True, window=(-1, 0))
        _close(out[i:i + 1], ref)


@pytest.mark.parametrize("d,h,kvh,new", [(64, 16, 4, 3), (128, 16, 4, 1), (128, 8, 8, 3), (64, 4, 1, 4)])
@pytest.mark.parametrize("left", [-1, 100])
def test_split_kv_decode_matches_reference(d, h, kvh, new, left):
    """The split-KV decode kernel (taken by flash_attn_with_kvcache for decode-sized
    steps) against the fp32 reference, including ragged lengths and a sliding window."""
    from myk_llm_b200.ops import ext, flash_attn_with_kvcache
    from myk_llm_b200.ops.reference import attention_ref

    torch.manual_seed(5)
    b, cap = 4, 2400
    kc = torch.randn(b, cap, kvh, d, device="cuda").bfloat16()
    vc = torch.randn(b, cap, kvh, d, device="cuda").bfloat16()
    lens = torch.tensor([0, 70, 1000, 2300], device="cuda", dtype=torch.int32)
    q = torch.randn(b, new, h, d, device="cuda", dtype=torch.bfloat16)
    kn = torch.randn(b, new, kvh, d, device="cuda", dtype=torch.bfloat16)
    vn = torch.randn(b, new, kvh, d, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):  # twice: the merge tickets must be left at zero
        kc2, vc2 = kc.clone(), vc.clone()
        out = flash_attn_with_kvcache(q, kc2, vc2, kn, vn, cache_seqlens=lens, causal=True, window_size=(left, 0))
        torch.cuda.synchronize()
        for i, n in enumerate(lens.tolist()):
            assert torch.equal(kc2[i, n:n + new], kn[i]) and torch.equal(vc2[i, n:n + new], vn[i])
            ref, _ = attention_ref(q[i:i + 1].float(), kc2[i:i + 1, :n + new].float(), vc2[i:i + 1, :n + new].float(),
                                   causal=True, window=(left, 0))
            _close(out[i:i + 1], ref)
    assert ext().take_status() == 0
