"""tcgen05 GEMM vs an fp32 PyTorch reference, over operand layouts, ragged edges, batch,
fp32 output, epilogue C and split-K accumulation."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b, a_mn, b_mn):
    am = a.float().transpose(-1, -2) if a_mn else a.float()
    bm = b.float().transpose(-1, -2) if b_mn else b.float()
    return am @ bm.transpose(-1, -2)


def _mk(m, n, k, a_mn, b_mn, batch=None):
    g = torch.Generator(device="cuda").manual_seed(0)
    lead = (batch,) if batch else ()
    a = torch.randn(*lead, *((k, m) if a_mn else (m, k)), device="cuda", generator=g).bfloat16()
    b = torch.randn(*lead, *((k, n) if b_mn else (n, k)), device="cuda", generator=g).bfloat16()
    return a, b


def _close(out, ref, rel=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= rel * scale, f"max err {err} vs scale {scale}"


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("shape", [(128, 128, 64), (256, 384, 256), (264, 200, 136), (1024, 1536, 1024)])
def test_gemm_layouts(a_mn, b_mn, shape):
    from myk_llm_b200.ops import gemm

    m, n, k = shape
    a, b = _mk(m, n, k, a_mn, b_mn)
    out = gemm(a, b, a_major="mn" if a_mn else "k", b_major="mn" if b_mn else "k")
    torch.cuda.synchronize()
    _close(out, _ref(a, b, a_mn, b_mn))


def test_gemm_fp32_out_and_alpha():
    from myk_llm_b200.ops import gemm

    a, b = _mk(512, 256, 320, False, False)
    out = gemm(a, b, out_dtype=torch.float32, alpha=0.5)
    _close(out, 0.5 * _ref(a, b, False, False), rel=1e-2)


def test_gemm_accumulate_split_k():
    from myk_llm_b200.ops import gemm

    # few output tiles, long K: the kernel splits K and reduces with TMA reduce-add
    a, b = _mk(4096, 256, 384, True, True)  # a: (K=4096, M=256)... rows are the reduction
    a = torch.randn(8192, 256, device="cuda").bfloat16()  # (K, M)
    b = torch.randn(8192, 384, device="cuda").bfloat16()  # (K, N)
    d = torch.randn(256, 384, device="cuda")
    base = d.clone()
    gemm(a, b, a_major="mn", b_major="mn", out=d, accumulate=True)
    _close(d, base + a.float().t() @ b.float(), rel=1e-2)


def test_gemm_batched_with_c():
    from myk_llm_b200.ops import gemm

    a, b = _mk(192, 192, 256, False, False, batch=3)
    c = torch.randn(3, 192, 192, device="cuda").bfloat16()
    out = gemm(a, b, alpha=2.0, beta=-0.5, c=c)
    _close(out, 2.0 * _ref(a, b, False, False) - 0.5 * c.float())


def test_linear_autograd_matches_reference():
    from myk_llm_b200.ops import linear

    torch.manual_seed(0)
    x = torch.randn(4, 96, 256, device="cuda", requires_grad=True)
    w = torch.randn(384, 256, device="cuda", requires_grad=True)
    y = linear(x, w)
    y.float().square().sum().backward()
    xr = x.detach().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    yr = xr.bfloat16().float() @ wr.bfloat16().float().t()
    yr.square().sum().backward()
    _close(y, yr)
    _close(x.grad, xr.grad, rel=3e-2)
    _close(w.grad, wr.grad, rel=3e-2)


@pytest.mark.parametrize("m", [1, 3, 17, 64, 100, 192, 256])
@pytest.mark.parametrize("nk", [(64, 64), (1000, 1000), (1536, 1024), (1024, 2816), (65536, 256)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_skinny_gemm(m, nk, out_dtype):
    """Split-K skinny GEMM (decode rows) against fp32, twice in a row (the split-K tickets
    must be left at zero)."""
    from myk_llm_b200.ops import ext

    n, k = nk
    a, b = _mk(m, n, k, False, False)
    ref = _ref(a, b, False, False)
    for _ in range(2):
        out = torch.empty(m, n, dtype=out_dtype, device="cuda")
        ext().gemm_skinny(a, b, out)
        torch.cuda.synchronize()
        _close(out, ref)


def test_linear_uses_skinny_rows():
    from myk_llm_b200.ops import linear

    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(2, 3, 512, device="cuda", generator=g).bfloat16()
    w = torch.randn(768, 512, device="cuda", generator=g)
    _close(linear(x, w), x.float() @ w.bfloat16().float().t())


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,batch", [(128, 256, 1), (312, 512, 2), (1024, 1536, 3), (2048, 640, 1)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_symmetric_gemm_matches_full(m, k, batch, out_dtype):
    """Symmetric mode (X X^T, and a symmetric product with a symmetric C) skips the tiles above
    the diagonal and mirrors the lower triangle: it must equal the full product."""
    from myk_llm_b200.ops import gemm

    torch.manual_seed(m + k)
    x = torch.randn(batch, m, k, device="cuda").bfloat16()
    full = gemm(x, x, out_dtype=out_dtype)
    sym = gemm(x, x, out_dtype=out_dtype, symmetric=True)
    ref = x.float() @ x.float().transpose(-1, -2)
    assert torch.equal(sym, sym.transpose(-1, -2))
    tol = 2e-2 if out_dtype == torch.bfloat16 else 1e-3
    assert ((sym.float() - ref).abs().max() / ref.abs().max()) < tol
    lower = torch.tril(torch.ones(m, m, device="cuda", dtype=torch.bool))
    assert torch.equal(sym[:, lower], full[:, lower])
    g = sym if out_dtype == torch.bfloat16 else sym.bfloat16()
    poly = gemm(g, g, alpha=0.5, beta=-1.5, c=g, symmetric=True)
    poly_ref = 0.5 * (g.float() @ g.float()) - 1.5 * g.float()
    assert torch.equal(poly, poly.transpose(-1, -2))
    assert ((poly.float() - poly_ref).abs().max() / poly_ref.abs().max()) < 2e-2


def test_gemm_rejects_layouts_tma_cannot_move():
    """Rows that are not a multiple of 16 bytes are refused with a clear error up front."""
    from myk_llm_b200.ops import gemm

    x = torch.randn(2, 300, 64, device="cuda").bfloat16()
    with pytest.raises(ValueError):
        gemm(x, x)  # output rows of 300 bf16 = 600 bytes
