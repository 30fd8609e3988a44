"""Memory-bound kernels (RMSNorm, add+RMSNorm, gated norm, SwiGLU, RoPE, embedding, CE,
AdamW, Muon prep/apply) vs their fp32 PyTorch statements."""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _close(a, b, tol):
    err = (a.float() - b.float()).abs().max().item()
    scale = b.float().abs().max().item() + 1e-6
    assert err <= tol * scale, f"err {err} scale {scale}"


@pytest.mark.parametrize("hidden", [64, 128, 1024, 2048])
@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16])
def test_rmsnorm_fwd_bwd(hidden, xdt):
    from myk_llm_b200 import ops

    if hidden == 64 and xdt == torch.float32:
        pytest.skip("width-64 norms run on bf16 q/k heads only")
    torch.manual_seed(0)
    x = torch.randn(333, hidden, device="cuda", dtype=xdt, requires_grad=True)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda")).requires_grad_(True)
    y = ops.rms_norm(x, w, 1e-6, out_dtype=torch.bfloat16)
    g = torch.randn_like(y)
    (y.float() * g.float()).sum().backward()
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    (yr * g.float()).sum().backward()
    _close(y, yr, 1e-2)
    _close(x.grad, xr.grad, 2e-2)
    _close(w.grad, wr.grad, 2e-2)


def test_add_rmsnorm():
    from myk_llm_b200 import ops

    torch.manual_seed(1)
    x = torch.randn(257, 1024, device="cuda", requires_grad=True)
    u = torch.randn(257, 1024, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(1024, device="cuda", requires_grad=True)
    s, y = ops.add_rms_norm(x, u, w, 1e-6, out_dtype=torch.bfloat16)
    gs, gy = torch.randn_like(s), torch.randn_like(y)
    ((s * gs).sum() + (y.float() * gy.float()).sum()).backward()
    xr, ur, wr = (t.detach().float().requires_grad_(True) for t in (x, u, w))
    sr = xr + ur
    yr = sr * torch.rsqrt(sr.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    ((sr * gs).sum() + (yr * gy.float()).sum()).backward()
    _close(s, sr, 1e-5)
    _close(y, yr, 1e-2)
    _close(x.grad, xr.grad, 2e-2)
    _close(u.grad, ur.grad, 2e-2)
    _close(w.grad, wr.grad, 2e-2)


@pytest.mark.parametrize("act", ["swish", "sigmoid"])
@pytest.mark.parametrize("width", [64, 128])
def test_gated_rmsnorm(act, width):
    from myk_llm_b200 import ops
    from myk_llm_b200.ops import reference as ref

    torch.manual_seed(2)
    o = torch.randn(64, 3, width, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    g = torch.randn(64, 3, width, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(width, device="cuda", requires_grad=True)
    y = ops.gated_rms_norm(o, g, w, 1e-5, act)
    gy = torch.randn_like(y)
    (y.float() * gy.float()).sum().backward()
    orf, grf, wrf = (t.detach().float().requires_grad_(True) for t in (o, g, w))
    yr = ref.gated_rms_norm_ref(orf, grf, wrf, 1e-5, act)
    (yr * gy.float()).sum().backward()
    _close(y, yr, 2e-2)
    _close(o.grad, orf.grad, 3e-2)
    _close(g.grad, grf.grad, 3e-2)
    _close(w.grad, wrf.grad, 3e-2)


def test_swiglu():
    from myk_llm_b200 import ops

    torch.manual_seed(3)
    gu = torch.randn(100, 2 * 704, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    a = ops.swiglu(gu)
    ga = torch.randn_like(a)
    (a.float() * ga.float()).sum().backward()
    r = gu.detach().float().requires_grad_(True)
    g, u = r.chunk(2, -1)
    ar = F.silu(g) * u
    (ar * ga.float()).sum().backward()
    _close(a, ar, 1e-2)
    _close(gu.grad, r.grad, 2e-2)


def test_rope_strided_and_inverse():
    from myk_llm_b200 import ops
    from myk_llm_b200.models.layers import RotaryEmbedding

    torch.manual_seed(4)
    rope = RotaryEmbedding(64, 512, 10000.0).cuda()
    qkv = torch.randn(2, 77, 6 * 64, device="cuda", dtype=torch.bfloat16)
    q = qkv[..., : 4 * 64].view(2, 77, 4, 64)  # strided view into the fused projection
    pos = torch.arange(77, device="cuda").expand(2, -1) + 5
    y = ops.apply_rope(q, rope.cos_cached, rope.sin_cached, pos)
    c = rope.cos_cached[pos].unsqueeze(2)
    s = rope.sin_cached[pos].unsqueeze(2)
    from myk_llm_b200.ops.reference import rope_ref

    _close(y, rope_ref(q.float(), c, s), 1e-2)
    q2 = q.detach().clone().requires_grad_(True)
    y2 = ops.apply_rope(q2, rope.cos_cached, rope.sin_cached, pos)
    gy = torch.randn_like(y2)
    (y2.float() * gy.float()).sum().backward()
    qr = q.detach().float().requires_grad_(True)
    (rope_ref(qr, c, s) * gy.float()).sum().backward()
    _close(q2.grad, qr.grad, 2e-2)


@pytest.mark.parametrize("d,heads,kv", [(64, 4, 2), (128, 8, 2)])
def test_fused_qkv_rope_matches_split_reference(d, heads, kv):
    from myk_llm_b200 import ops
    from myk_llm_b200.models.layers import RotaryEmbedding
    from myk_llm_b200.ops.reference import rope_ref

    torch.manual_seed(5)
    rope = RotaryEmbedding(d, 512, 10000.0).cuda()
    width = (heads + 2 * kv) * d
    # a strided row view (as a slice of a wider buffer) exercises the row stride
    base = torch.randn(3, 45, width + 64, device="cuda", dtype=torch.bfloat16)
    qkv = base[..., :width].detach().requires_grad_(True)
    pos = torch.randint(0, 500, (3, 45), device="cuda")
    q, k, v = ops.rope_qkv(qkv, rope.cos_cached, rope.sin_cached, pos, heads, kv)
    assert q.is_contiguous() and k.is_contiguous() and v.is_contiguous()
    gq, gk, gv = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    (q.float() * gq.float()).sum().add_((k.float() * gk.float()).sum()).add_((v.float() * gv.float()).sum()).backward()
    ref = qkv.detach().float().requires_grad_(True)
    rq, rk, rv = ref.split((heads * d, kv * d, kv * d), dim=-1)
    c = rope.cos_cached[pos].unsqueeze(2)
    s = rope.sin_cached[pos].unsqueeze(2)
    rq = rope_ref(rq.reshape(3, 45, heads, d), c, s)
    rk = rope_ref(rk.reshape(3, 45, kv, d), c, s)
    rv = rv.reshape(3, 45, kv, d)
    _close(q, rq, 1e-2)
    _close(k, rk, 1e-2)
    assert torch.equal(v.float(), rv)
    ((rq * gq.float()).sum() + (rk * gk.float()).sum() + (rv * gv.float()).sum()).backward()
    _close(qkv.grad, ref.grad, 2e-2)


def test_embedding():
    from myk_llm_b200 import ops

    w = torch.randn(1000, 128, device="cuda", requires_grad=True)
    ids = torch.randint(0, 1000, (4, 33), device="cuda")
    out = ops.embedding(ids, w)
    g = torch.randn_like(out)
    (out * g).sum().backward()
    wr = w.detach().clone().requires_grad_(True)
    (F.embedding(ids, wr) * g).sum().backward()
    _close(out, F.embedding(ids, w.detach()), 1e-6)
    _close(w.grad, wr.grad, 1e-5)


@pytest.mark.parametrize("z", [0.0, 1e-4])
def test_fused_linear_ce(z):
    from myk_llm_b200.ops import fused_linear_cross_entropy
    from myk_llm_b200.ops.reference import linear_cross_entropy_ref

    torch.manual_seed(5)
    n, h, v = 1000, 256, 4096
    hid = (0.5 * torch.randn(n, h, device="cuda")).bfloat16().requires_grad_(True)
    w = (0.05 * torch.randn(v, h, device="cuda")).requires_grad_(True)
    t = torch.randint(0, v, (n,), device="cuda")
    t[::7] = -100
    norm = float((t != -100).sum())
    loss, ce, zs = fused_linear_cross_entropy(hid, w, t, norm, z, chunk_size=384)
    loss.backward()
    hr = hid.detach().float().requires_grad_(True)
    wr = w.detach().bfloat16().float().requires_grad_(True)
    lr_, cer, zr = linear_cross_entropy_ref(hr, wr, t, norm, z)
    lr_.backward()
    assert abs(loss.item() - lr_.item()) < 2e-2 * abs(lr_.item())
    assert abs(ce.item() - cer.item()) < 2e-2 * abs(cer.item())
    _close(hid.grad, hr.grad, 5e-2)
    _close(w.grad, wr.grad, 5e-2)


def test_fused_linear_ce_scaled_backward_and_main_grad_check():
    from myk_llm_b200.ops import fused_linear_cross_entropy
    from myk_llm_b200.ops.loss import check_unscaled_main_grad
    from myk_llm_b200.ops.reference import linear_cross_entropy_ref

    torch.manual_seed(6)
    n, h, v = 512, 128, 2048
    hid = (0.5 * torch.randn(n, h, device="cuda")).bfloat16().requires_grad_(True)
    w = (0.05 * torch.randn(v, h, device="cuda")).requires_grad_(True)
    t = torch.randint(0, v, (n,), device="cuda")
    loss, _, _ = fused_linear_cross_entropy(hid, w, t, float(n))
    (3.0 * loss).backward()  # a scaled loss: both gradients carry the factor
    hr = hid.detach().float().requires_grad_(True)
    wr = w.detach().bfloat16().float().requires_grad_(True)
    (3.0 * linear_cross_entropy_ref(hr, wr, t, float(n), 0.0)[0]).backward()
    _close(hid.grad, hr.grad, 5e-2)
    _close(w.grad, wr.grad, 5e-2)
    # with a main_grad buffer the weight gradient is added during forward: only an
    # unscaled backward is right, and a scaled one is reported at the next check
    w2 = w.detach().clone().requires_grad_(True)
    w2.main_grad = torch.zeros_like(w2)
    loss2, _, _ = fused_linear_cross_entropy(hid.detach().requires_grad_(True), w2, t, float(n))
    loss2.backward()
    check_unscaled_main_grad()
    _close(w2.main_grad, wr.grad / 3.0, 5e-2)
    loss3, _, _ = fused_linear_cross_entropy(hid.detach().requires_grad_(True), w2, t, float(n))
    (2.0 * loss3).backward()
    with pytest.raises(RuntimeError):
        check_unscaled_main_grad()
    check_unscaled_main_grad()  # the report clears the counter


def test_adamw_multi_tensor():
    from myk_llm_b200.ops import adamw_multi_tensor
    from myk_llm_b200.ops.reference import adamw_ref

    torch.manual_seed(6)
    shapes = [(1000,), (37, 91), (4096, 8), (5,)]
    ps = [torch.randn(s, device="cuda") for s in shapes]
    gs = [torch.randn(s, device="cuda") for s in shapes]
    ms = [torch.randn(s, device="cuda").abs() for s in shapes]
    vs = [torch.randn(s, device="cuda").abs() for s in shapes]
    ref = [[t.clone() for t in ts] for ts in (ps, gs, ms, vs)]
    adamw_multi_tensor(ps, gs, ms, vs, 3, 1e-3, 0.9, 0.95, 1e-8, 0.1)
    for i in range(len(shapes)):
        adamw_ref(ref[0][i], ref[1][i], ref[2][i], ref[3][i], 3, 1e-3, 0.9, 0.95, 1e-8, 0.1)
        _close(ps[i], ref[0][i], 1e-5)
        _close(ms[i], ref[2][i], 1e-5)
        _close(vs[i], ref[3][i], 1e-5)


def test_newton_schulz_matches_reference():
    from myk_llm_b200.ops import batched_newton_schulz_orthogonalize
    from myk_llm_b200.ops.reference import newton_schulz_ref

    torch.manual_seed(7)
    for shape in [(4, 256, 512), (3, 512, 256), (2, 384, 384)]:
        g = torch.randn(*shape, device="cuda")
        out = batched_newton_schulz_orthogonalize(g, 5)
        ref = newton_schulz_ref(g, 5)
        _close(out, ref, 6e-2)


def test_optimizer_kernels_apply_device_grad_scale():
    from myk_llm_b200.ops import adamw_multi_tensor, muon_prepare

    torch.manual_seed(9)
    scale = torch.tensor(0.37, device="cuda")
    ps = [torch.randn(s, device="cuda") for s in [(1000,), (37, 91)]]
    gs = [torch.randn_like(p) for p in ps]
    ms = [torch.randn_like(p).abs() for p in ps]
    vs = [torch.randn_like(p).abs() for p in ps]
    a = [[t.clone() for t in ts] for ts in (ps, ms, vs)]
    b = [[t.clone() for t in ts] for ts in (ps, ms, vs)]
    adamw_multi_tensor(a[0], gs, a[1], a[2], 3, 1e-2, 0.9, 0.95, 1e-8, 0.1, grad_scale=scale)
    adamw_multi_tensor(b[0], [g * scale for g in gs], b[1], b[2], 3, 1e-2, 0.9, 0.95, 1e-8, 0.1)
    for x, y in zip(a[0] + a[1] + a[2], b[0] + b[1] + b[2]):
        assert torch.allclose(x, y, atol=1e-6, rtol=1e-5)
    g2 = [torch.randn(64, 96, device="cuda") for _ in range(3)]
    m1 = [torch.randn(64, 96, device="cuda") for _ in range(3)]
    m2 = [m.clone() for m in m1]
    o1 = torch.empty(3, 64, 96, device="cuda", dtype=torch.bfloat16)
    o2 = torch.empty_like(o1)
    muon_prepare(g2, m1, 0.95, True, o1, grad_scale=scale)
    muon_prepare([g * scale for g in g2], m2, 0.95, True, o2)
    assert torch.equal(o1, o2)
    for x, y in zip(m1, m2):
        assert torch.allclose(x, y, atol=1e-6)


def test_split_cols_and_strided_linear():
    from myk_llm_b200 import ops

    torch.manual_seed(10)
    base = torch.randn(2, 300, 96 + 64 + 32 + 8, device="cuda", dtype=torch.bfloat16)
    x = base[..., :192].detach().requires_grad_(True)  # strided rows
    a, b, c = ops.split_cols(x, (96, 64, 32))
    assert a.is_contiguous() and b.shape == (2, 300, 64)
    ra, rb, rc = x.detach().split((96, 64, 32), dim=-1)
    assert torch.equal(a, ra) and torch.equal(b, rb) and torch.equal(c, rc)
    ga, gb, gc = torch.randn_like(a), torch.randn_like(b), torch.randn_like(c)
    ((a.float() * ga.float()).sum() + (b.float() * gb.float()).sum() + (c.float() * gc.float()).sum()).backward()
    assert torch.equal(x.grad, torch.cat([ga, gb, gc], -1))
    # a linear reading a column slice of a wider activation (strided rows, no copy)
    w = (0.05 * torch.randn(128, 64, device="cuda")).requires_grad_(True)
    xs = base[..., 96:160].detach().requires_grad_(True)
    y = ops.linear(xs, w)
    gy = torch.randn_like(y)
    (y.float() * gy.float()).sum().backward()
    xr = xs.detach().float().requires_grad_(True)
    wr = w.detach().bfloat16().float().requires_grad_(True)
    yr = xr @ wr.t()
    (yr * gy.float()).sum().backward()
    _close(y, yr, 1e-2)
    _close(xs.grad, xr.grad, 2e-2)
    _close(w.grad, wr.grad, 2e-2)


def test_fused_ngram_embedding_matches_statement():
    """Hash + gather + sum in one kernel: the same rows as the integer-op statement of the
    bucket function, the same sums, and the scatter-add backward into every order's
    gradient rows (also with left context from a prefix)."""
    import torch.nn as nn

    from myk_llm_b200.models.embeddings import NgramEmbedding
    from myk_llm_b200.models.config import NgramEmbeddingConfig

    torch.manual_seed(0)
    cfg = NgramEmbeddingConfig(orders=[2, 3, 4], num_buckets=1000, dim=64, layers=[0])
    emb = NgramEmbedding(cfg, vocab_size=500, hidden_size=64).cuda()
    for t in emb.tables:
        nn.init.normal_(t.weight)
    ids = torch.randint(0, 500, (3, 37), device="cuda")
    prefix = torch.randint(0, 500, (3, 2), device="cuda")
    for pre in (None, prefix):
        got = emb.lookup(ids, pre)
        rows = emb.row_ids(ids, pre)
        want = sum(emb.tables[k].weight[rows[k] - k * cfg.num_buckets] for k in range(3))
        assert torch.equal(got, want)
        g = torch.randn_like(got)
        for t in emb.tables:
            t.weight.grad = None
        got.backward(g)
        for k, t in enumerate(emb.tables):
            ref = torch.zeros_like(t.weight).index_add_(0, (rows[k] - k * cfg.num_buckets).reshape(-1),
                                                        g.reshape(-1, 64))
            assert torch.allclose(t.weight.grad, ref, atol=1e-5)


def test_cast_bf16_matches_torch_rounding():
    """The weight cast kernel rounds like torch (nearest even), including infinities,
    NaN, denormals and values at the rounding midpoints."""
    from myk_llm_b200.ops import ext

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(4096 * 1024 + 16, device="cuda", generator=g) * 3.0
    x[:8] = torch.tensor([float("inf"), -float("inf"), 0.0, -0.0, 1e-40, -1e-42, 3.4e38, 1.00390625], device="cuda")
    x[8] = float("nan")
    mid = torch.arange(1, 8, device="cuda", dtype=torch.int32) * 65536 + 32768  # exact midpoints
    x[16:23] = mid.view(torch.float32)
    got = ext().cast_bf16(x)
    want = x.to(torch.bfloat16)
    same = (got.view(torch.int16) == want.view(torch.int16)) | (got.isnan() & want.isnan())
    assert bool(same.all())
