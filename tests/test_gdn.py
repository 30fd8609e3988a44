"""Gated delta rule: the chunked statement against the token recurrence (CPU, float64),
and the CUDA kernels (chunk forward/backward, recurrent decode, short convolution)
against the fp32 PyTorch oracles."""

import pytest
import torch
import torch.nn.functional as F

from myk_llm_b200.ops import reference as ref
from myk_llm_b200.ops.gdn_chunk import chunk_bwd, chunk_fwd


def _token_recurrence(q, k, v, g, b, s0, per_channel=False):
    s = s0
    outs = []
    for t in range(q.shape[0]):
        s = (torch.exp(g[t])[:, None] if per_channel else torch.exp(g[t])) * s
        u = b[t] * (v[t] - s.t() @ k[t])
        s = s + k[t][:, None] * u[None, :]
        outs.append(s.t() @ q[t])
    return torch.stack(outs), s


def _inputs(T, dk, dv, per_channel=False, seed=0):
    gen = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(T, dk, generator=gen, dtype=torch.float64), dim=-1) * dk ** -0.5
    k = F.normalize(torch.randn(T, dk, generator=gen, dtype=torch.float64), dim=-1)
    v = torch.randn(T, dv, generator=gen, dtype=torch.float64)
    g = -torch.rand(*((T, dk) if per_channel else (T,)), generator=gen, dtype=torch.float64) * 0.5
    b = torch.rand(T, generator=gen, dtype=torch.float64)
    s0 = torch.randn(dk, dv, generator=gen, dtype=torch.float64) * 0.1
    return q, k, v, g, b, s0


@pytest.mark.parametrize("T", [1, 63, 64, 150])
def test_chunk_forward_matches_recurrence(T):
    q, k, v, g, b, s0 = _inputs(T, 16, 24)
    o_ref, s_ref = _token_recurrence(q, k, v, g, b, s0)
    o, s, states = chunk_fwd(q, k, v, g, b, s0)
    assert len(states) == (T + 63) // 64
    torch.testing.assert_close(o, o_ref, rtol=0, atol=1e-12)
    torch.testing.assert_close(s, s_ref, rtol=0, atol=1e-12)


def test_chunk_forward_per_channel_matches_recurrence():
    q, k, v, g, b, s0 = _inputs(100, 16, 8, per_channel=True)
    o_ref, s_ref = _token_recurrence(q, k, v, g, b, s0, per_channel=True)
    o, s, _ = chunk_fwd(q, k, v, g, b, s0, per_channel=True)
    torch.testing.assert_close(o, o_ref, rtol=0, atol=1e-10)
    torch.testing.assert_close(s, s_ref, rtol=0, atol=1e-10)


@pytest.mark.parametrize("T", [40, 150])
def test_chunk_backward_matches_autograd(T):
    q, k, v, g, b, s0 = _inputs(T, 16, 24, seed=1)
    leaves = [x.clone().requires_grad_(True) for x in (q, k, v, g, b, s0)]
    o_ref, s_ref = _token_recurrence(*leaves)
    gen = torch.Generator().manual_seed(2)
    do = torch.randn(o_ref.shape, generator=gen, dtype=torch.float64)
    dsf = torch.randn(s_ref.shape, generator=gen, dtype=torch.float64)
    ((o_ref * do).sum() + (s_ref * dsf).sum()).backward()
    _, _, states = chunk_fwd(q, k, v, g, b, s0)
    grads = chunk_bwd(q, k, v, g, b, states, do, dsf)
    for got, leaf in zip(grads, leaves):
        torch.testing.assert_close(got, leaf.grad, rtol=0, atol=1e-10)


# ----------------------------------------------------------------------------- GPU


def _gdn_case(bsz, T, H, seed=0, device="cuda"):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(bsz, T, H, 128, generator=gen).to(device, torch.bfloat16)
    k = torch.randn(bsz, T, H, 128, generator=gen).to(device, torch.bfloat16)
    v = torch.randn(bsz, T, H, 128, generator=gen).to(device, torch.bfloat16)
    g = (-torch.rand(bsz, T, H, generator=gen) * 0.3).to(device)
    b = torch.rand(bsz, T, H, generator=gen).to(device)
    return q, k, v, g, b


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6)).item()


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["batch", "packed"])
def test_gdn_chunk_kernels_match_reference(layout):
    from myk_llm_b200.ops import gdn

    dev = torch.device("cuda")
    if layout == "batch":
        q, k, v, g, b = _gdn_case(2, 150, 2)
        cu = None
        init = torch.randn(2, 2, 128, 128, device=dev) * 0.05
    else:
        q, k, v, g, b = _gdn_case(1, 300, 2)
        cu = torch.tensor([0, 37, 150, 300], device=dev, dtype=torch.int32)
        init = None
    leaves = [x.clone().requires_grad_(True) for x in (q, k, v, g, b)]
    o, fin = gdn.gated_delta_rule(*leaves, initial_state=init, cu_seqlens=cu, output_final_state=True)
    ref_leaves = [x.detach().float().clone().requires_grad_(True) for x in (q, k, v, g, b)]
    o_ref, fin_ref = ref.delta_rule_ref(*ref_leaves, initial_state=init, cu_seqlens=cu)
    o_ref32 = o_ref.float()
    assert _rel(o, o_ref32) < 2e-2
    assert _rel(fin, fin_ref) < 1e-2
    do = torch.randn_like(o_ref32)
    (o.float() * do).sum().backward()
    (o_ref32 * do).sum().backward()
    for name, a, r in zip("qkvgb", leaves, ref_leaves):
        assert _rel(a.grad, r.grad) < 3e-2, (name, _rel(a.grad, r.grad))
    from myk_llm_b200.ops import ext

    assert ext().take_status() == 0


@pytest.mark.gpu
def test_gdn_recurrent_decode_matches_reference():
    from myk_llm_b200.ops import gdn

    q, k, v, g, b = _gdn_case(2, 3, 4, seed=3)
    init = torch.randn(2, 4, 128, 128, device="cuda") * 0.05
    with torch.no_grad():
        o, fin = gdn.gated_delta_rule(q, k, v, g, b, initial_state=init, output_final_state=True)
    o_ref, fin_ref = ref.delta_rule_ref(q, k, v, g, b, initial_state=init)
    assert _rel(o, o_ref) < 2e-2
    assert _rel(fin, fin_ref) < 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["batch", "packed"])
def test_causal_conv1d_kernels_match_reference(layout):
    from myk_llm_b200.ops import gdn

    gen = torch.Generator().manual_seed(5)
    if layout == "batch":
        x = torch.randn(2, 70, 96, generator=gen).cuda().bfloat16()
        cu = None
    else:
        x = torch.randn(1, 90, 96, generator=gen).cuda().bfloat16()
        cu = torch.tensor([0, 2, 40, 90], device="cuda", dtype=torch.int32)
    w = (torch.randn(96, 4, generator=gen) * 0.3).cuda()
    xl, wl = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    y, fin = gdn.causal_conv1d(xl, wl, cu_seqlens=cu, return_final_state=True)
    xr, wr = x.float().clone().requires_grad_(True), w.clone().requires_grad_(True)
    y_ref, fin_ref = ref.causal_conv1d_ref(xr, wr, cu_seqlens=cu)
    assert _rel(y, y_ref) < 1e-2
    torch.testing.assert_close(fin.float(), fin_ref.float(), rtol=0, atol=1e-2)
    dy = torch.randn_like(y_ref.float())
    (y.float() * dy).sum().backward()
    (y_ref.float() * dy).sum().backward()
    assert _rel(xl.grad, xr.grad) < 1e-2
    assert _rel(wl.grad, wr.grad) < 1e-2


@pytest.mark.parametrize("per_channel", [False, True])
@pytest.mark.parametrize("packed", [False, True])
def test_batched_chunked_statement_matches_recurrence_and_its_gradients(per_channel, packed):
    """The chunked statement run over every sequence and head at once (the GPU path for
    per-channel decay and for head dims other than 128) against the token recurrence:
    outputs, final states and the gradients of every input, for packed documents of
    unequal lengths (one of a single token) and for a batch of rows."""
    from myk_llm_b200.ops.gdn import _chunked_torch

    torch.manual_seed(3)
    H, dk, dv = 2, 16, 8
    if packed:
        B, T, cu = 1, 100, torch.tensor([0, 37, 38, 100], dtype=torch.int32)
    else:
        B, T, cu = 2, 70, None
    seqs = 3 if packed else B
    leaves = [torch.randn(B, T, H, dk), torch.randn(B, T, H, dk), torch.randn(B, T, H, dv),
              -torch.rand(B, T, H, *((dk,) if per_channel else ())) * 0.3, torch.rand(B, T, H),
              torch.randn(seqs, H, dk, dv) * 0.1]
    a = [t.clone().requires_grad_() for t in leaves]
    b = [t.clone().requires_grad_() for t in leaves]
    o, fin = _chunked_torch(*a[:5], a[5], cu, per_channel)
    o_ref, fin_ref = ref.delta_rule_ref(*b[:5], initial_state=b[5], cu_seqlens=cu, per_channel_decay=per_channel)
    torch.testing.assert_close(o, o_ref, atol=2e-5, rtol=2e-5)
    torch.testing.assert_close(fin, fin_ref, atol=2e-5, rtol=2e-5)
    wo, wf = torch.randn_like(o), torch.randn_like(fin)
    ((o * wo).sum() + (fin * wf).sum()).backward()
    ((o_ref * wo).sum() + (fin_ref * wf).sum()).backward()
    for x, y in zip(a, b):
        torch.testing.assert_close(x.grad, y.grad, atol=1e-4, rtol=1e-4)
