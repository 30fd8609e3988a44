"""Plain PyTorch statements of every op the CUDA kernels implement.

These run on the CPU path (tests, the tiny fp32 config) and are the fp32 oracles the GPU
tests compare the kernels against.  They are written for clarity, not speed.

Semantics follow the reference's ops:

* attention: ``src/myk_llm/ops/flash_attn.py:13-18,147-151`` (queries aligned to the end
  of the keys, sliding window ``(left, right)``, rows without keys output 0, GQA);
* fused linear cross-entropy + z-loss: ``src/myk_llm/ops/fused_ce.py:20-107``;
* Newton-Schulz: ``src/myk_llm/train/optim.py:17-32``;
* Gated DeltaNet / KDA, short convolution and gated norm: the fla semantics the reference
  calls from ``src/myk_llm/model/mixers.py:220-314``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

IGNORE_INDEX = -100
NS_COEFFICIENTS = (3.4445, -4.7750, 2.0315)


# ---------------------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------------------
def _attend_one(q, k, v, causal, window, scale, softcap=0.0):
    """q (Lq, H, d), k/v (Lk, KVH, d) -> (Lq, H, d) and lse (H, Lq) in natural log."""
    lq, h, _ = q.shape
    lk, kvh, _ = k.shape
    group = h // kvh
    kk = k.repeat_interleave(group, dim=1)
    vv = v.repeat_interleave(group, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kk.float()) * scale
    if softcap > 0:
        s = softcap * torch.tanh(s / softcap)
    qpos = torch.arange(lq, device=q.device)[:, None] + (lk - lq)
    kpos = torch.arange(lk, device=q.device)[None, :]
    allowed = torch.ones(lq, lk, dtype=torch.bool, device=q.device)
    left, right = window
    if causal:
        allowed &= kpos <= qpos
    if left >= 0:
        allowed &= kpos >= qpos - left
    if right >= 0 and not causal:
        allowed &= kpos <= qpos + right
    s = s.masked_fill(~allowed[None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)  # (H, Lq)
    p = torch.exp(s - lse[..., None])
    p = torch.nan_to_num(p, nan=0.0)
    out = torch.einsum("hqk,khd->qhd", p, vv.float())
    empty = ~allowed.any(-1)  # (Lq,)
    out[empty] = 0.0
    lse = lse.masked_fill(empty[None], float("inf"))
    return out, lse


def attention_ref(q, k, v, causal=True, window=(-1, -1), softmax_scale=None, seqused_k=None):
    """Dense batch: q (B, Lq, H, d), k/v (B, Lk, KVH, d); returns (out, lse (B, H, Lq))."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.size(-1))
    outs, lses = [], []
    for b in range(q.size(0)):
        kb, vb = k[b], v[b]
        if seqused_k is not None:
            n = int(seqused_k[b])
            kb, vb = kb[:n], vb[:n]
        o, l = _attend_one(q[b], kb, vb, causal, window, scale)
        outs.append(o)
        lses.append(l)
    return torch.stack(outs).to(q.dtype), torch.stack(lses)


def attention_varlen_ref(q, k, v, cu_q, cu_k, causal=True, window=(-1, -1), softmax_scale=None):
    """Packed: q (Tq, H, d), k/v (Tk, KVH, d); one segment per document."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.size(-1))
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.full((q.size(1), q.size(0)), float("inf"), device=q.device)
    cq, ck = cu_q.tolist(), cu_k.tolist()
    for i in range(len(cq) - 1):
        qs, qe, ks, ke = cq[i], cq[i + 1], ck[i], ck[i + 1]
        if qe == qs:
            continue
        o, l = _attend_one(q[qs:qe], k[ks:ke], v[ks:ke], causal, window, scale)
        out[qs:qe] = o
        lse[:, qs:qe] = l
    return out.to(q.dtype), lse


# ---------------------------------------------------------------------------------------
# elementwise / normalisation
# ---------------------------------------------------------------------------------------
def rms_norm_ref(x, weight, eps):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return y * weight.float()


def swiglu_ref(gate_up):
    gate, up = gate_up.float().chunk(2, dim=-1)
    return F.silu(gate) * up


def rotate_pairs(x):
    """Interleaved-pair rotation: (x0, x1) -> (-x1, x0) for each pair (2i, 2i+1)."""
    x1, x2 = x[..., ::2], x[..., 1::2]
    return torch.stack((-x2, x1), dim=-1).flatten(-2)


def rope_ref(x, cos, sin):
    """x (..., S, H, d) with cos/sin (..., S, 1, d) already gathered at the positions."""
    xf = x.float()
    return (xf * cos + rotate_pairs(xf) * sin).to(x.dtype)


def gated_rms_norm_ref(o, gate, weight, eps, activation="swish"):
    of = o.float()
    y = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    if gate is None:
        return y
    g = gate.float()
    return y * (F.silu(g) if activation in ("swish", "silu") else torch.sigmoid(g))


# ---------------------------------------------------------------------------------------
# loss
# ---------------------------------------------------------------------------------------
def linear_cross_entropy_ref(hidden, weight, targets, normalizer, z_loss=0.0):
    """Returns (loss, ce_sum, z_sum) with loss = (ce_sum + z_loss * z_sum) / normalizer,
    z = logsumexp(logits)^2 over supervised tokens."""
    h = hidden.reshape(-1, hidden.size(-1))
    t = targets.reshape(-1)
    logits = (h @ weight.t()).float()
    valid = t != IGNORE_INDEX
    lse = torch.logsumexp(logits, dim=-1)
    tgt = logits.gather(1, t.clamp(min=0)[:, None])[:, 0]
    ce = torch.where(valid, lse - tgt, torch.zeros_like(lse))
    z = torch.where(valid, lse * lse, torch.zeros_like(lse))
    ce_sum, z_sum = ce.sum(), z.sum()
    loss = (ce_sum + z_loss * z_sum) / normalizer
    return loss, ce_sum.detach(), z_sum.detach()


# ---------------------------------------------------------------------------------------
# optimizer math
# ---------------------------------------------------------------------------------------
def newton_schulz_ref(g, steps, eps=1e-7):
    a, b, c = NS_COEFFICIENTS
    x = g.bfloat16()
    tall = g.size(-2) > g.size(-1)
    if tall:
        x = x.transpose(-1, -2)
    x = x / x.float().norm(dim=(-2, -1), keepdim=True).clamp(min=eps).to(x.dtype)
    for _ in range(steps):
        gram = x @ x.transpose(-1, -2)
        poly = b * gram + c * (gram @ gram)
        x = a * x + poly @ x
    return x.transpose(-1, -2) if tall else x


def adamw_ref(p, g, m, v, step, lr, beta1, beta2, eps, wd):
    """In-place AdamW (decoupled decay), torch.optim.AdamW semantics."""
    p.mul_(1 - lr * wd)
    m.lerp_(g, 1 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1**step
    bc2 = 1 - beta2**step
    denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
    p.addcdiv_(m, denom, value=-lr / bc1)


# ---------------------------------------------------------------------------------------
# Gated DeltaNet / KDA
# ---------------------------------------------------------------------------------------
def causal_conv1d_ref(x, weight, bias=None, cu_seqlens=None, initial_state=None, activation=True):
    """Depthwise causal convolution over time.

    x (B, T, D); weight (D, K); output y_t = silu(sum_i w[:, i] * x_{t-K+1+i} + b).
    With ``cu_seqlens`` (B must be 1) each document starts from zeros.  Returns
    (y, final_state) where final_state (B, D, K-1) holds the last K-1 inputs.
    """
    bsz, t_len, dim = x.shape
    k = weight.size(-1)
    w = weight.reshape(dim, k).float()

    def run(seg, init):
        # seg (T, D); init (D, K-1) or None
        pad = init.t().float() if init is not None else seg.new_zeros(k - 1, dim, dtype=torch.float32)
        full = torch.cat([pad, seg.float()], 0)
        out = torch.zeros(seg.size(0), dim, dtype=torch.float32, device=seg.device)
        for i in range(k):
            out += full[i : i + seg.size(0)] * w[:, i]
        if bias is not None:
            out += bias.float()
        state = full[-(k - 1):].t() if k > 1 else full.new_zeros(dim, 0)
        return (F.silu(out) if activation else out), state

    if cu_seqlens is not None:
        assert bsz == 1
        cu = cu_seqlens.tolist()
        ys, states = [], []
        for i in range(len(cu) - 1):
            y, s = run(x[0, cu[i]:cu[i + 1]], None)
            ys.append(y)
            states.append(s)
        return torch.cat(ys, 0)[None].to(x.dtype), torch.stack(states)
    ys, states = [], []
    for b in range(bsz):
        y, s = run(x[b], None if initial_state is None else initial_state[b])
        ys.append(y)
        states.append(s)
    return torch.stack(ys).to(x.dtype), torch.stack(states)


def gdn_gate_ref(a, A_log, dt_bias):
    """log-space decay g = -exp(A_log) * softplus(a + dt_bias)."""
    return -torch.exp(A_log.float()) * F.softplus(a.float() + dt_bias.float())


def delta_rule_ref(q, k, v, g, beta, initial_state=None, cu_seqlens=None, scale=None,
                   l2norm=True, per_channel_decay=False):
    """Gated delta rule, token by token.

    q/k (B, T, H, dk), v (B, T, H, dv), g (B, T, H) (or (B, T, H, dk) for KDA) log decay,
    beta (B, T, H) already in (0, 1).  State S (H, dk, dv):
        S <- S * exp(g_t);  u = beta_t (v_t - S^T k_t);  S <- S + k_t u^T;  o_t = S^T q_t.
    Returns (o (B, T, H, dv), final states (N, H, dk, dv)).
    """
    bsz, t_len, heads, dk = q.shape
    dv = v.size(-1)
    scale = scale if scale is not None else dk ** -0.5
    qf, kf, vf = q.float(), k.float(), v.float()
    if l2norm:
        qf = F.normalize(qf, dim=-1, eps=1e-6)
        kf = F.normalize(kf, dim=-1, eps=1e-6)
    qf = qf * scale
    gf, bf = g.float(), beta.float()
    out = torch.zeros(bsz, t_len, heads, dv, dtype=torch.float32, device=q.device)

    def run(b, start, end, state):
        s = state.clone() if state is not None else torch.zeros(heads, dk, dv, device=q.device)
        for t in range(start, end):
            decay = torch.exp(gf[b, t])
            s = s * (decay[:, :, None] if per_channel_decay else decay[:, None, None])
            kt = kf[b, t]
            pred = torch.einsum("hk,hkv->hv", kt, s)
            u = bf[b, t][:, None] * (vf[b, t] - pred)
            s = s + kt[:, :, None] * u[:, None, :]
            out[b, t] = torch.einsum("hk,hkv->hv", qf[b, t], s)
        return s

    finals = []
    if cu_seqlens is not None:
        cu = cu_seqlens.tolist()
        for i in range(len(cu) - 1):
            init = initial_state[i] if initial_state is not None else None
            finals.append(run(0, cu[i], cu[i + 1], init))
    else:
        for b in range(bsz):
            init = initial_state[b] if initial_state is not None else None
            finals.append(run(b, 0, t_len, init))
    return out.to(v.dtype), torch.stack(finals)
