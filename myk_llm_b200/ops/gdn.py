"""Gated DeltaNet / Kimi Delta Attention ops: short causal convolution, decay gates,
the gated delta rule (chunked for training, recurrent for decode) and the gated norm.

Semantics are those of the flash-linear-attention calls in the reference
(``src/myk_llm/model/mixers.py:220-314``): q and k are L2-normalised inside the op, the
scale is ``head_k_dim ** -0.5``, the decay is ``g = -exp(A_log) * softplus(a + dt_bias)`` in
log space (per head for GDN, per key channel for KDA), beta arrives already passed
through a sigmoid.

CUDA kernels (``csrc/gdn.cu``, ``csrc/gdn_tc.cu``):

* ``conv1d_fwd/bwd``: depthwise causal conv + SiLU over the packed q/k/v, resetting at
  document boundaries;
* ``gdn_chunk_fwd/bwd``: the chunked delta rule (chunk 64, head dims 128) on the tcgen05
  tensor cores: chunk-parallel prep / output / gradient kernels (one CTA per chunk and
  head) around the two state recurrences (one CTA per sequence, head and 64 value
  columns, the fp32 state slice kept in TMEM); the algorithm is stated in
  :mod:`myk_llm_b200.ops.gdn_chunk`.  Per-channel (KDA) decay runs that statement in
  PyTorch on the GPU;
* ``gdn_recurrent``: token-by-token decode over a state cache;
* ``gdn_spec_window``: one speculative-decoding window over a committed state plus the
  previous window's pending inputs (:func:`spec_window`).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import reference as ref
from ._ext import ext


def gdn_gate(a: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor) -> torch.Tensor:
    """Log-space decay per head: -exp(A_log) * softplus(a + dt_bias), fp32."""
    return -torch.exp(A_log.float()) * F.softplus(a.float() + dt_bias.float())


def kda_gate(f: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor) -> torch.Tensor:
    """Per-channel KDA decay: -exp(A_log[h]) * softplus(f + dt_bias), f (B, T, H, dk)."""
    heads, dk = f.shape[-2], f.shape[-1]
    return -torch.exp(A_log.float()).view(heads, 1) * F.softplus(f.float() + dt_bias.float().view(heads, dk))


class _Conv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, cu, init):
        y, final = ext().conv1d_fwd(x, w, cu, init)
        ctx.save_for_backward(x, w, cu, init)
        return y, final

    @staticmethod
    def backward(ctx, dy, _dfinal):
        x, w, cu, init = ctx.saved_tensors
        dx, dw = ext().conv1d_bwd(dy.contiguous(), x, w, cu, init)
        return dx, dw.to(w.dtype), None, None


def causal_conv1d(x, weight, cu_seqlens=None, initial_state=None, return_final_state=False):
    """x (B, T, D), weight (D, K) -> (silu(conv(x)), final_state (B or N, D, K-1) or None)."""
    if not x.is_cuda or (initial_state is not None and torch.is_grad_enabled()):
        y, fin = ref.causal_conv1d_ref(x, weight, cu_seqlens=cu_seqlens, initial_state=initial_state)
        return y, (fin.to(x.dtype) if return_final_state else None)
    xb = x.contiguous()
    y, fin = _Conv.apply(xb, weight.contiguous(), cu_seqlens, initial_state)
    return y, (fin if return_final_state else None)


class _DeltaRule(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, init, cu):
        o, final, *saved = ext().gdn_chunk_fwd(q, k, v, g, beta, init, cu, False)
        ctx.save_for_backward(q, k, v, g, beta, init, cu, *saved)
        return o, final

    @staticmethod
    def backward(ctx, do, dfinal):
        q, k, v, g, beta, init, cu, *saved = ctx.saved_tensors
        dq, dk, dv, dg, db, dinit = ext().gdn_chunk_bwd(do.contiguous(), q, k, v, g, beta, init, cu, list(saved),
                                                        dfinal, False)
        return dq, dk, dv, dg, db, (dinit if ctx.needs_input_grad[5] else None), None


def _chunked_torch(q, k, v, g, beta, initial_state, cu_seqlens, per_channel):
    """Differentiable chunked statement (``gdn_chunk.chunk_fwd``) per sequence and head;
    the path for per-channel (KDA) decay on the GPU."""
    from .gdn_chunk import chunk_fwd

    bsz, t_len, heads, dk = q.shape
    qf = F.normalize(q.float(), dim=-1, eps=1e-6) * dk ** -0.5
    kf = F.normalize(k.float(), dim=-1, eps=1e-6)
    spans = ([(0, a, b) for a, b in zip(cu_seqlens.tolist()[:-1], cu_seqlens.tolist()[1:])] if cu_seqlens is not None
             else [(b, 0, t_len) for b in range(bsz)])
    rows, finals = [], []
    for i, (b, a, e) in enumerate(spans):
        outs, fins = [], []
        for h in range(heads):
            s0 = initial_state[i, h] if initial_state is not None else None
            o, s, _ = chunk_fwd(qf[b, a:e, h], kf[b, a:e, h], v[b, a:e, h], g[b, a:e, h], beta[b, a:e, h], s0,
                                per_channel=per_channel)
            outs.append(o)
            fins.append(s)
        rows.append(torch.stack(outs, 1))
        finals.append(torch.stack(fins))
    if cu_seqlens is not None:
        o = torch.cat(rows, 0)[None]
    else:
        o = torch.stack(rows)
    return o.to(v.dtype), torch.stack(finals)


def gated_delta_rule(q, k, v, g, beta, initial_state=None, cu_seqlens=None, cu_seqlens_cpu=None,
                     output_final_state=False, per_channel_decay=False):
    """o_t = S_t^T (q_t / sqrt(dk)) with S_t = exp(g_t) S_{t-1} + k_t (beta_t (v_t - S^T k_t))^T,
    q/k L2-normalised.  Returns (o (B, T, H, dv), final state (N, H, dk, dv) fp32 or None)."""
    if not q.is_cuda:
        o, fin = ref.delta_rule_ref(q, k, v, g, beta, initial_state=initial_state, cu_seqlens=cu_seqlens,
                                    per_channel_decay=per_channel_decay)
        return o, (fin if output_final_state else None)
    if not torch.is_grad_enabled() and q.shape[1] <= 64 and cu_seqlens is None:
        o, fin = ext().gdn_recurrent(q.contiguous(), k.contiguous(), v.contiguous(), g.contiguous(),
                                     beta.contiguous(), initial_state, bool(per_channel_decay))
        return o, (fin if output_final_state else None)
    if per_channel_decay or q.shape[-1] != 128 or v.shape[-1] != 128 or v.shape[-2] != q.shape[-2]:
        o, fin = _chunked_torch(q, k, v, g, beta, initial_state, cu_seqlens, per_channel_decay)
        return o, (fin if output_final_state else None)
    cu = cu_seqlens.int() if cu_seqlens is not None else None
    o, fin = _DeltaRule.apply(q.contiguous(), k.contiguous(), v.contiguous(), g.float().contiguous(),
                              beta.float().contiguous(), initial_state, cu)
    return o, (fin if output_final_state else None)


def spec_window(q, k, v, g, beta, state, pending_inputs, pending, per_channel_decay=False):
    """One speculative-decoding window of the gated delta rule.

    ``state`` (B, H, dk, dv) fp32 is the committed state of every row; ``pending_inputs``
    = (q, k, v, g, beta) of the previous window, of which row b accepted the first
    ``pending[b]`` tokens.  Folds those into ``state`` in place (the new committed state),
    runs this window's W tokens from it and returns their outputs (B, W, H, dv); this
    window's inputs are copied into ``pending_inputs`` for the next call.  So a window can
    be verified and only the accepted prefix committed, with one state read and one state
    write per call.
    """
    pq, pk, pv, pg, pb = pending_inputs
    g, beta = g.float().contiguous(), beta.float().contiguous()
    if q.is_cuda:
        return ext().gdn_spec_window(q.contiguous(), k.contiguous(), v.contiguous(), g, beta, state, pq, pk, pv, pg, pb,
                                     pending, bool(per_channel_decay))
    for b in range(q.size(0)):
        n = int(pending[b])
        if n > 0:
            _, fin = ref.delta_rule_ref(pq[b:b + 1, :n], pk[b:b + 1, :n], pv[b:b + 1, :n], pg[b:b + 1, :n],
                                        pb[b:b + 1, :n], initial_state=state[b:b + 1],
                                        per_channel_decay=per_channel_decay)
            state[b] = fin[0]
    o, _ = ref.delta_rule_ref(q, k, v, g, beta, initial_state=state, per_channel_decay=per_channel_decay)
    for dst, src in zip(pending_inputs, (q, k, v, g, beta)):
        dst.copy_(src)
    return o.to(v.dtype)
