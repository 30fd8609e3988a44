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
    """Differentiable chunked statement (``gdn_chunk.chunk_fwd_batched``) over every
    sequence and head at once; the path for per-channel (KDA) decay and for head dims other
    than 128 on the GPU.  Packed documents are gathered into rows padded at the end to the
    longest document (padding leaves the state unchanged) and scattered back."""
    from .gdn_chunk import chunk_fwd_batched

    bsz, t_len, heads, dk = q.shape
    dv = v.shape[-1]
    qf = F.normalize(q.float(), dim=-1, eps=1e-6) * dk ** -0.5
    kf = F.normalize(k.float(), dim=-1, eps=1e-6)
    gf, bf, vf = g.float(), beta.float(), v.float()
    if cu_seqlens is not None:
        cu = cu_seqlens.to(device="cpu", dtype=torch.long)
        lens = cu[1:] - cu[:-1]
        n, width = lens.numel(), max(1, int(lens.max())) if lens.numel() else 1
        pos = torch.arange(width)
        valid = pos[None, :] < lens[:, None]  # (n, width)
        idx = (cu[:-1, None] + pos[None, :]).clamp(max=max(0, t_len - 1))
        valid_d, idx_d = valid.to(q.device), idx.to(q.device)

        def rows(x):  # (1, T, ...) -> (n, width, ...) with zeros past each document
            y = x[0][idx_d]
            return y * valid_d.view(n, width, *([1] * (y.dim() - 2))).to(y.dtype)
        qf, kf, vf, gf, bf = (rows(t) for t in (qf, kf, vf, gf, bf))
    else:
        n, width = bsz, t_len
    # (n, width, heads, d) -> (n * heads, width, d)
    def flat(x):
        return x.transpose(1, 2).reshape(n * heads, width, *x.shape[3:])
    s0 = initial_state.reshape(n * heads, dk, dv) if initial_state is not None else None
    o, fin = chunk_fwd_batched(flat(qf), flat(kf), flat(vf), flat(gf), flat(bf), s0, per_channel=per_channel)
    o = o.reshape(n, heads, width, dv).transpose(1, 2)
    if cu_seqlens is not None:
        o = o[valid_d][None]
    return o.to(v.dtype), fin.reshape(n, heads, dk, dv)


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
