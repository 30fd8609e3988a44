"""Memory-bound fused ops: RMSNorm (+ residual add), SwiGLU, RoPE, gates, embedding.

On CUDA each is one sm_100a kernel per direction (``csrc/norm.cu``, ``csrc/elementwise.cu``):
the reference has Inductor generate these from ``torch.compile(Block._forward)``
(``src/myk_llm/model/transformer.py:250-257``).  Statistics are kept in fp32.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import reference as ref
from ._ext import ext


def _c(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------------------
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps, out_dtype):
        shape = x.shape
        x2 = _c(x.reshape(-1, shape[-1]))
        y, rstd = ext().rmsnorm_fwd(x2, w, None, float(eps), out_dtype)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dx, dw = ext().rmsnorm_bwd(_c(dy.reshape(x2.shape)), x2, w, rstd, None, False)
        return dx.view(ctx.shape), dw, None, None


class _AddRMSNorm(torch.autograd.Function):
    """s = x + u; y = rmsnorm(s).  Returns (s, y); s keeps x's dtype."""

    @staticmethod
    def forward(ctx, x, u, w, eps, out_dtype):
        shape = x.shape
        x2 = _c(x.reshape(-1, shape[-1]))
        u2 = _c(u.reshape(-1, shape[-1]))
        s = torch.empty_like(x2)
        y, rstd = ext().rmsnorm_fwd(x2, w, (u2, s), float(eps), out_dtype)
        ctx.save_for_backward(s, w, rstd)
        ctx.shape, ctx.u_dtype = shape, u.dtype
        return s.view(shape), y.view(shape)

    @staticmethod
    def backward(ctx, ds, dy):
        s, w, rstd = ctx.saved_tensors
        res = _c(ds.reshape(s.shape)) if ds is not None else None
        if ctx.u_dtype == torch.bfloat16 and s.dtype == torch.float32:
            # the bf16 gradient of the update branch comes out of the same kernel
            dx, dw, du = ext().rmsnorm_bwd(_c(dy.reshape(s.shape)), s, w, rstd, res, True)
            return dx.view(ctx.shape), du.view(ctx.shape), dw, None, None
        dx, dw = ext().rmsnorm_bwd(_c(dy.reshape(s.shape)), s, w, rstd, res, False)
        dx = dx.view(ctx.shape)
        du = dx if ctx.u_dtype == dx.dtype else dx.to(ctx.u_dtype)
        return dx, du, dw, None, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, out_dtype: torch.dtype | None = None):
    out_dtype = out_dtype or torch.promote_types(x.dtype, weight.dtype)
    if not x.is_cuda:
        return ref.rms_norm_ref(x, weight, eps).to(out_dtype)
    return _RMSNorm.apply(x, weight, eps, out_dtype)


def add_rms_norm(x: torch.Tensor, update: torch.Tensor, weight: torch.Tensor, eps: float,
                 out_dtype: torch.dtype | None = None):
    """(x + update, rmsnorm(x + update)) in one pass over memory."""
    out_dtype = out_dtype or torch.promote_types(x.dtype, weight.dtype)
    if not x.is_cuda:
        s = x + update
        return s, rms_norm(s, weight, eps, out_dtype)
    return _AddRMSNorm.apply(x, update, weight, eps, out_dtype)


class _GatedRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, g, w, eps, act):
        shape = o.shape
        o2 = _c(o.reshape(-1, shape[-1]))
        g2 = _c(g.reshape(-1, shape[-1])) if g is not None else None
        y, rstd = ext().gated_rmsnorm_fwd(o2, g2, w, float(eps), int(act))
        ctx.save_for_backward(o2, g2, w, rstd)
        ctx.shape, ctx.act, ctx.has_g = shape, act, g is not None
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        o2, g2, w, rstd = ctx.saved_tensors
        do, dg, dw = ext().gated_rmsnorm_bwd(_c(dy.reshape(o2.shape)), o2, g2, w, rstd, int(ctx.act))
        return do.view(ctx.shape), (dg.view(ctx.shape) if ctx.has_g else None), dw, None, None


def gated_rms_norm(o, gate, weight, eps, activation="swish"):
    if not o.is_cuda:
        return ref.gated_rms_norm_ref(o, gate, weight, eps, activation).to(o.dtype)
    act = 0 if activation in ("swish", "silu") else 1
    return _GatedRMSNorm.apply(o, gate, weight, eps, act)


# ---------------------------------------------------------------------------------------
# SwiGLU and gates
# ---------------------------------------------------------------------------------------
class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu2 = _c(gu)
        ctx.save_for_backward(gu2)
        return ext().swiglu_fwd(gu2)

    @staticmethod
    def backward(ctx, da):
        (gu,) = ctx.saved_tensors
        return ext().swiglu_bwd(_c(da), gu)


def swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up where gate/up are the two halves of the last dimension."""
    if not gate_up.is_cuda:
        g, u = gate_up.chunk(2, dim=-1)
        return F.silu(g) * u
    return _SwiGLU.apply(gate_up)


def sigmoid_gate(x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """x * sigmoid(g) (attention output gate)."""
    return x * torch.sigmoid(g.float()).to(x.dtype)


def silu(x: torch.Tensor) -> torch.Tensor:
    return F.silu(x)


class _SplitCols(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, widths):
        return tuple(ext().split_cols(x, list(widths)))

    @staticmethod
    def backward(ctx, *grads):
        return torch.cat([g.contiguous() for g in grads], dim=-1), None


def split_cols(x: torch.Tensor, widths) -> tuple[torch.Tensor, ...]:
    """Split the last dimension of ``x`` (..., sum(widths)) into contiguous tensors in one
    pass (a plain ``split`` returns strided views, and copying those is slow)."""
    lead = x.shape[:-1]
    widths = tuple(int(w) for w in widths)
    x2 = x.reshape(-1, x.shape[-1])
    if not x.is_cuda or x.dtype != torch.bfloat16 or any(w % 8 for w in widths) or x2.stride(-1) != 1 \
            or x2.stride(0) % 8 or x2.data_ptr() % 16:
        return tuple(t.contiguous() for t in x.split(widths, dim=-1))
    return tuple(t.view(*lead, w) for t, w in zip(_SplitCols.apply(x2, widths), widths))


# ---------------------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------------------
class _Rope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin, pos):
        y = ext().rope(x, cos, sin, pos, False)
        ctx.save_for_backward(cos, sin, pos)
        return y

    @staticmethod
    def backward(ctx, dy):
        cos, sin, pos = ctx.saved_tensors
        return ext().rope(dy, cos, sin, pos, True), None, None, None


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, position_ids: torch.Tensor) -> torch.Tensor:
    """Rotate x (B, S, H, D) with interleaved pairs to positions (B, S) using fp32 tables."""
    if not x.is_cuda:
        c = cos[position_ids].unsqueeze(2)
        s = sin[position_ids].unsqueeze(2)
        return ref.rope_ref(x, c, s)
    pos = position_ids.expand(x.shape[0], x.shape[1])
    if pos.dtype != torch.int64:
        pos = pos.long()
    return _Rope.apply(x, cos, sin, _c(pos))


class _RopeQKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cos, sin, pos, heads: int, kv_heads: int):
        q, k, v = ext().rope_qkv_fwd(qkv, cos, sin, pos, heads, kv_heads)
        ctx.save_for_backward(cos, sin, pos)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos, sin, pos = ctx.saved_tensors
        return ext().rope_qkv_bwd(dq, dk, dv, cos, sin, pos), None, None, None, None, None


def rope_qkv(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, position_ids: torch.Tensor, heads: int,
             kv_heads: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Split a fused QKV projection (B, S, (heads + 2 kv_heads) d) into rotated q (B, S, heads, d),
    rotated k and v (B, S, kv_heads, d) in one pass (one kernel forward, one backward that
    writes the QKV gradient directly)."""
    b, s_, width = qkv.shape
    d = width // (heads + 2 * kv_heads)
    if not qkv.is_cuda or d not in (64, 128) or qkv.dtype != torch.bfloat16:
        q, k, v = qkv.split((heads * d, kv_heads * d, kv_heads * d), dim=-1)
        q, k = q.view(b, s_, heads, d), k.view(b, s_, kv_heads, d)
        return apply_rope(q, cos, sin, position_ids), apply_rope(k, cos, sin, position_ids), \
            v.view(b, s_, kv_heads, d)
    pos = position_ids.expand(b, s_)
    if pos.dtype != torch.int64:
        pos = pos.long()
    return _RopeQKV.apply(qkv, cos, sin, _c(pos), heads, kv_heads)


# ---------------------------------------------------------------------------------------
# embedding
# ---------------------------------------------------------------------------------------
class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w):
        ids2 = _c(ids.reshape(-1))
        out = ext().embedding_fwd(ids2, w)
        ctx.save_for_backward(ids2)
        ctx.w = w
        ctx.shape = ids.shape
        return out.view(*ids.shape, w.shape[1])

    @staticmethod
    def backward(ctx, dout):
        (ids2,) = ctx.saved_tensors
        w = ctx.w
        main = getattr(w, "main_grad", None)
        if main is not None:
            ext().embedding_bwd(ids2, _c(dout.reshape(-1, w.shape[1])), main)
            return None, None
        grad = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        ext().embedding_bwd(ids2, _c(dout.reshape(-1, w.shape[1])), grad)
        return None, grad.to(w.dtype)


def embedding(ids: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Row gather; the output keeps the table's dtype (fp32 master tables give an fp32
    residual stream, as under the reference's autocast)."""
    if not ids.is_cuda:
        return F.embedding(ids, weight)
    return _Embedding.apply(ids, weight)


def ngram_lookup(tokens, tables, orders, context, num_buckets):
    """Sum over orders of ``table_k[hash_k(tokens)]`` -> (batch, seq, dim); ``tokens`` carries
    ``context`` columns of left context.  CUDA: the fused hash + gather + sum kernel."""
    from ..models.embeddings import _NgramEmbed, ngram_bucket_ids

    if tokens.is_cuda:
        return _NgramEmbed.apply(tokens, context, tuple(orders), *tables)
    total = None
    for n, table in zip(orders, tables):
        rows = F.embedding(ngram_bucket_ids(tokens, n, context, num_buckets), table)
        total = rows if total is None else total + rows
    return total
