"""Linear layers on the tcgen05 GEMM.

``gemm`` computes ``D[m, n] = alpha * sum_k A[m, k] * B[n, k] + beta * C[m, n]`` with bf16
operands and fp32 accumulation in tensor memory.  Each operand is passed either K-major
(the reduction dimension is contiguous) or MN-major (the output dimension is
contiguous), which covers the forward ``x W^T``, the data gradient ``dy W`` and the weight
gradient ``dy^T x`` of a linear layer without any transposing copy.  With
``accumulate=True`` the fp32 output is added to atomically, which also lets the kernel
split K across CTAs when the output has too few tiles to fill the 148 SMs.

The reference runs these through cuBLAS under autocast (``nn.Linear`` in
``src/myk_llm/model/*.py``); here every block linear is this kernel.

Master weights stay fp32.  The bf16 copy a GEMM reads is cached on the parameter and
refreshed when the parameter's version counter changes (i.e. after an optimizer step), so
gradient accumulation and the backward pass reuse one cast per step.  A parameter that
carries a ``main_grad`` fp32 buffer receives its weight gradient accumulated in place by
the GEMM epilogue (no separate gradient tensor, no extra add).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_major: str = "k", b_major: str = "k",
         out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16, alpha: float = 1.0,
         beta: float = 0.0, c: torch.Tensor | None = None, accumulate: bool = False,
         symmetric: bool = False) -> torch.Tensor:
    """See module docstring.  ``a`` is (.., M, K) for K-major or (.., K, M) for M-major; ``b`` is
    (.., N, K) for K-major or (.., K, N) for N-major.  Leading dims are a batch.  ``symmetric``
    promises a symmetric result (e.g. X X^T): tiles above the diagonal are not computed and
    the lower triangle is mirrored onto them."""
    a_mn, b_mn = a_major == "mn", b_major == "mn"
    if not a.is_cuda:
        am = a.transpose(-1, -2) if a_mn else a
        bm = b.transpose(-1, -2) if b_mn else b
        res = alpha * (am.float() @ bm.float().transpose(-1, -2))
        if c is not None and beta != 0.0:
            res = res + beta * c.float()
        if out is None:
            return res.to(out_dtype)
        if accumulate:
            out.add_(res.to(out.dtype))
        else:
            out.copy_(res)
        return out
    m = a.shape[-1] if a_mn else a.shape[-2]
    n = b.shape[-1] if b_mn else b.shape[-2]
    if out is None:
        out = torch.empty(*a.shape[:-2], m, n, dtype=out_dtype, device=a.device)
    for name, t in (("a", a), ("b", b), ("out", out), ("c", c)):
        _check_tma_operand(name, t)
    ext().gemm(a, b, out, c, a_mn, b_mn, float(alpha), float(beta), bool(accumulate), bool(symmetric))
    return out


def _check_tma_operand(name: str, t: torch.Tensor | None) -> None:
    """The GEMM moves every operand with TMA: 16-byte aligned base, unit inner stride and
    row / batch strides that are multiples of 16 bytes (e.g. bf16 rows of a multiple of 8)."""
    if t is None:
        return
    es = t.element_size()
    ok = t.stride(-1) == 1 and t.data_ptr() % 16 == 0 and (t.stride(-2) * es) % 16 == 0 and \
        (t.dim() < 3 or t.size(0) == 1 or (t.stride(0) * es) % 16 == 0)
    if not ok:
        raise ValueError(f"gemm: operand {name} {tuple(t.shape)} strides {t.stride()} ({t.dtype}) does not meet the "
                         "TMA layout rules (unit inner stride, 16-byte aligned rows and base)")


_WEIGHT_EPOCH = [0]
# Forward linears with at most this many token rows (decode steps, small batches) use the
# split-K skinny GEMM, which streams the weight with every SM instead of a few output tiles.
SKINNY_MAX_ROWS = 64


def invalidate_weight_cache() -> None:
    """Called after every optimizer step: parameters updated by kernels (or by peers'
    stores into symmetric memory) do not bump PyTorch's version counters, so the cached
    bf16 copies are keyed on this epoch as well."""
    _WEIGHT_EPOCH[0] += 1


def bf16_weight(w: torch.Tensor) -> torch.Tensor:
    """bf16 copy of a (usually fp32 master) weight, cast once per parameter update."""
    if w.dtype == torch.bfloat16:
        return w if w.is_contiguous() else w.contiguous()
    cache = getattr(w, "_mykb_bf16", None)
    key = (w._version, _WEIGHT_EPOCH[0], w.data_ptr())
    if cache is not None and cache[0] == key:
        return cache[1]
    wd = w.detach()
    if wd.is_cuda and wd.dtype == torch.float32 and wd.is_contiguous() and wd.numel() % 4 == 0 \
            and wd.data_ptr() % 16 == 0:
        wb = ext().cast_bf16(wd)
    else:
        wb = wd.to(torch.bfloat16).contiguous()
    try:
        w._mykb_bf16 = (key, wb)
    except AttributeError:  # pragma: no cover - tensors that refuse attributes
        pass
    return wb


def _gemm_rows(t: torch.Tensor) -> torch.Tensor:
    """``t`` as the GEMM reads it: rows may be strided (a column slice of a wider matrix, read
    through the TMA row stride) as long as elements are contiguous and rows 16-byte aligned;
    anything else is copied."""
    if t.dim() == 2 and t.stride(-1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0:
        return t
    return t.contiguous()


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor):
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        wb = bf16_weight(w)
        if x2.shape[0] <= SKINNY_MAX_ROWS and k % 8 == 0:
            x2 = x2.contiguous()
            y = torch.empty(x2.shape[0], wb.shape[0], dtype=torch.bfloat16, device=x2.device)
            ext().gemm_skinny(x2, wb, y)
        else:
            x2 = _gemm_rows(x2)
            y = gemm(x2, wb)
        ctx.save_for_backward(x2, wb)
        ctx.w = w
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        x2, wb = ctx.saved_tensors
        w = ctx.w
        n = wb.shape[0]
        dy2 = dy.reshape(-1, n)
        if dy2.dtype != torch.bfloat16:
            dy2 = dy2.to(torch.bfloat16)
        dy2 = _gemm_rows(dy2)
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dy2, wb, b_major="mn").view(ctx.x_shape)
            if ctx.x_dtype != torch.bfloat16:
                dx = dx.to(ctx.x_dtype)
        if ctx.needs_input_grad[1]:
            main = getattr(w, "main_grad", None)
            if main is not None:
                gemm(dy2, x2, a_major="mn", b_major="mn", out=main, accumulate=True)
                w._mykb_grad_added = True
            else:
                dw = gemm(dy2, x2, a_major="mn", b_major="mn", out_dtype=torch.float32)
                if w.dtype != torch.float32:
                    dw = dw.to(w.dtype)
        return dx, dw


def linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """y = x W^T (no bias).  CUDA: bf16 tcgen05 GEMM, the block-scaled MXFP8 GEMMs for
    weights converted by ``convert_to_mxfp8_training``, or the float8 GEMMs for weights
    converted by ``convert_to_float8_training``; CPU: ``F.linear`` in x's dtype.  A weight
    row-sharded by the parameter-sharded runtime goes through its handle, whose GEMMs
    gather the weight from the other GPUs as they run."""
    shard = getattr(weight, "_mykb_shard", None)
    if shard is not None:  # a row-sharded weight of the parameter-sharded runtime
        return shard.linear(x, weight)
    if not x.is_cuda:
        return F.linear(x, weight.to(x.dtype))
    fmt = getattr(weight, "_mykb_mxfp8", None)
    if fmt is not None:
        from .mxfp8 import eligible_shapes, mx_linear

        if eligible_shapes(x, weight) and x.numel() // x.shape[-1] > SKINNY_MAX_ROWS:
            return mx_linear(x, weight, fmt)
    recipe = getattr(weight, "_mykb_fp8", None)
    if recipe is not None:
        from .float8 import eligible_shapes as fp8_eligible, fp8_linear

        if fp8_eligible(x, weight) and x.numel() // x.shape[-1] > SKINNY_MAX_ROWS:
            return fp8_linear(x, weight, recipe)
    return _Linear.apply(x, weight)
