"""Float8 training linears with dynamic per-tensor or per-row scaling.

The reference's ``parallel.float8`` accepts the torchao recipes ``tensorwise``, ``rowwise``
and ``rowwise_with_gw_hp`` besides ``mxfp8`` (``src/myk_llm/train/config.py:113``,
``src/myk_llm/train/distributed.py:71-105``).  This module is this framework's own
implementation of those three scaling statements for the three GEMMs of a linear layer
(``y = x W^T``, ``dx = dy W``, ``dW = dy^T x``):

* ``tensorwise``: one scale per operand tensor, ``amax / fp8_max``.  ``x`` and ``W`` are
  E4M3, the output gradient ``dy`` is E5M2 (its wider range holds gradient outliers).
* ``rowwise``: one scale per row of each operand along the GEMM's reduction dimension,
  rounded to a power of two; every operand is E4M3.  Each GEMM needs its operands scaled
  along its own reduction axis, so ``W`` is also quantized column-wise for ``dx`` and
  ``dy`` / ``x`` column-wise (over tokens) for ``dW``.
* ``rowwise_with_gw_hp``: ``y`` and ``dx`` as in ``rowwise``; ``dW`` stays a bf16 GEMM
  (the weight gradient keeps high precision), accumulated into ``main_grad`` by the
  tcgen05 GEMM epilogue when the parameter has one.

Activations and gradients are quantised by this framework's kernels (``csrc/fp8.cu``: a
fused per-row amax+cast, a per-tensor amax then cast, and a per-column amax then
transposing cast for the weight-gradient operands).  The float8 GEMMs are this
framework's tcgen05 block-scaled GEMM (``csrc/mxfp8.cu``) run with unit block scales, the
per-tensor / per-row dequantisation scales applied to the fp32 accumulator in its
epilogue (``fp8_scaled_gemm``).  On the CPU the same
statement ``(a * s_a) @ (b * s_b)`` is evaluated in fp32, so the CPU tests check the
scaling rules exactly.  The quantised weight (both orientations) is cached on the
parameter and rebuilt after each optimizer step, like the bf16 weight copy of the plain
linear.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.nn as nn

RECIPES = ("tensorwise", "rowwise", "rowwise_with_gw_hp")
E4M3, E5M2 = torch.float8_e4m3fn, torch.float8_e5m2
_FP8_MAX = {E4M3: 448.0, E5M2: 57344.0}
_AMAX_EPS = 1e-12


def quantize(x: torch.Tensor, dtype: torch.dtype, rowwise: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(fp8 values, fp32 dequantisation scale) of a 2-D tensor.  ``rowwise`` gives one scale
    per row (shape (R, 1), a power of two) over the last dimension; otherwise one scalar
    scale for the whole tensor.  ``x ~= q.float() * scale``."""
    fmax = _FP8_MAX[dtype]
    a = x.abs()
    amax = (a.amax(dim=-1, keepdim=True) if rowwise else a.amax()).float().clamp_min(_AMAX_EPS)
    inv = fmax / amax
    if rowwise:   # keep the exponent bits alone: inv rounded down to a power of two
        inv = (inv.view(torch.int32) & 0x7F800000).view(torch.float32)
    q = (x.float() * inv).clamp_(-fmax, fmax).to(dtype)
    return q, inv.reciprocal()


def _kernel_ok(x: torch.Tensor) -> bool:
    return (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous()
            and x.shape[1] % 8 == 0 and x.data_ptr() % 16 == 0)


def quantize_act(x: torch.Tensor, dtype: torch.dtype, rowwise: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """:func:`quantize` of an activation or gradient; contiguous bf16 CUDA tensors go through
    the fused quantiser kernels (``csrc/fp8.cu``), which compute the same statement."""
    if _kernel_ok(x):
        from ._ext import ext

        e5 = dtype == E5M2
        return tuple(ext().fp8_quant_rows(x, e5, True) if rowwise else ext().fp8_quant_tensor(x, e5))
    return quantize(x, dtype, rowwise)


def quantize_act_t(x: torch.Tensor, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row :func:`quantize` of ``x^T`` (one scale per column of ``x``), written transposed;
    the fused column-amax + transposing cast kernels for contiguous bf16 CUDA tensors."""
    if _kernel_ok(x) and x.shape[0] % 16 == 0:
        from ._ext import ext

        return tuple(ext().fp8_quant_cols_t(x, dtype == E5M2, True))
    return quantize(x.t().contiguous(), dtype, True)


_UNIT_ATOMS: dict[tuple, torch.Tensor] = {}


def _unit_atoms(rows: int, k: int, device) -> torch.Tensor:
    """Block-scale atoms of value 2^0 (E8M0 127) for an fp8 operand of ``rows`` x ``k``."""
    key = ((rows + 127) // 128, k // 128, str(device))
    atoms = _UNIT_ATOMS.get(key)
    if atoms is None:
        atoms = _UNIT_ATOMS[key] = torch.full((key[0] * key[1] * 512,), 127, dtype=torch.uint8, device=device)
    return atoms


def scaled_mm(a: torch.Tensor, sa: torch.Tensor, b: torch.Tensor, sb: torch.Tensor,
              out_dtype: torch.dtype) -> torch.Tensor:
    """``(a * sa) @ (b * sb)^T`` for fp8 ``a`` (M, K) and ``b`` (N, K), both K-contiguous;
    ``sa`` is a scalar or (M, 1), ``sb`` a scalar or (N, 1).  CUDA: the tcgen05 block-scaled
    GEMM with unit block scales and the per-tensor / per-row scales applied in its
    epilogue (``fp8_scaled_gemm``); K must be a multiple of 128 (``eligible_shapes``)."""
    if not a.is_cuda:
        return ((a.float() * sa) @ (b.float() * sb).t()).to(out_dtype)
    from ._ext import ext

    m, k = a.shape
    n = b.shape[0]
    if k % 128:
        raise ValueError(f"float8 GEMM needs the reduction size to be a multiple of 128, got {k}")
    d = torch.empty(m, n, dtype=out_dtype, device=a.device)
    ext().fp8_scaled_gemm(a.contiguous().view(torch.uint8), _unit_atoms(m, k, a.device), a.dtype == E5M2,
                          b.contiguous().view(torch.uint8), _unit_atoms(n, k, b.device), b.dtype == E5M2,
                          sa.reshape(-1).float().contiguous(), sb.reshape(-1).float().contiguous(), d)
    return d


class _WeightCache:
    """Quantised copies of one weight for the current parameter version: ``(q, s)`` with the
    reduction over K (forward) and ``(qt, st)`` of ``W^T`` with the reduction over N (``dx``)."""

    @staticmethod
    def get(w: torch.Tensor, rowwise: bool):
        from .linear import _WEIGHT_EPOCH

        key = (w._version, _WEIGHT_EPOCH[0], w.data_ptr(), rowwise)
        cache = getattr(w, "_mykb_fp8_cache", None)
        if cache is not None and cache[0] == key:
            return cache[1]
        wd = w.detach()
        if rowwise:
            q, s = quantize(wd, E4M3, True)
            qt, st = quantize(wd.t().contiguous(), E4M3, True)
        else:
            q, s = quantize(wd, E4M3, False)
            qt, st = q.t().contiguous(), s
        val = (q, s, qt, st)
        try:
            w._mykb_fp8_cache = (key, val)
        except AttributeError:  # pragma: no cover - tensors that refuse attributes
            pass
        return val


class _Fp8Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor, recipe: str):
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        rowwise = recipe != "tensorwise"
        q, s, qt, st = _WeightCache.get(w, rowwise)
        xq, xs = quantize_act(x2, E4M3, rowwise)
        y = scaled_mm(xq, xs, q, s, torch.bfloat16)
        ctx.recipe, ctx.w = recipe, w
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        if recipe == "tensorwise":
            ctx.save_for_backward(xq, xs)   # reused for dW: scalar scale, any orientation
        else:
            ctx.save_for_backward(x2)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        w, recipe = ctx.w, ctx.recipe
        n = w.shape[0]
        dy2 = dy.reshape(-1, n).contiguous()
        rowwise = recipe != "tensorwise"
        _, _, qt, st = _WeightCache.get(w, rowwise)
        dx = dw = None
        if recipe == "tensorwise":
            xq, xs = ctx.saved_tensors
            gq, gs = quantize_act(dy2, E5M2, False)
            if ctx.needs_input_grad[0]:
                dx = scaled_mm(gq, gs, qt, st, torch.bfloat16)
            if ctx.needs_input_grad[1]:
                dw = scaled_mm(gq.t().contiguous(), gs, xq.t().contiguous(), xs, torch.float32)
        else:
            (x2,) = ctx.saved_tensors
            if ctx.needs_input_grad[0]:
                gq, gs = quantize_act(dy2, E4M3, True)
                dx = scaled_mm(gq, gs, qt, st, torch.bfloat16)
            if ctx.needs_input_grad[1]:
                if recipe == "rowwise":
                    gtq, gts = quantize_act_t(dy2, E4M3)
                    xtq, xts = quantize_act_t(x2, E4M3)
                    dw = scaled_mm(gtq, gts, xtq, xts, torch.bfloat16).float()
                else:
                    dw = _high_precision_wgrad(dy2, x2, w)
        if dx is not None:
            dx = dx.view(ctx.x_shape).to(ctx.x_dtype)
        if dw is not None:
            main = getattr(w, "main_grad", None)
            if main is not None:
                main.add_(dw)
                w._mykb_grad_added = True
                dw = None
            else:
                dw = dw.to(w.dtype)
        return dx, dw, None


def _high_precision_wgrad(dy2: torch.Tensor, x2: torch.Tensor, w: torch.Tensor) -> torch.Tensor | None:
    """bf16 ``dy^T x`` in fp32.  On CUDA this is the tcgen05 GEMM, which accumulates straight
    into ``main_grad`` when the parameter has one; then None is returned (nothing to add)."""
    from .linear import _gemm_rows, gemm

    g = dy2.to(torch.bfloat16)
    xb = x2.to(torch.bfloat16)
    if not g.is_cuda:
        return g.float().t() @ xb.float()
    g, xb = _gemm_rows(g), _gemm_rows(xb)
    main = getattr(w, "main_grad", None)
    if main is not None:
        gemm(g, xb, a_major="mn", b_major="mn", out=main, accumulate=True)
        w._mykb_grad_added = True
        return None
    return gemm(g, xb, a_major="mn", b_major="mn", out_dtype=torch.float32)


def fp8_linear(x: torch.Tensor, w: torch.Tensor, recipe: str) -> torch.Tensor:
    """y = x W^T with float8 operands under ``recipe`` (one of :data:`RECIPES`)."""
    if recipe not in RECIPES:
        raise ValueError(f"float8 recipe must be one of {RECIPES}, got {recipe!r}")
    return _Fp8Linear.apply(x, w, recipe)


def eligible_shapes(x: torch.Tensor, w: torch.Tensor) -> bool:
    """The tcgen05 float8 GEMMs reduce over K (forward), N (data gradient) and the token
    count M (weight gradient) in blocks of 128, so all three must be multiples of 128;
    other linears stay in bf16."""
    rows = x.numel() // max(x.shape[-1], 1)
    return w.shape[0] % 128 == 0 and w.shape[1] % 128 == 0 and x.shape[-1] == w.shape[1] and rows % 128 == 0


class Float8Linear(nn.Linear):
    """An ``nn.Linear`` whose three matmuls run in float8 (same parameters and state dict)."""

    fp8_recipe = "tensorwise"

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from .linear import linear

        y = linear(x, self.weight)
        return y + self.bias if self.bias is not None else y


def convert_to_float8_training(model: nn.Module, recipe: str,
                               module_filter_fn: Callable[[nn.Module, str], bool] | None = None) -> int:
    """Turn eligible ``nn.Linear`` modules into :class:`Float8Linear` in place; their weights
    are routed through :func:`fp8_linear` by :func:`myk_llm_b200.ops.linear`.  Returns the
    number converted (the count the reference's ``convert_float8`` reports)."""
    if recipe not in RECIPES:
        raise ValueError(f"float8 recipe must be one of {RECIPES}, got {recipe!r}")
    n = 0
    for fqn, mod in model.named_modules():
        if type(mod) is not nn.Linear or (module_filter_fn is not None and not module_filter_fn(mod, fqn)):
            continue
        mod.__class__ = Float8Linear
        mod.fp8_recipe = recipe
        mod.weight._mykb_fp8 = recipe
        n += 1
    return n
