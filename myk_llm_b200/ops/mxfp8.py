"""MXFP8 training linears: block-scaled fp8 GEMMs on tcgen05 (``csrc/mxfp8.cu``).

Every eligible linear computes, with 1 x 32 blocks of fp8 sharing one power-of-two
(E8M0) scale along each GEMM's reduction dimension:

* forward  ``y = x W^T``      x and W quantized along K;
* dgrad    ``dx = dy W``      dy along N (grad format) x W^T along N;
* wgrad    ``dW = dy^T x``    dy^T and x^T along the token dimension, accumulated in fp32
  into the parameter's ``main_grad`` (or returned).

One pass of :func:`mx_quantize` produces both the row-blocked and the transposed,
column-blocked copy of a matrix.  Scales round up (RCEIL, ``2^ceil(log2(amax/fp8_max))``)
so no element overflows; elements round to nearest even.  Forward operands are E4M3;
gradients are E4M3 (the reference's choice, ``src/myk_llm/ops/mxfp8.py:118-157``) or E5M2
(``parallel.mxfp8_grad_dtype``).  Parameters stay plain fp32 tensors, so checkpoints
are the same as bf16 runs; a converted linear is marked through its weight and
:func:`myk_llm_b200.ops.linear` routes it here.  Weights are quantized once per optimizer
step (cached like the bf16 weight copies).

Token counts that are not a multiple of 128 are zero-padded for the GEMMs; linears whose
feature dimensions are not multiples of 128 stay bf16.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.nn as nn

from ._ext import ext

FP8_MAX = {"e4m3": 448.0, "e5m2": 57344.0}
TORCH_FP8 = {"e4m3": torch.float8_e4m3fn, "e5m2": torch.float8_e5m2}


# ------------------------------------------------------------------ torch statement
def block_exponents(x: torch.Tensor, fmt: str) -> torch.Tensor:
    """E8M0 exponents (unbiased, int) of the 1 x 32 blocks along the last dim:
    ceil(log2(amax / fp8_max)), computed exactly from the float bits; amax 0 -> -127."""
    xf = x.float().reshape(*x.shape[:-1], x.shape[-1] // 32, 32)
    q = xf.abs().amax(-1) / FP8_MAX[fmt]
    mant, ex = torch.frexp(q)  # q = mant * 2^ex, mant in [0.5, 1)
    e = torch.where(mant == 0.5, ex - 1, ex)
    e = torch.where(q == 0, torch.full_like(e, -127), e)
    return e.clamp(-127, 127)


def quantize_ref(x: torch.Tensor, fmt: str = "e4m3") -> tuple[torch.Tensor, torch.Tensor]:
    """(fp8 values (torch float8 dtype), exponents) of 1 x 32 blocks along the last dim."""
    e = block_exponents(x, fmt)
    scale = torch.exp2(e.float()).repeat_interleave(32, -1)
    q = (x.float() / scale).to(TORCH_FP8[fmt])
    return q, e


def dequantize_ref(q: torch.Tensor, e: torch.Tensor) -> torch.Tensor:
    return q.float() * torch.exp2(e.float()).repeat_interleave(32, -1)


def atoms_to_exponents(atoms: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """Unbiased exponents (rows, k / 32) from the kernel's 512-byte scale atoms."""
    r = torch.arange(rows, device=atoms.device)[:, None]
    kb = torch.arange(k // 32, device=atoms.device)[None, :]
    off = ((r // 128) * (k // 128) + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
    return atoms.long()[off] - 127


# ------------------------------------------------------------------ kernels
def mx_quantize(x: torch.Tensor, fmt: str = "e4m3", dim0: bool = True, dim1: bool = False) -> list[torch.Tensor]:
    """bf16 (R, C) -> [q0 (R, C), s0] and/or [q1 (C, R), s1]: fp8 bits (uint8) and scale
    atoms for the row-blocked matrix and for its transpose blocked along R."""
    return ext().mx_quantize(x.contiguous(), fmt == "e5m2", dim0, dim1)


def mx_gemm(a, sa, a_fmt: str, b, sb, b_fmt: str, out: torch.Tensor | None = None,
            out_dtype: torch.dtype = torch.bfloat16, accumulate: bool = False) -> torch.Tensor:
    """(M, K) x (N, K)^T on fp8 operands from :func:`mx_quantize`."""
    if out is None:
        out = torch.empty(a.shape[0], b.shape[0], dtype=out_dtype, device=a.device)
    ext().mx_gemm(a, sa, a_fmt == "e5m2", b, sb, b_fmt == "e5m2", out, bool(accumulate))
    return out


# ------------------------------------------------------------------ linear
def _weight_operands(w: torch.Tensor) -> list[torch.Tensor]:
    """[W q0, s0, W^T q1, s1] (E4M3), re-quantized when the weight changed."""
    from .linear import _WEIGHT_EPOCH, bf16_weight

    shard = getattr(w, "_mykb_shard", None)
    if shard is not None:  # row-sharded by the parameter-sharded runtime: gathered in fp8
        return shard.mx_operands()
    key = (w._version, _WEIGHT_EPOCH[0], w.data_ptr())
    cache = getattr(w, "_mykb_mx", None)
    if cache is not None and cache[0] == key:
        return cache[1]
    ops = mx_quantize(bf16_weight(w), "e4m3", dim0=True, dim1=True)
    w._mykb_mx = (key, ops)
    return ops


def _pad_rows(x: torch.Tensor, multiple: int = 128) -> torch.Tensor:
    pad = (-x.shape[0]) % multiple
    return x if pad == 0 else torch.cat([x, x.new_zeros(pad, x.shape[1])])


class _MXLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, w: torch.Tensor, grad_fmt: str):
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        m = x2.shape[0]
        xp = _pad_rows(x2.to(torch.bfloat16))
        xq, xs, xtq, xts = mx_quantize(xp, "e4m3", dim0=True, dim1=True)
        wq, ws, wtq, wts = _weight_operands(w)
        y = mx_gemm(xq, xs, "e4m3", wq, ws, "e4m3")[:m]
        ctx.save_for_backward(xtq, xts, wtq, wts)
        ctx.w, ctx.m, ctx.grad_fmt = w, m, grad_fmt
        ctx.x_shape, ctx.x_dtype = x.shape, x.dtype
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        xtq, xts, wtq, wts = ctx.saved_tensors
        w, m, gf = ctx.w, ctx.m, ctx.grad_fmt
        dy2 = _pad_rows(dy.reshape(-1, w.shape[0]).to(torch.bfloat16))
        dq, ds, dtq, dts = mx_quantize(dy2, gf, dim0=True, dim1=True)
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = mx_gemm(dq, ds, gf, wtq, wts, "e4m3")[:m].view(ctx.x_shape)
            if ctx.x_dtype != torch.bfloat16:
                dx = dx.to(ctx.x_dtype)
        if ctx.needs_input_grad[1]:
            main = getattr(w, "main_grad", None)
            if main is not None:
                mx_gemm(dtq, dts, gf, xtq, xts, "e4m3", out=main, accumulate=True)
                w._mykb_grad_added = True
            else:
                dw = mx_gemm(dtq, dts, gf, xtq, xts, "e4m3", out_dtype=torch.float32)
                if w.dtype != torch.float32:
                    dw = dw.to(w.dtype)
        return dx, dw, None


def eligible_shapes(x: torch.Tensor, w: torch.Tensor) -> bool:
    return x.is_cuda and w.shape[0] % 128 == 0 and w.shape[1] % 128 == 0 and x.shape[-1] == w.shape[1]


def mx_linear(x: torch.Tensor, w: torch.Tensor, grad_fmt: str = "e4m3") -> torch.Tensor:
    """y = x W^T with MXFP8 operands (forward E4M3, gradients ``grad_fmt``)."""
    return _MXLinear.apply(x, w, grad_fmt)


class MXFP8Linear(nn.Linear):
    """An ``nn.Linear`` whose matmuls run in MXFP8 (same parameters and state dict)."""

    mx_grad_dtype = "e4m3"

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from .linear import linear

        y = linear(x, self.weight)
        return y + self.bias if self.bias is not None else y


def convert_to_mxfp8_training(model: nn.Module, module_filter_fn: Callable[[nn.Module, str], bool] | None = None,
                              grad_dtype: str = "e4m3") -> int:
    """Turn eligible ``nn.Linear`` modules into :class:`MXFP8Linear` in place (their weights
    get routed through the MXFP8 GEMMs by :func:`myk_llm_b200.ops.linear`).  Returns the
    number converted.  The interface of the reference's ``convert_to_mxfp8_training``
    (``src/myk_llm/ops/mxfp8.py:200-212``)."""
    if grad_dtype not in FP8_MAX:
        raise ValueError(f"grad_dtype must be e4m3 or e5m2, got {grad_dtype!r}")
    n = 0
    for fqn, mod in model.named_modules():
        if type(mod) is not nn.Linear or (module_filter_fn is not None and not module_filter_fn(mod, fqn)):
            continue
        mod.__class__ = MXFP8Linear
        mod.mx_grad_dtype = grad_dtype
        mod.weight._mykb_mxfp8 = grad_dtype
        n += 1
    return n
