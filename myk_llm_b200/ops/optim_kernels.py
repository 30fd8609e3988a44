"""Optimizer math on the GPU: Newton-Schulz orthogonalisation on the tcgen05 GEMM, a
multi-tensor AdamW kernel and the fused Muon momentum / update kernels.

Newton-Schulz follows the reference (``src/myk_llm/train/optim.py:17-32`` and
``src/myk_llm/ops/muon.py:218-268``): bf16, quintic coefficients (3.4445, -4.7750,
2.0315), Frobenius normalisation, tall matrices processed as their transpose.  Here the
transpose is never materialised: for a tall Y (r > c) the iteration is written on Y
itself, ``Y <- a Y + Y (b G + c G G)`` with ``G = Y^T Y``, which the GEMM expresses by
declaring Y MN-major.  ``G G`` uses the symmetry of G (its K-major and MN-major layouts
coincide) and the ``a X +`` / ``b G +`` terms ride in the GEMM epilogue (``beta * C``).
"""

from __future__ import annotations

import torch

from . import reference as ref
from ._ext import ext
from .linear import gemm

NS_COEFFICIENTS = ref.NS_COEFFICIENTS


def batched_syrk(x: torch.Tensor, alpha: float = 1.0, beta: float = 0.0, bias: torch.Tensor | None = None):
    """alpha * X X^T + beta * bias for a batch of bf16 matrices (B, r, c)."""
    if not x.is_cuda:
        out = alpha * (x.float() @ x.float().transpose(-1, -2))
        if bias is not None:
            out = out + beta * bias.float()
        return out.to(x.dtype)
    return gemm(x, x, alpha=alpha, beta=beta, c=bias, symmetric=bias is None and x.shape[-2] >= 2048)


def frobenius_normalize_(x: torch.Tensor, eps: float = 1e-7) -> torch.Tensor:
    """x /= max(||x||_F, eps) per matrix of a (B, r, c) batch, in place (bf16)."""
    if x.is_cuda:
        ext().frob_normalize_(x, float(eps))
        return x
    n = x.float().norm(dim=(-2, -1), keepdim=True).clamp(min=eps)
    x.copy_((x.float() / n).to(x.dtype))
    return x


def batched_newton_schulz_orthogonalize(g: torch.Tensor, steps: int, transposed: bool | None = None,
                                        eps: float = 1e-7) -> torch.Tensor:
    """Approximate U V^T of each matrix in ``g`` (B, r, c); returns bf16 (B, r, c)."""
    if g.dim() == 2:
        return batched_newton_schulz_orthogonalize(g[None], steps, transposed, eps)[0]
    if not g.is_cuda:
        return ref.newton_schulz_ref(g, steps, eps)
    a, b, c = NS_COEFFICIENTS
    x = g.to(torch.bfloat16).contiguous() if g.dtype != torch.bfloat16 else g.clone()
    frobenius_normalize_(x, eps)
    r, cdim = x.shape[-2], x.shape[-1]
    tall = (r > cdim) if transposed is None else transposed
    # The Gram matrix and the polynomial in it are symmetric, so their tiles above the
    # diagonal can be skipped and mirrored.  Measured on B200 this pays for wide matrices
    # (2048 x 11264: 1.5x per iteration) and not for near-square ones (aspect <= 3, where
    # the mirror pass and uneven tile counts cost what the skipped tiles save).
    sym = min(r, cdim) >= 2048 and max(r, cdim) >= 4 * min(r, cdim)
    for _ in range(steps):
        if tall:
            gram = gemm(x, x, a_major="mn", b_major="mn", symmetric=sym)  # (c, c) = Y^T Y
            poly = gemm(gram, gram, alpha=c, beta=b, c=gram, symmetric=sym)
            x = gemm(x, poly, alpha=1.0, beta=a, c=x)  # Y poly (poly symmetric)
        else:
            gram = gemm(x, x, symmetric=sym)  # (r, r) = X X^T
            poly = gemm(gram, gram, alpha=c, beta=b, c=gram, symmetric=sym)
            x = gemm(poly, x, b_major="mn", alpha=1.0, beta=a, c=x)
    return x


# ---------------------------------------------------------------------------------------
# AdamW
# ---------------------------------------------------------------------------------------
def adamw_multi_tensor(params, grads, exp_avgs, exp_avg_sqs, step: int, lr: float, beta1: float, beta2: float,
                       eps: float, weight_decay: float, grad_scale: torch.Tensor | None = None) -> None:
    """One AdamW step (torch.optim.AdamW semantics, decoupled decay) over lists of fp32
    tensors, in a single kernel launch on CUDA.  ``grad_scale`` (a one-element fp32 device
    tensor, e.g. the clipping coefficient) multiplies every gradient as it is read."""
    if not params:
        return
    if not params[0].is_cuda:
        for p, g, m, v in zip(params, grads, exp_avgs, exp_avg_sqs):
            g = g.to(p.dtype) if grad_scale is None else g.to(p.dtype) * grad_scale
            ref.adamw_ref(p, g, m, v, step, lr, beta1, beta2, eps, weight_decay)
        return
    ext().adamw_step(params, grads, exp_avgs, exp_avg_sqs, int(step), float(lr), float(beta1), float(beta2),
                     float(eps), float(weight_decay), _scale(grad_scale))


def _scale(t: torch.Tensor | None) -> torch.Tensor | None:
    return None if t is None else t.reshape(1).to(torch.float32).contiguous()


# ---------------------------------------------------------------------------------------
# Muon momentum / update
# ---------------------------------------------------------------------------------------
def muon_prepare(grads, bufs, momentum: float, nesterov: bool, out: torch.Tensor,
                 grad_scale: torch.Tensor | None = None) -> None:
    """buf <- lerp(buf, g, 1-mu); u = lerp(g, buf, mu) if nesterov else buf; out[i] = bf16(u).
    ``out`` is a (n, r, c) bf16 stack; ``grad_scale`` multiplies g as it is read."""
    if out.is_cuda:
        ext().muon_prepare(grads, bufs, float(momentum), bool(nesterov), out, _scale(grad_scale))
        return
    for i, (g, m) in enumerate(zip(grads, bufs)):
        if grad_scale is not None:
            g = g.to(m.dtype) * grad_scale
        m.lerp_(g.to(m.dtype), 1 - momentum)
        u = g.to(m.dtype).lerp(m, momentum) if nesterov else m
        out[i].copy_(u)


def muon_apply(params, orth: torch.Tensor, lr: float, weight_decay: float, step_scale: float) -> None:
    """p <- p * (1 - lr*wd) + step_scale * orth[i]."""
    if orth.is_cuda:
        ext().muon_apply(params, orth, float(lr * weight_decay), float(step_scale))
        return
    for i, p in enumerate(params):
        p.mul_(1 - lr * weight_decay)
        p.add_(orth[i].to(p.dtype), alpha=step_scale)
