"""Fused linear + cross-entropy + z-loss.

``fused_linear_cross_entropy(hidden, weight, targets, normalizer, z_loss)`` returns
``(loss, ce_sum, z_sum)`` with ``loss = (sum CE + z_loss * sum lse^2) / normalizer`` over
supervised targets (``ignore_index`` rows contribute nothing), as in the reference
(``src/myk_llm/ops/fused_ce.py:111-140``).

Like the reference, the gradients are produced during the forward pass and scaled by the
incoming gradient in backward, so the (tokens, vocab) logits never exist all at once.
Per chunk of rows, on CUDA:

1. ``logits = h W^T`` on the tcgen05 GEMM (bf16 out);
2. one kernel (``csrc/loss.cu``) computes each row's log-sum-exp in fp32, the CE and z
   terms, and overwrites the logits with ``(softmax * (1 + 2 z lse) - onehot) / normalizer``;
3. ``dh = G W`` and ``dW += G^T h`` on the tcgen05 GEMM, the latter accumulated in fp32
   straight into the weight's gradient buffer.
"""

from __future__ import annotations

import torch

from . import reference as ref
from ._ext import ext
from .linear import bf16_weight, gemm


class _FusedLinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, normalizer, z_coef, ignore_index, chunk_size):
        n, hdim = hidden.shape
        vocab = weight.shape[0]
        hb = hidden if hidden.dtype == torch.bfloat16 else hidden.to(torch.bfloat16)
        hb = hb.contiguous()
        wb = bf16_weight(weight)
        main = getattr(weight, "main_grad", None)
        grad_w = main if main is not None else torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        grad_h = torch.empty(n, hdim, dtype=torch.bfloat16, device=hidden.device)
        ce = torch.zeros((), dtype=torch.float32, device=hidden.device)
        zs = torch.zeros((), dtype=torch.float32, device=hidden.device)
        logits = torch.empty(min(chunk_size, n), vocab, dtype=torch.bfloat16, device=hidden.device)
        scale = 1.0 / float(normalizer)
        for start in range(0, n, chunk_size):
            end = min(n, start + chunk_size)
            rows = end - start
            lg = logits[:rows]
            h_c = hb[start:end]
            gemm(h_c, wb, out=lg)
            ext().ce_fwd_grad(lg, targets[start:end], float(scale), float(z_coef), int(ignore_index), ce, zs)
            gemm(lg, wb, b_major="mn", out=grad_h[start:end])
            gemm(lg, h_c, a_major="mn", b_major="mn", out=grad_w, accumulate=True)
        loss = (ce + z_coef * zs) * scale
        ctx.has_main = main is not None
        ctx.weight = weight
        ctx.save_for_backward(grad_h, grad_w if main is None else torch.empty(0))
        ctx.hidden_dtype = hidden.dtype
        return loss, ce, zs

    @staticmethod
    def backward(ctx, grad_loss, _g_ce, _g_z):
        grad_h, grad_w = ctx.saved_tensors
        # in place, scale applied in fp32 (a 0-dim fp32 factor keeps the bf16 result dtype);
        # no host synchronisation anywhere in this backward
        gh = grad_h.mul_(grad_loss)
        if gh.dtype != ctx.hidden_dtype:
            gh = gh.to(ctx.hidden_dtype)
        if ctx.has_main:
            # The weight gradient was accumulated into main_grad during forward, which is
            # only right for an unscaled loss (loss.backward()).  Count violations on the
            # device; check_unscaled_main_grad() reports them at the next logging sync.
            _scale_errors(grad_loss.device).add_((grad_loss != 1).to(torch.int32))
            return gh, None, None, None, None, None, None
        gw = (grad_w * grad_loss).to(ctx.weight.dtype)
        return gh, gw, None, None, None, None, None


_SCALE_ERRORS: dict[torch.device, torch.Tensor] = {}


def _scale_errors(device: torch.device) -> torch.Tensor:
    t = _SCALE_ERRORS.get(device)
    if t is None:
        t = _SCALE_ERRORS[device] = torch.zeros((), dtype=torch.int32, device=device)
    return t


def check_unscaled_main_grad() -> None:
    """Raise if a fused CE whose weight gradient goes straight into ``main_grad`` was
    back-propagated with a scaled loss since the last call (synchronises the device)."""
    for t in _SCALE_ERRORS.values():
        if int(t.item()):
            t.zero_()
            raise RuntimeError("fused CE with a main_grad buffer needs an unscaled loss.backward()")


def fused_linear_cross_entropy(hidden, weight, targets, normalizer, z_loss=0.0, ignore_index=-100, chunk_size=8192):
    """Returns (loss, ce_sum, z_sum); see module docstring."""
    if not hidden.is_cuda:
        return ref.linear_cross_entropy_ref(hidden, weight.to(hidden.dtype), targets, normalizer, z_loss)
    h = hidden.reshape(-1, hidden.size(-1))
    t = targets.reshape(-1)
    if t.dtype != torch.int64:
        t = t.long()
    return _FusedLinearCE.apply(h, weight, t.contiguous(), float(normalizer), float(z_loss), ignore_index,
                                max(128, int(chunk_size)))
