"""Training objectives, run as the model's ``head`` callback inside forward: next-token
cross entropy with z-loss, multi-token prediction (MTP) and logit distillation from a
frozen teacher.

Every loss is divided by one normaliser, the number of supervised next-token targets of
the whole optimizer step (all micro-batches of all ranks), so gradient accumulation and
data parallelism give the exact per-token mean (the reference's convention,
``src/myk_llm/train/objectives.py:83-117``).

The losses follow the fused cross-entropy's pattern: the gradients with respect to the
hidden states and the output weight are produced while the loss is computed (chunk by
chunk, so at most one chunk of logits is alive) and the backward pass only scales them.
The CE and MTP heads are ``ops.fused_linear_cross_entropy``; the distillation KL is
``_DistillKL`` below.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F

from .. import ops
from ..data.config import IGNORE_INDEX, Batch
from ..models import ModelOutput, MykLLM
from .config import DistillConfig, ObjectiveConfig


@dataclass
class LossOutput:
    loss: torch.Tensor
    sums: dict[str, torch.Tensor] = field(default_factory=dict)  # detached per-token sums for logging


def mtp_targets(targets: torch.Tensor, depth: int) -> torch.Tensor:
    """Targets of MTP head ``depth``: position ``i`` predicts token ``i + 1 + depth``.  A
    position is supervised only if all ``depth + 1`` next-token targets ``i .. i + depth``
    are (the window crosses no document seam and no prompt token)."""
    padded = F.pad(targets, (0, depth), value=IGNORE_INDEX)
    windows = padded.unfold(-1, depth + 1, 1)  # (..., seq, depth + 1)
    ok = (windows != IGNORE_INDEX).all(-1)
    return torch.where(ok, windows[..., depth], torch.full_like(targets, IGNORE_INDEX))


class Teacher:
    """A frozen HuggingFace causal LM: its decoder's last hidden states and its output
    embedding, restricted to the student's vocabulary by ``row_map`` (``row_map[new] =
    old``) when the student uses a pruned tokenizer."""

    def __init__(self, config: DistillConfig, device: torch.device) -> None:
        from transformers import AutoModelForCausalLM

        lm = AutoModelForCausalLM.from_pretrained(config.teacher, dtype=torch.bfloat16)
        lm = lm.to(device).eval().requires_grad_(False)
        self.decoder = lm.get_decoder()
        head = lm.get_output_embeddings().weight.detach()
        if config.row_map:
            rows = torch.as_tensor(np.load(config.row_map), dtype=torch.long, device=device)
            head = head[rows]
        self.weight = head

    @torch.no_grad()
    def hidden(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.decoder(input_ids=input_ids).last_hidden_state


class _DistillKL(torch.autograd.Function):
    """``sum_valid T^2 KL(teacher || student)`` with student logits ``h W^T / T``.  Per
    chunk of rows: both log-softmaxes in fp32, the KL, and the gradient of the KL with
    respect to the student logits, ``T (softmax(s) - softmax(t))`` (times the valid mask),
    turned into ``dh`` and ``dW`` right away; backward scales them by the incoming
    gradient.  Nothing of size (rows, vocab) outlives its chunk."""

    @staticmethod
    def forward(ctx, hidden, weight, teacher_hidden, teacher_weight, valid, temperature: float, chunk: int):
        t = float(temperature)
        w32 = weight.detach()
        dh = torch.zeros_like(hidden, dtype=torch.float32)
        dw = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        total = torch.zeros((), dtype=torch.float32, device=hidden.device)
        for a in range(0, hidden.shape[0], chunk):
            h, th, m = hidden[a:a + chunk], teacher_hidden[a:a + chunk], valid[a:a + chunk].float()
            s_log = F.log_softmax(ops.linear(h.detach(), w32).float() / t, dim=-1)
            t_log = F.log_softmax((th @ teacher_weight.t()).float() / t, dim=-1)
            t_prob = t_log.exp()
            total += ((t_prob * (t_log - s_log)).sum(-1) * m).sum() * (t * t)
            g = (s_log.exp() - t_prob) * (m * t).unsqueeze(-1)  # d(T^2 KL) / d(student logits)
            dh[a:a + chunk] = g @ w32.float()
            dw += g.t() @ h.detach().float()
        ctx.save_for_backward(dh, dw)
        ctx.dtypes = (hidden.dtype, weight.dtype)
        return total

    @staticmethod
    def backward(ctx, grad):
        dh, dw = ctx.saved_tensors
        return (dh * grad).to(ctx.dtypes[0]), (dw * grad).to(ctx.dtypes[1]), None, None, None, None, None


def distillation_kl_sum(hidden, weight, teacher_hidden, teacher_weight, valid, temperature: float,
                        chunk_size: int) -> torch.Tensor:
    return _DistillKL.apply(hidden, weight, teacher_hidden, teacher_weight, valid, temperature, chunk_size)


def _ce_chunk(cfg: ObjectiveConfig, h: torch.Tensor) -> int:
    # On B200 the logits GEMMs need large chunks to fill the 148 SMs; the chunk only bounds
    # the transient (chunk x vocab) bf16 logits buffer.
    return max(cfg.loss_chunk_size, 8192) if h.is_cuda else cfg.loss_chunk_size


class StepLoss:
    """The ``head`` callback of one micro-batch: every configured loss, normalised by the
    step's global target count."""

    def __init__(self, objective: "Objective", batch: Batch, normalizer: float) -> None:
        self.objective, self.batch, self.normalizer = objective, batch, normalizer

    def __call__(self, model: MykLLM, out: ModelOutput) -> LossOutput:
        cfg, teacher, batch, norm = self.objective.config, self.objective.teacher, self.batch, self.normalizer
        w = model.output_weight
        sums: dict[str, torch.Tensor] = {}
        ce_weight = 1.0 - cfg.distill.weight if teacher is not None else 1.0
        loss, sums["ce"], sums["z"] = ops.fused_linear_cross_entropy(
            out.hidden, w, batch.targets, norm / ce_weight, cfg.z_loss, chunk_size=_ce_chunk(cfg, out.hidden))
        if teacher is not None:
            flat = out.hidden.reshape(-1, out.hidden.shape[-1])
            valid = (batch.targets != IGNORE_INDEX).reshape(-1)
            kl = distillation_kl_sum(flat, w, teacher.hidden(batch.input_ids).reshape(flat.shape[0], -1),
                                     teacher.weight, valid, cfg.distill.temperature, cfg.distill.chunk_size)
            loss = loss + kl * (cfg.distill.weight / norm)
            sums["kl"] = kl.detach()
        if cfg.mtp_weight > 0:
            for depth, h in enumerate(model.mtp_hidden(out, batch.input_ids), start=1):
                extra, sums[f"mtp{depth}_ce"], _ = ops.fused_linear_cross_entropy(
                    h, w, mtp_targets(batch.targets, depth), norm / cfg.mtp_weight, chunk_size=_ce_chunk(cfg, h))
                loss = loss + extra
        return LossOutput(loss, sums)


class Objective:
    """Holds the objective config and the (optional) teacher; ``head(batch, normalizer)``
    returns the callback the model runs on its final hidden states."""

    def __init__(self, config: ObjectiveConfig, device: torch.device) -> None:
        self.config = config
        self.teacher = Teacher(config.distill, device) if config.distill.teacher else None

    def head(self, batch: Batch, normalizer: float) -> StepLoss:
        return StepLoss(self, batch, normalizer)
