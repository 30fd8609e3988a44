"""Training objectives: next-token cross entropy (+ z-loss), multi-token prediction and
logit distillation, run as the model's ``head`` callback inside forward.

All losses are divided by one normaliser, the number of supervised next-token targets
of the whole optimizer step (all micro-batches, all ranks), so gradient accumulation and
data parallelism give the exact per-token mean (reference:
``src/myk_llm/train/objectives.py:83-117``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable

import numpy as np
import torch
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from .. import ops
from ..data.config import IGNORE_INDEX, Batch
from ..models import ModelOutput, MykLLM
from .config import DistillConfig, ObjectiveConfig


@dataclass
class LossOutput:
    loss: torch.Tensor
    sums: dict[str, torch.Tensor] = field(default_factory=dict)


def mtp_targets(targets: torch.Tensor, depth: int) -> torch.Tensor:
    """Position i predicts token i+1+depth; supervised only if every next-token target in
    between is supervised (no seam, no prompt)."""
    shifted = F.pad(targets[:, depth:], (0, depth), value=IGNORE_INDEX)
    valid = targets != IGNORE_INDEX
    for off in range(1, depth + 1):
        valid &= F.pad(targets[:, off:], (0, off), value=IGNORE_INDEX) != IGNORE_INDEX
    return torch.where(valid, shifted, IGNORE_INDEX)


class Teacher:
    """Frozen HuggingFace teacher whose output head is restricted to the student vocab."""

    def __init__(self, config: DistillConfig, device: torch.device) -> None:
        from transformers import AutoModelForCausalLM

        model = AutoModelForCausalLM.from_pretrained(config.teacher, dtype=torch.bfloat16).to(device).eval()
        model.requires_grad_(False)
        self.decoder = model.get_decoder()
        w = model.get_output_embeddings().weight
        if config.row_map:
            rm = torch.from_numpy(np.load(config.row_map).astype(np.int64)).to(device)
            w = w.index_select(0, rm)
        self.weight = w.detach()

    @torch.no_grad()
    def hidden(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.decoder(input_ids=input_ids).last_hidden_state


def distillation_kl_sum(hidden, weight, teacher_hidden, teacher_weight, valid, temperature: float, chunk_size: int):
    """Sum over valid tokens of T^2 KL(teacher || student), chunked and recomputed in
    backward so only O(chunk x vocab) logits are alive."""

    def chunk_kl(h, t, m):
        s = F.log_softmax(ops.linear(h, weight).float() / temperature, dim=-1)
        te = F.log_softmax((t @ teacher_weight.t()).float() / temperature, dim=-1)
        return ((te.exp() * (te - s)).sum(-1) * m).sum() * temperature ** 2

    total = hidden.new_zeros((), dtype=torch.float32)
    for a in range(0, hidden.size(0), chunk_size):
        b = a + chunk_size
        total = total + checkpoint(chunk_kl, hidden[a:b], teacher_hidden[a:b], valid[a:b], use_reentrant=False)
    return total


class Objective:
    def __init__(self, config: ObjectiveConfig, device: torch.device) -> None:
        self.config = config
        self.teacher = Teacher(config.distill, device) if config.distill.teacher else None

    def head(self, batch: Batch, normalizer: float) -> Callable[[MykLLM, ModelOutput], LossOutput]:
        cfg = self.config

        def run(model: MykLLM, out: ModelOutput) -> LossOutput:
            w = model.output_weight
            sums: dict[str, torch.Tensor] = {}
            ce_scale = 1.0 - cfg.distill.weight if self.teacher is not None else 1.0
            loss, sums["ce"], sums["z"] = ops.fused_linear_cross_entropy(
                out.hidden, w, batch.targets, normalizer / ce_scale, cfg.z_loss, chunk_size=_chunk(cfg, out.hidden))
            if self.teacher is not None:
                valid = (batch.targets != IGNORE_INDEX).reshape(-1).float()
                kl = distillation_kl_sum(out.hidden.reshape(-1, out.hidden.size(-1)), w,
                                         self.teacher.hidden(batch.input_ids).reshape(valid.numel(), -1),
                                         self.teacher.weight, valid, cfg.distill.temperature, cfg.distill.chunk_size)
                loss = loss + cfg.distill.weight * kl / normalizer
                sums["kl"] = kl.detach()
            mtp = model.mtp_hidden(out, batch.input_ids) if cfg.mtp_weight > 0 else []
            for depth, h in enumerate(mtp, start=1):
                l_, sums[f"mtp{depth}_ce"], _ = ops.fused_linear_cross_entropy(
                    h, w, mtp_targets(batch.targets, depth), normalizer / cfg.mtp_weight,
                    chunk_size=_chunk(cfg, h))
                loss = loss + l_
            return LossOutput(loss, sums)

        return run


def _chunk(cfg: ObjectiveConfig, h: torch.Tensor) -> int:
    # On B200 a larger chunk keeps the logits GEMMs at full tile occupancy; the chunk only
    # bounds the transient logits buffer (chunk x vocab bf16).
    return max(cfg.loss_chunk_size, 8192) if h.is_cuda else cfg.loss_chunk_size
