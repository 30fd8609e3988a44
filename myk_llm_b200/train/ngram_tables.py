"""Hashed n-gram tables trained with lazy (sparse) Adam, on the GPU or in host memory.

A step looks up only a small fraction of the tables (a few hundred thousand distinct rows
whatever the bucket count), so ``optimizer.ngram.update: lazy`` updates only those rows:

1. ``begin_step`` takes the distinct row ids of the step's micro-batches, brings those
   rows up to date (``catch_up``) and gathers their weights into one compact leaf tensor
   that the forward reads (its gradient is compact too and enters the global clip);
2. ``step`` applies AdamW to the touched rows with their compact gradients, in place in
   the tables, and stamps the rows' last-update step.

Rows a step does not touch keep their weights and moments (LazyAdam; bias correction by
the global step count).  ``catch_up`` restores what dense AdamW would have done with zero
gradients: a row last updated at step s and touched again at step t first receives the
t - 1 - s skipped updates in closed form (momentum drift, moment decay, weight decay),
exact except for eps, bias correction and a learning rate that changed inside the gap.

On CUDA both phases are single kernels (``csrc/ngram.cu``) that read and write the table
rows in place, without compact copies of the moments.  ``placement: host`` keeps weights,
moments and last-update steps in pinned host memory and runs the same kernels on the
rows through their mapped device addresses, so only the touched rows cross the host
link and the result equals ``placement: gpu`` exactly; ``prefetch`` is accepted for
config compatibility (the kernels stream the rows on demand).

Behaviour follows the reference's ``src/myk_llm/train/ngram_tables.py:86-411``
(begin_step / rows_for / step / catch_up / state_dict / export_weights), with the same
checkpoint file (``ngram_tables.pt``: weight, exp_avg, exp_avg_sq, last_step, step).
"""

from __future__ import annotations

import math
from pathlib import Path
from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..models.embeddings import NgramEmbedding
from .config import NgramOptimConfig

STATE_NAMES = ("weight", "exp_avg", "exp_avg_sq", "last_step")


class SparseNgramTables:
    """Owns the n-gram tables of ``module`` (stacked as (orders x buckets, dim)), their Adam
    state and the current step's staged rows.  The module's own table parameters become
    empty placeholders and its lookups go through ``row_source``.  Construct while the
    model is still on the CPU so that host-placed tables never reach the GPU."""

    def __init__(self, module: NgramEmbedding, config: NgramOptimConfig, lr: float, betas: tuple[float, float],
                 eps: float, device: torch.device, max_rows_per_step: int) -> None:
        if config.update != "lazy":
            raise ValueError("SparseNgramTables implements optimizer.ngram.update=lazy")
        self.module, self.config, self.device = module, config, torch.device(device)
        self.host = config.placement == "host"
        self.rowwise = config.second_moment == "rowwise"
        self.lr, self.betas, self.eps = lr * config.lr_scale, (float(betas[0]), float(betas[1])), eps
        self.lr_multiplier = 1.0
        self.num_buckets, self.num_orders = module.num_buckets, len(module.tables)
        self.dim = module.tables[0].embedding_dim
        self.max_rows = max_rows_per_step
        rows = self.num_orders * self.num_buckets
        pin = self.host and self.device.type == "cuda"
        store = torch.device("cpu") if self.host else self.device

        def make(*shape, dtype=torch.float32, zero=True):
            t = torch.empty(*shape, dtype=dtype, device=store, pin_memory=pin)
            return t.zero_() if zero else t

        weight = make(rows, self.dim, zero=False)
        for k, table in enumerate(module.tables):  # copy table by table, freeing each
            weight[k * self.num_buckets:(k + 1) * self.num_buckets].copy_(table.weight.detach())
            table.weight = nn.Parameter(torch.empty(0, self.dim), requires_grad=False)
        self.state = [weight, make(rows, self.dim), make(rows) if self.rowwise else make(rows, self.dim),
                      make(rows, dtype=torch.int32)]
        self.step_count = 0
        module.row_source = self.rows_for
        self._ids: torch.Tensor | None = None
        self._leaf: torch.Tensor | None = None
        self._stats = self._zero_stats()

    # -- views ---------------------------------------------------------------------------
    @property
    def weight(self) -> torch.Tensor:
        return self.state[0]

    @property
    def exp_avg(self) -> torch.Tensor:
        return self.state[1]

    @property
    def exp_avg_sq(self) -> torch.Tensor:
        return self.state[2]

    def num_parameters(self) -> int:
        return self.weight.numel()

    def state_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.state)

    def _hyper(self, step: int) -> tuple:
        lr = self.lr * self.lr_multiplier
        return (step, lr, self.config.weight_decay, self.betas[0], self.betas[1], self.eps, self.rowwise)

    @property
    def _cuda(self) -> bool:
        return self.device.type == "cuda"

    # -- the training step -----------------------------------------------------------------
    def _unique_ids(self, input_ids: list[torch.Tensor]) -> torch.Tensor:
        ids = torch.cat([self.module.row_ids(x.to(self.device, non_blocking=True)).flatten() for x in input_ids])
        return torch.unique(ids)  # sorted

    def begin_step(self, input_ids: list[torch.Tensor], next_input_ids: list[torch.Tensor] | None = None) -> None:
        """Stage the rows of this optimizer step's micro-batches (``input_ids``)."""
        if self._ids is not None:
            raise RuntimeError("begin_step called twice without step()")
        ids = self._unique_ids(input_ids)
        rows = self._stage(ids, self.step_count + 1, catch_up=self.config.catch_up, write_back=True)
        self._ids = ids
        self._leaf = rows.detach().requires_grad_()
        self._stats["steps_staged"] += 1
        self._stats["rows"] += ids.numel()

    def parameters(self) -> list[torch.Tensor]:
        """The current step's compact rows (for gradient clipping)."""
        return [self._leaf] if self._leaf is not None else []

    def rows_for(self, ids: torch.Tensor) -> torch.Tensor:
        """Summed rows (batch, seq_len, dim) of row ids (orders, batch, seq_len)."""
        if self._ids is not None and torch.is_grad_enabled():
            return F.embedding(torch.searchsorted(self._ids, ids), self._leaf).sum(0)
        if self._ids is not None:
            raise RuntimeError("no-grad forward between begin_step and step")
        unique, inverse = torch.unique(ids, return_inverse=True)
        rows = self._stage(unique.to(self.device), self.step_count + 1, catch_up=self.config.catch_up,
                           write_back=False)
        return F.embedding(inverse.to(self.device), rows).sum(0)

    def set_lr_multiplier(self, multiplier: float) -> None:
        self.lr_multiplier = multiplier

    @torch.no_grad()
    def step(self) -> None:
        """AdamW on the staged rows, in place in the tables."""
        ids, leaf = self._ids, self._leaf
        if ids is None or leaf is None:
            raise RuntimeError("step() without begin_step()")
        self._ids = self._leaf = None
        self.step_count += 1
        self._stats["steps"] += 1
        grad = leaf.grad
        if grad is None:
            self._stamp(ids)
            return
        if self._cuda:
            from ..ops import ext

            ext().ngram_adam(ids, grad.float().contiguous(), *self.state, *self._hyper(self.step_count))
        else:
            self._adam_torch(ids, grad.float())

    # -- CUDA / torch implementations ------------------------------------------------------
    def _stage(self, ids: torch.Tensor, step: int, catch_up: bool, write_back: bool) -> torch.Tensor:
        if self._cuda:
            from ..ops import ext

            return ext().ngram_stage(ids, *self.state, *self._hyper(step), catch_up, write_back)
        w, m, v, last = (t.index_select(0, ids) for t in self.state)
        if catch_up and step > 1:
            self._catch_up_torch(w, m, v, last, step)
            if write_back:
                for dst, src in zip(self.state[:3], (w, m, v)):
                    dst.index_copy_(0, ids, src)
        return w

    def _stamp(self, ids: torch.Tensor) -> None:
        last = self.state[3]
        if last.device == ids.device:
            last.index_fill_(0, ids, self.step_count)
        else:
            last.index_fill_(0, ids.to(last.device), self.step_count)

    def _catch_up_torch(self, w, m, v, last, step: int) -> None:
        b1, b2 = self.betas
        lr = self.lr * self.lr_multiplier
        decay = 1 - lr * self.config.weight_decay
        k = (step - 1 - last.long()).clamp(min=0).float()
        q = b1 / math.sqrt(b2) / decay
        drift = q * (1 - torch.pow(torch.tensor(q), k)) / (1 - q)
        bias = math.sqrt(1 - b2 ** (step - 1)) / (1 - b1 ** (step - 1))
        second = v[:, None] if self.rowwise else v
        w.sub_(m * (drift * lr * bias)[:, None] / (second.sqrt() + self.eps))
        if self.config.weight_decay:
            w.mul_(torch.pow(torch.tensor(decay), k)[:, None])
        m.mul_(torch.pow(torch.tensor(b1), k)[:, None])
        d2 = torch.pow(torch.tensor(b2), k)
        v.mul_(d2 if self.rowwise else d2[:, None])

    def _adam_torch(self, ids: torch.Tensor, grad: torch.Tensor) -> None:
        b1, b2 = self.betas
        lr = self.lr * self.lr_multiplier
        w, m, v = (t.index_select(0, ids) for t in self.state[:3])
        w.mul_(1 - lr * self.config.weight_decay)
        m.add_(grad - m, alpha=1 - b1)
        if self.rowwise:
            v.mul_(b2).add_(grad.square().mean(1), alpha=1 - b2)
            second = v[:, None]
        else:
            v.mul_(b2).add_(grad * grad, alpha=1 - b2)
            second = v
        bias1 = 1 - b1 ** self.step_count
        sb2 = math.sqrt(1 - b2 ** self.step_count)
        w.sub_(lr / bias1 * m / (second.sqrt() / sb2 + self.eps))
        for dst, src in zip(self.state[:3], (w, m, v)):
            dst.index_copy_(0, ids, src)
        self._stamp(ids)

    # -- logging, checkpoints, export ------------------------------------------------------
    @staticmethod
    def _zero_stats() -> dict[str, float]:
        return {"steps": 0, "steps_staged": 0, "rows": 0}

    def pop_stats(self) -> dict[str, float]:
        stats, steps = self._stats, max(1, self._stats["steps_staged"])
        self._stats = self._zero_stats()
        return {"ngram/rows_per_step": stats["rows"] / steps}

    def flush(self) -> None:
        if self._cuda:
            torch.cuda.current_stream(self.device).synchronize()

    def state_dict(self) -> dict[str, Any]:
        self.flush()
        return {**dict(zip(STATE_NAMES, self.state)), "step": self.step_count}

    def load_state_dict(self, state: dict[str, Any], load_optimizer: bool = True) -> None:
        self.flush()
        self._ids = self._leaf = None
        self.weight.copy_(state["weight"])
        if load_optimizer:
            for name, tensor in zip(STATE_NAMES[1:], self.state[1:]):
                tensor.copy_(state[name])
            self.step_count = int(state["step"])

    def save(self, directory: Path) -> None:
        torch.save(self.state_dict(), Path(directory) / "ngram_tables.pt")

    def load(self, directory: Path, load_optimizer: bool = True) -> None:
        path = Path(directory) / "ngram_tables.pt"
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: checkpoint was not trained with optimizer.ngram.update=lazy")
        self.load_state_dict(torch.load(path, map_location="cpu", mmap=True, weights_only=True), load_optimizer)

    def export_weights(self, chunk_rows: int = 1 << 20) -> dict[str, torch.Tensor]:
        """The tables (caught up when ``catch_up``) under the model's own parameter names, on
        the CPU (for model.safetensors)."""
        self.flush()
        rows = self.weight.size(0)
        if self.config.catch_up:
            parts = []
            for start in range(0, rows, chunk_rows):
                ids = torch.arange(start, min(start + chunk_rows, rows), device=self.device)
                parts.append(self._stage(ids, self.step_count + 1, catch_up=True, write_back=False).cpu())
            weight = torch.cat(parts)
        else:
            weight = self.weight.cpu()
        nb = self.num_buckets
        return {f"embed.ngram.tables.{k}.weight": weight[k * nb:(k + 1) * nb].clone() for k in range(self.num_orders)}

    def close(self) -> None:
        self.flush()
