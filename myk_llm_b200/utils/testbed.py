"""Shared machinery of the small single-GPU research testbeds (:mod:`myk_llm_b200.arith`,
:mod:`myk_llm_b200.lc`): packing generated examples into training rows, and the training
loop around a model, an objective and periodic evaluations.

Packing.  Each example is one document of ``(ids, targets)`` (targets already shifted:
``targets[i]`` is the token after ``ids[i]`` where supervised, else ``IGNORE_INDEX``).
Rows of ``row_len`` tokens take examples in order; an example that does not fit starts
the next row, and the unused tail of a row is padding in a document of its own, never
supervised.  Rows go straight into a pinned host batch (``RowPacker``), so the copy to the
GPU is one asynchronous transfer.  ``PackedExamples`` runs this inside DataLoader workers,
each with its own deterministic random stream.

Training (``TestbedLoop``): AdamW / Muon from ``build_optimizers``, the schedule's learning
rate per step, bf16 autocast, the objective's normalised loss, gradient clipping, a
metrics line every ``log_interval`` steps and an evaluation callback every
``eval_interval`` steps.
"""

from __future__ import annotations

import contextlib
import time
from dataclasses import dataclass
from typing import Any, Callable, Iterator

import numpy as np
import torch
from torch.utils.data import DataLoader, IterableDataset, get_worker_info

from .. import ops
from ..data.config import IGNORE_INDEX, Batch, RowPacker

Example = tuple[np.ndarray, np.ndarray]  # (ids, shifted targets), int64 each


def pack_rows(examples: Iterator[Example], row_len: int, pad_id: int) -> Iterator[tuple[np.ndarray, np.ndarray,
                                                                                        list[int]]]:
    """Endless (ids, targets, document lengths) rows of ``row_len`` tokens."""
    pending: Example | None = None
    while True:
        ids = np.full(row_len, pad_id, dtype=np.int64)
        tgt = np.full(row_len, IGNORE_INDEX, dtype=np.int64)
        lengths: list[int] = []
        fill = 0
        while True:
            ex = pending if pending is not None else next(examples)
            pending = None
            n = len(ex[0])
            if n > row_len:
                raise ValueError(f"an example of {n} tokens exceeds the row length {row_len}")
            if fill + n > row_len:
                pending = ex
                break
            ids[fill:fill + n], tgt[fill:fill + n] = ex
            lengths.append(n)
            fill += n
        if fill < row_len:
            lengths.append(row_len - fill)
        yield ids, tgt, lengths


class PackedExamples(IterableDataset):
    """Batches of packed rows from ``make_examples(rng)`` (an endless example iterator);
    worker ``w`` of the DataLoader draws from ``numpy.random.default_rng([seed, w])``."""

    def __init__(self, make_examples: Callable[[np.random.Generator], Iterator[Example]], rows: int, row_len: int,
                 pad_id: int, seed: int) -> None:
        super().__init__()
        self.make_examples, self.rows, self.row_len, self.pad_id, self.seed = make_examples, rows, row_len, pad_id, seed

    def __iter__(self) -> Iterator[Batch]:
        info = get_worker_info()
        rng = np.random.default_rng([self.seed, info.id if info is not None else 0])
        source = pack_rows(self.make_examples(rng), self.row_len, self.pad_id)
        while True:
            packer = RowPacker(self.rows, self.row_len, pin=info is None and torch.cuda.is_available())
            for r in range(self.rows):
                ids, tgt, lengths = next(source)
                packer.view[0, r], packer.view[1, r] = ids, tgt
                packer.seqlens.append(torch.tensor(lengths, dtype=torch.int32))
            packer.masked = True
            yield packer.batch()


def packed_loader(dataset: PackedExamples, num_workers: int) -> DataLoader:
    return DataLoader(dataset, batch_size=None, num_workers=num_workers, pin_memory=torch.cuda.is_available(),
                      persistent_workers=num_workers > 0, prefetch_factor=8 if num_workers > 0 else None)


def autocast_for(device: torch.device):
    return torch.autocast("cuda", dtype=torch.bfloat16) if device.type == "cuda" else contextlib.nullcontext()


@dataclass
class LoopSettings:
    steps: int
    log_interval: int
    eval_interval: int
    grad_clip: float
    run_name: str


class TestbedLoop:
    """The training loop shared by the testbeds.  ``forward(batch, head)`` runs the model
    with the objective head; ``evaluate(step)`` is called every ``eval_interval`` steps
    (not at the last, which the caller evaluates with more examples)."""

    def __init__(self, settings: LoopSettings, model: torch.nn.Module, optimizers, schedule, objective,
                 forward: Callable[[Batch, Any], Any], metrics, device: torch.device) -> None:
        from ..train.optim import lr_multiplier

        self.s, self.model, self.optimizers, self.objective = settings, model, optimizers, objective
        self.forward, self.metrics, self.device = forward, metrics, device
        self.base_lrs = [[g["lr"] for g in o.param_groups] for o in optimizers]
        self.lr_at = lambda step: lr_multiplier(step, settings.steps, schedule)
        self.started = time.perf_counter()

    def _update(self, step: int, batch: Batch) -> tuple[float, int]:
        from ..train.optim import set_lr

        set_lr(self.optimizers, self.base_lrs, self.lr_at(step))
        targets = batch.num_targets
        with autocast_for(self.device):
            out = self.forward(batch, self.objective.head(batch, float(max(1, targets))))
        out.loss.backward()
        torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.s.grad_clip or float("inf"))
        for opt in self.optimizers:
            opt.step()
            opt.zero_grad(set_to_none=True)
        ops.invalidate_weight_cache()
        return float(out.sums["ce"]), targets

    def run(self, batches: Iterator[Batch], evaluate: Callable[[int], None] | None = None) -> None:
        window_t, loss, count = time.perf_counter(), 0.0, 0
        for step in range(1, self.s.steps + 1):
            batch = next(batches).to(self.device)
            ce, n = self._update(step, batch)
            loss, count = loss + ce, count + n
            if step % self.s.log_interval == 0:
                rate = self.s.log_interval * batch.input_ids.numel() / (time.perf_counter() - window_t)
                rec = {"train/loss": loss / max(1, count), "perf/tokens_per_s": rate}
                self.metrics.log(step, rec)
                print(f"[{self.s.run_name}] step {step} loss {rec['train/loss']:.4f} {rate:,.0f} tok/s", flush=True)
                window_t, loss, count = time.perf_counter(), 0.0, 0
            if evaluate is not None and self.s.eval_interval and step % self.s.eval_interval == 0 \
                    and step != self.s.steps:
                evaluate(step)
                window_t = time.perf_counter()

    @property
    def minutes(self) -> float:
        return (time.perf_counter() - self.started) / 60
